// Split-KV decode across GPUs with a peer-memory exchange instead of a collective.
//
// One long stream's cache is sharded by position over the ranks of one node (config 5b: the 27B
// hybrid's gated head_dim-256 attention at 131072 positions).  Every step each rank computes the
// (unnormalised o, m, l) rows of its slice; they have to reach every rank, which then merges them
// by log-sum-exp and applies the sigmoid gate.  Instead of an NCCL all-gather between two kernels:
//
//   push kernel   merges this rank's split-KV partials (lse_merge over its own splits) and stores
//                 each finished row straight into every rank's gather buffer over NVLink (plain
//                 peer stores; no TMA, no multicast), then adds the number of rows it wrote to an
//                 arrival counter of each rank (system-scope release).
//   merge kernel  one thread per CTA waits (bounded spin, system-scope acquire) until every
//                 source's counter reaches step * rows, then the CTA merges the nranks rows and
//                 applies the gate; the last CTA to finish advances this rank's step counter.
//
// The gather buffers are double-buffered by step parity: rank r can write step e+2 into a peer
// only after its own merge of step e+1, which needed that peer's step-e+1 rows, which the peer
// pushes only after its merge of step e -- so a buffer is never overwritten while it is read.
// The step counter lives in device memory, so a captured CUDA graph replays correctly.
// A wait that runs out records BG_ETIMEOUT (bg_device_status) and the CTA writes zeros.
#include "attn.h"
#include "tma.cuh"

namespace bg {
namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct PushArgs {
  float *gather[BG_MAX_PEERS];
  uint32_t *flags[BG_MAX_PEERS];
  uint32_t nranks, rank;
  const uint32_t *step;
};

// Weighted sum over `n` rows of stride `stride` (one warp, lane owns DPL columns): returns the
// unnormalised o, the merged max M and sum L.  Each pass over 32 sources first loads every source's
// (m, l) lane-parallel and then its o values in batches of 8 before any arithmetic, so a warp waits
// for memory once per batch instead of once per source.
template <int DPL, bool CG>
__device__ __forceinline__ void merge_rows(const float *base, uint64_t stride, uint32_t n, uint32_t lane,
                                           float (&acc)[DPL], float &Mout, float &Lout) {
  constexpr uint32_t D = DPL * 32;
  auto ld = [](const float *p) { return CG ? __ldcg(p) : __ldg(p); };
  float M = -INFINITY;
  for (uint32_t s = lane; s < n; s += 32) {
    const float l = ld(base + s * stride + D + 1), m = ld(base + s * stride + D);
    M = l > 0.f ? fmaxf(M, m) : M;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float L = 0.f;
#pragma unroll
  for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
  for (uint32_t g0 = 0; g0 < n; g0 += 32) {
    const uint32_t s = g0 + lane;
    float f = 0.f;
    if (s < n) {
      const float l = ld(base + s * stride + D + 1);
      f = l > 0.f ? expf(ld(base + s * stride + D) - M) : 0.f;  // empty slots may hold any bits
      L = fmaf(l > 0.f ? l : 0.f, f, L);
    }
    const uint32_t cnt = min(32u, n - g0);
    for (uint32_t b0 = 0; b0 < cnt; b0 += 8) {
      float v[8][DPL];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < DPL; ++j)
          v[i][j] = b0 + i < cnt ? ld(base + (g0 + b0 + i) * stride + lane + 32 * j) : 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float fs = __shfl_sync(0xffffffffu, f, (b0 + i) & 31);
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[j] = fs != 0.f ? fmaf(v[i][j], fs, acc[j]) : acc[j];
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  Mout = M;
  Lout = L;
}

// Rows [8 block, 8 block + 8), one warp per row: merge `nsplit` local partials and store the result
// row into slot (parity, rank) of every rank's gather buffer.
template <int DPL>
__global__ void __launch_bounds__(256) lse_push_kernel(const float *__restrict__ part, uint32_t nsplit, uint32_t rows,
                                                       PushArgs x) {
  constexpr uint32_t D = DPL * 32;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t row = blockIdx.x * 8 + warp;
  const uint32_t e = *x.step + 1;
  if (row < rows) {
    float acc[DPL], M, L;
    merge_rows<DPL, false>(part + (uint64_t)row * (D + 2), (uint64_t)rows * (D + 2), nsplit, lane, acc, M, L);
    const uint64_t off = (((uint64_t)(e & 1) * x.nranks + x.rank) * rows + row) * (D + 2);
    for (uint32_t r = 0; r < x.nranks; ++r) {
      float *dst = x.gather[r] + off;
#pragma unroll
      for (int j = 0; j < DPL; ++j) dst[lane + 32 * j] = acc[j];
      if (lane == 0) {
        dst[D] = L > 0.f ? M : -INFINITY;
        dst[D + 1] = L;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t n = min(8u, rows - blockIdx.x * 8);  // rows this block wrote (grid covers rows)
    __threadfence_system();  // this block's rows, in every rank, before the counters
    for (uint32_t r = 0; r < x.nranks; ++r) atomicAdd_system(x.flags[r] + x.rank, n);
  }
}

template <int DPL>
__global__ void __launch_bounds__(256) lse_merge_peer_kernel(const float *gather, const uint32_t *flags,
                                                             uint32_t nranks, uint32_t rows, uint32_t *step,
                                                             uint32_t *done, uint32_t spin_limit,
                                                             const float *__restrict__ gate, void *out, int out_f16) {
  constexpr uint32_t D = DPL * 32;
  __shared__ uint32_t s_e;
  __shared__ int s_ok;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    const uint32_t e = *step + 1;
    const uint32_t target = e * rows;
    int ok = 1;
    for (uint32_t r = 0; r < nranks && ok; ++r) {
      uint32_t it = 0;
      // counters grow by `rows` per step; the signed difference survives wrap-around
      while ((int32_t)(ld_acquire_sys(flags + r) - target) < 0) {
        if (++it > spin_limit) {
          atomicExch(&g_device_error, BG_ETIMEOUT);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    s_e = e;
    s_ok = ok;
  }
  __syncthreads();
  const uint32_t row = blockIdx.x * 8 + warp;
  if (row < rows) {
    const uint32_t e = s_e;
    float acc[DPL], M = -INFINITY, L = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
    if (s_ok)  // rows written by peers: read past L1
      merge_rows<DPL, true>(gather + ((uint64_t)(e & 1) * nranks * rows + row) * (D + 2), (uint64_t)rows * (D + 2),
                            nranks, lane, acc, M, L);
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const uint64_t i = (uint64_t)row * D + lane + 32 * j;
      float o = L > 0.f ? acc[j] / L : 0.f;
      if (gate) o = o / (1.0f + expf(-gate[i]));
      if (out_f16) static_cast<__half *>(out)[i] = __float2half_rn(o);
      else static_cast<float *>(out)[i] = o;
    }
  }
  // the last CTA to finish advances the step (the next push / merge read it in stream order)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0;
      __threadfence();
      atomicAdd(step, 1u);
    }
  }
}

}  // namespace

int launch_lse_push(const float *partials, uint32_t nsplit, uint32_t rows, uint32_t D, const bg_peer_exchange *x,
                    cudaStream_t st) {
  PushArgs a;
  for (int i = 0; i < BG_MAX_PEERS; ++i) {
    a.gather[i] = i < (int)x->nranks ? x->gather[i] : nullptr;
    a.flags[i] = i < (int)x->nranks ? x->flags[i] : nullptr;
  }
  a.nranks = x->nranks;
  a.rank = x->rank;
  a.step = x->step;
  const uint32_t blocks = (rows + 7) / 8;
  if (D == 64) lse_push_kernel<2><<<blocks, 256, 0, st>>>(partials, nsplit, rows, a);
  else if (D == 128) lse_push_kernel<4><<<blocks, 256, 0, st>>>(partials, nsplit, rows, a);
  else if (D == 256) lse_push_kernel<8><<<blocks, 256, 0, st>>>(partials, nsplit, rows, a);
  else return BG_EUNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int launch_lse_merge_peer(const bg_peer_exchange *x, uint32_t rows, uint32_t D, const float *gate, void *out,
                          int out_f16, cudaStream_t st) {
  const float *g = x->gather[x->rank];
  const uint32_t *f = x->flags[x->rank];
  const uint32_t lim = x->spin_limit ? x->spin_limit : (1u << 22);
  const uint32_t blocks = (rows + 7) / 8;
  if (D == 64)
    lse_merge_peer_kernel<2><<<blocks, 256, 0, st>>>(g, f, x->nranks, rows, x->step, x->done, lim, gate, out, out_f16);
  else if (D == 128)
    lse_merge_peer_kernel<4><<<blocks, 256, 0, st>>>(g, f, x->nranks, rows, x->step, x->done, lim, gate, out, out_f16);
  else if (D == 256)
    lse_merge_peer_kernel<8><<<blocks, 256, 0, st>>>(g, f, x->nranks, rows, x->step, x->done, lim, gate, out, out_f16);
  else
    return BG_EUNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int poll_device_error_peer() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return BG_ELAUNCH;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  return v;
}

}  // namespace bg
