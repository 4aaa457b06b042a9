// Split-KV decode across GPUs with a peer-memory exchange instead of a collective.
//
// One long stream's cache is sharded by position over the ranks of one node (config 5b: the 27B
// hybrid's gated head_dim-256 attention at 131072 positions).  Every step each rank computes the
// (unnormalised o, m, l) rows of its slice; they have to reach every rank, which then merges them
// by log-sum-exp and applies the sigmoid gate.  Instead of an NCCL all-gather between two kernels:
//
//   exchange      one kernel, one CTA per row: this rank's split-KV partials of the row are merged
//                 (log-sum-exp over its own splits) and the result is stored straight into every
//                 rank's gather buffer over NVLink (plain peer stores; no TMA, no multicast); the
//                 row's arrival counter on every rank is incremented (system-scope release); then
//                 the CTA waits (bounded spin: lane r polls rank r's counter with relaxed
//                 system-scope loads, then one acquire fence) until every rank's counter for the
//                 row reaches the step number, merges the nranks rows, applies the gate and writes
//                 the output; the last CTA to finish advances this rank's step counter.
// It is the default step after either decode kernel (a separate push and merge kernel pair cost
// one more kernel boundary, ~2.5 us per step at 2 GPUs).  The tensor-core decode kernel can
// instead do all of it in its epilogue (the last CTA of each (sequence, kv head) group, found with
// a per-group ticket; opt-in with BGATTN_PEER_FUSED=1), which measured slower at 2 GPUs.
//
// The gather buffers are double-buffered by step parity: rank r can write step e+2 into a peer
// only after its own exchange kernel of step e+1 finished, which needed that peer's step-e+1 rows,
// which the peer pushes only after its exchange of step e finished -- so a buffer is never
// overwritten while it is read.
// The step counter lives in device memory, so a captured CUDA graph replays correctly.
// A wait that runs out records BG_ETIMEOUT (bg_device_status) and the CTA writes zeros.
#include "attn.h"
#include "merge.cuh"
#include "tma.cuh"

namespace bg {
namespace {

#ifdef BG_TRACE
// Compile-time timing trace (-DBG_TRACE, never in the shipped build), %globaltimer ns of the last
// step, exchange CTA r: [r][0] entry (after its wait), [1] local merge done, [2] counters raised,
// [3] output written, [256 + r][0] every rank's row arrived.  Read with bg_ptrace_read.
__device__ unsigned long long g_ptrace[512][4];
__device__ __forceinline__ unsigned long long ptime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#endif

// One CTA per row: its 8 warps merge the `nsplit` local partials in one pass (warp w: splits w,
// w + 8, ..., (m, l, o) loaded in batches of 8 before any arithmetic, a running max per warp), the
// warp states meet in shared memory rescaled to the common max, and warp 0 stores the row into slot
// (parity, rank) of every rank's gather buffer, counts it on every rank, waits for every rank's
// row, merges them, gates and writes the output row.  Launched as a programmatic dependent of the
// decode kernel (griddepcontrol.wait before the first read of the partials).  nsplit == 0: this
// rank's slice is empty and it pushes an empty row.
template <int DPL>
__global__ void __launch_bounds__(256) lse_exchange_kernel(const float *__restrict__ part, uint32_t nsplit, PeerArgs x,
                                                           const float *__restrict__ gate, void *out, int out_f16) {
  constexpr uint32_t D = DPL * 32;
  __shared__ float red[8][D];
  __shared__ float lsum[8];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t rows = x.rows, row = blockIdx.x;
  asm volatile("griddepcontrol.wait;" ::: "memory");
#ifdef BG_TRACE
  if (threadIdx.x == 0 && row < 256) g_ptrace[row][0] = ptime();
#endif
  const uint32_t e = *x.step + 1;
  const uint64_t stride = (uint64_t)rows * (D + 2);
  const float *base = part + (uint64_t)row * (D + 2);
  // one pass: each warp loads (m, l, o) of its splits in batches of 8 and keeps a running
  // (max, sum, o) of its own; the 8 warp states are rescaled to the common max in shared memory
  float acc[DPL], L = 0.f, Mw = -INFINITY;
#pragma unroll
  for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
  for (uint32_t s0 = warp; s0 < nsplit; s0 += 64) {
    float v[8][DPL], mv[8], lv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t sp = s0 + 8 * i;
      const bool in = sp < nsplit;
      const float *src = base + (uint64_t)(in ? sp : 0) * stride;
      lv[i] = in ? __ldcg(src + D + 1) : 0.f;
      mv[i] = in ? __ldcg(src + D) : 0.f;
#pragma unroll
      for (int j = 0; j < DPL; ++j) v[i][j] = in ? __ldcg(src + lane + 32 * j) : 0.f;
    }
    float Mb = Mw;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (lv[i] > 0.f) Mb = fmaxf(Mb, mv[i]);  // empty slots may hold any bits
    if (Mb != Mw) {
      const float c = Mw == -INFINITY ? 0.f : expf(Mw - Mb);
      L *= c;
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[j] *= c;
      Mw = Mb;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (lv[i] > 0.f) {
        const float f = expf(mv[i] - Mw);
        L = fmaf(lv[i], f, L);
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[j] = fmaf(v[i][j], f, acc[j]);
      }
    }
  }
  __shared__ float mws[8];
#pragma unroll
  for (int j = 0; j < DPL; ++j) red[warp][lane + 32 * j] = acc[j];
  if (lane == 0) {
    lsum[warp] = L;
    mws[warp] = Mw;
  }
  __syncthreads();
  if (warp != 0) return;
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < 8; ++w) M = fmaxf(M, mws[w]);
  L = 0.f;
#pragma unroll
  for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const float f = mws[w] == -INFINITY ? 0.f : expf(mws[w] - M);
    L = fmaf(lsum[w], f, L);
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[j] = fmaf(red[w][lane + 32 * j], f, acc[j]);
  }
#ifdef BG_TRACE
  if (lane == 0 && row < 256) g_ptrace[row][1] = ptime();
#endif
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
  __threadfence_system();  // the row, in every rank, before its counters
  __syncwarp();
  if (lane < x.nranks) atomicAdd_system(x.flags[lane] + (uint64_t)x.rank * rows + row, 1u);
#ifdef BG_TRACE
  if (lane == 0 && row < 256) g_ptrace[row][2] = ptime();
#endif
  // every rank's row of this step (rows written by peers: read past L1)
  const bool ok = peer_wait_row_warp(x, row, e, &g_device_error, lane);
#ifdef BG_TRACE
  if (lane == 0 && row < 256) g_ptrace[256 + row][0] = ptime();
#endif
  // one round trip: every rank's (m, l, o) of the row is loaded before any arithmetic
  M = -INFINITY;
  L = 0.f;
#pragma unroll
  for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
  if (ok) {
    const float *src0 = x.gather[x.rank] + ((uint64_t)(e & 1) * x.nranks * rows + row) * (D + 2);
    float mv[BG_MAX_PEERS], lv[BG_MAX_PEERS], v[BG_MAX_PEERS][DPL];
#pragma unroll
    for (int r = 0; r < BG_MAX_PEERS; ++r) {
      const bool in = r < (int)x.nranks;
      const float *src = src0 + (uint64_t)(in ? r : 0) * rows * (D + 2);
      lv[r] = in ? __ldcg(src + D + 1) : 0.f;
      mv[r] = in ? __ldcg(src + D) : 0.f;
#pragma unroll
      for (int j = 0; j < DPL; ++j) v[r][j] = in ? __ldcg(src + lane + 32 * j) : 0.f;
    }
#pragma unroll
    for (int r = 0; r < BG_MAX_PEERS; ++r)
      if (lv[r] > 0.f) M = fmaxf(M, mv[r]);  // empty rows may hold any bits
#pragma unroll
    for (int r = 0; r < BG_MAX_PEERS; ++r) {
      if (lv[r] > 0.f) {
        const float f = expf(mv[r] - M);
        L = fmaf(lv[r], f, L);
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[j] = fmaf(v[r][j], f, acc[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < DPL; ++j) {
    const uint64_t i = (uint64_t)row * D + lane + 32 * j;
    float o = L > 0.f ? acc[j] / L : 0.f;  // a timed-out wait writes zeros
    if (gate) o = o / (1.0f + expf(-gate[i]));
    if (out_f16) static_cast<__half *>(out)[i] = __float2half_rn(o);
    else static_cast<float *>(out)[i] = o;
  }
#ifdef BG_TRACE
  if (lane == 0 && row < 256) g_ptrace[row][3] = ptime();
#endif
  if (lane == 0) {
    // every CTA has read the step before it counts itself done: the last one advances it
    __threadfence();
    if (atomicAdd(x.done, 1u) == gridDim.x - 1) {
      *x.done = 0;
      __threadfence();
      atomicAdd(x.step, 1u);
    }
  }
}

// 256-thread launch configuration with programmatic stream serialization (the kernel may be
// scheduled while the previous one in the stream finishes; it waits in griddepcontrol.wait)
void pdl_config(cudaLaunchConfig_t &cfg, cudaLaunchAttribute (&attr)[1], dim3 grid, cudaStream_t st) {
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
}

}  // namespace

PeerArgs peer_args(const bg_peer_exchange *x, uint32_t rows) {
  PeerArgs a;
  for (int i = 0; i < BG_MAX_PEERS; ++i) {
    a.gather[i] = i < (int)x->nranks ? x->gather[i] : nullptr;
    a.flags[i] = i < (int)x->nranks ? x->flags[i] : nullptr;
  }
  a.step = x->step;
  a.done = x->done;
  a.tickets = x->tickets;
  a.nranks = x->nranks;
  a.rank = x->rank;
  a.spin_limit = x->spin_limit ? x->spin_limit : (1u << 22);
  a.rows = rows;
  return a;
}

int launch_lse_exchange(const float *partials, uint32_t nsplit, uint32_t rows, uint32_t D, const bg_peer_exchange *x,
                        const float *gate, void *out, int out_f16, cudaStream_t st) {
  const PeerArgs a = peer_args(x, rows);
  if (rows == 0) return BG_OK;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  pdl_config(cfg, attr, dim3(rows), st);
  cudaError_t err;
  if (D == 64) err = cudaLaunchKernelEx(&cfg, lse_exchange_kernel<2>, partials, nsplit, a, gate, out, out_f16);
  else if (D == 128) err = cudaLaunchKernelEx(&cfg, lse_exchange_kernel<4>, partials, nsplit, a, gate, out, out_f16);
  else if (D == 256) err = cudaLaunchKernelEx(&cfg, lse_exchange_kernel<8>, partials, nsplit, a, gate, out, out_f16);
  else return BG_EUNSUPPORTED;
  return err == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int poll_device_error_peer() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return BG_ELAUNCH;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  return v;
}

}  // namespace bg

#ifdef BG_TRACE
extern "C" int bg_ptrace_read(unsigned long long *dst, size_t n) {
  return cudaMemcpyFromSymbol(dst, bg::g_ptrace, n * sizeof(unsigned long long)) == cudaSuccess ? 0 : -1;
}
#endif
