// Split-KV decode across GPUs with a peer-memory exchange instead of a collective.
//
// One long stream's cache is sharded by position over the ranks of one node (config 5b: the 27B
// hybrid's gated head_dim-256 attention at 131072 positions).  Every step each rank computes the
// (unnormalised o, m, l) rows of its slice; they have to reach every rank, which then merges them
// by log-sum-exp and applies the sigmoid gate.  Instead of an NCCL all-gather between two kernels:
//
//   push          this rank's split-KV partials are merged (log-sum-exp over its own splits) and
//                 each finished row is stored straight into every rank's gather buffer over NVLink
//                 (plain peer stores; no TMA, no multicast); then the row's arrival counter on
//                 every rank is incremented (system-scope release).
//   merge         for each row, wait (bounded spin, system-scope acquire) until every source's
//                 counter for the row reaches the step number, merge the nranks rows, apply the
//                 gate; the last CTA to finish advances this rank's step counter.
// These two kernels are the default step after either decode kernel.  The tensor-core decode
// kernel can instead do both in its epilogue (the last CTA of each (sequence, kv head) group,
// found with a per-group ticket, merges, pushes, waits and writes the output; opt-in with
// BGATTN_PEER_FUSED=1), which makes a step one launch but measured no faster at 2 GPUs.
//
// The gather buffers are double-buffered by step parity: rank r can write step e+2 into a peer
// only after its own merge of step e+1, which needed that peer's step-e+1 rows, which the peer
// pushes only after its merge of step e -- so a buffer is never overwritten while it is read.
// The step counter lives in device memory, so a captured CUDA graph replays correctly.
// A wait that runs out records BG_ETIMEOUT (bg_device_status) and the CTA writes zeros.
#include "attn.h"
#include "merge.cuh"
#include "tma.cuh"

namespace bg {
namespace {

// One CTA per row: its 8 warps merge the `nsplit` local partials (warp w: splits w, w + 8, ...,
// loaded in batches of 8 before any arithmetic), the partial sums meet in shared memory, and warp 0
// stores the row into slot (parity, rank) of every rank's gather buffer, then counts it on every
// rank.  Launched as a programmatic dependent of the decode kernel (griddepcontrol.wait before the
// first read of the partials).
template <int DPL>
__global__ void __launch_bounds__(256) lse_push_kernel(const float *__restrict__ part, uint32_t nsplit, PeerArgs x) {
  constexpr uint32_t D = DPL * 32;
  __shared__ float red[8][D];
  __shared__ float lsum[8];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t rows = x.rows, row = blockIdx.x;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const uint32_t e = *x.step + 1;
  const uint64_t stride = (uint64_t)rows * (D + 2);
  const float *base = part + (uint64_t)row * (D + 2);
  float M = -INFINITY;
  for (uint32_t s = lane; s < nsplit; s += 32) {
    const float l = __ldcg(base + s * stride + D + 1), m = __ldcg(base + s * stride + D);
    if (l > 0.f) M = fmaxf(M, m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float acc[DPL], L = 0.f;
#pragma unroll
  for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
  for (uint32_t s0 = warp; s0 < nsplit; s0 += 64) {
    float v[8][DPL], f[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t sp = s0 + 8 * i;
      const bool in = sp < nsplit;
      const float *src = base + (uint64_t)(in ? sp : 0) * stride;
      const float l = in ? __ldcg(src + D + 1) : 0.f, m = in ? __ldcg(src + D) : 0.f;
      f[i] = l > 0.f ? expf(m - M) : 0.f;  // empty slots may hold any bits
      L = fmaf(l > 0.f ? l : 0.f, f[i], L);
#pragma unroll
      for (int j = 0; j < DPL; ++j) v[i][j] = in ? __ldcg(src + lane + 32 * j) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (f[i] != 0.f)
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[j] = fmaf(v[i][j], f[i], acc[j]);
  }
#pragma unroll
  for (int j = 0; j < DPL; ++j) red[warp][lane + 32 * j] = acc[j];
  if (lane == 0) lsum[warp] = L;
  __syncthreads();
  if (warp != 0) return;
#pragma unroll
  for (int w = 1; w < 8; ++w)
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[j] += red[w][lane + 32 * j];
  L = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) L += lsum[w];
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
}

// One warp per row: wait for every rank's row of this step, merge, gate, write; the last CTA to
// finish advances the step.
template <int DPL>
__global__ void __launch_bounds__(256) lse_merge_peer_kernel(PeerArgs x, const float *__restrict__ gate, void *out,
                                                             int out_f16) {
  constexpr uint32_t D = DPL * 32;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t rows = x.rows, row = blockIdx.x * 8 + warp;
  // a programmatic dependent of the push kernel: nothing is read before that grid completed
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t e = *x.step + 1;
  if (row < rows) {
    int ok = 1;
    if (lane == 0) ok = peer_wait_row(x, row, e, &g_device_error);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    float acc[DPL], M = -INFINITY, L = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
    if (ok)  // rows written by peers: read past L1
      merge_rows<DPL, true>(x.gather[x.rank] + ((uint64_t)(e & 1) * x.nranks * rows + row) * (D + 2),
                            (uint64_t)rows * (D + 2), x.nranks, lane, acc, M, L);
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const uint64_t i = (uint64_t)row * D + lane + 32 * j;
      float o = L > 0.f ? acc[j] / L : 0.f;
      if (gate) o = o / (1.0f + expf(-gate[i]));
      if (out_f16) static_cast<__half *>(out)[i] = __float2half_rn(o);
      else static_cast<float *>(out)[i] = o;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
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

int launch_lse_push(const float *partials, uint32_t nsplit, uint32_t rows, uint32_t D, const bg_peer_exchange *x,
                    cudaStream_t st) {
  const PeerArgs a = peer_args(x, rows);
  if (rows == 0) return BG_OK;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  pdl_config(cfg, attr, dim3(rows), st);
  cudaError_t err;
  if (D == 64) err = cudaLaunchKernelEx(&cfg, lse_push_kernel<2>, partials, nsplit, a);
  else if (D == 128) err = cudaLaunchKernelEx(&cfg, lse_push_kernel<4>, partials, nsplit, a);
  else if (D == 256) err = cudaLaunchKernelEx(&cfg, lse_push_kernel<8>, partials, nsplit, a);
  else return BG_EUNSUPPORTED;
  return err == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int launch_lse_merge_peer(const bg_peer_exchange *x, uint32_t rows, uint32_t D, const float *gate, void *out,
                          int out_f16, cudaStream_t st) {
  const PeerArgs a = peer_args(x, rows);
  const uint32_t blocks = (rows + 7) / 8;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  pdl_config(cfg, attr, dim3(blocks), st);
  cudaError_t err;
  if (D == 64) err = cudaLaunchKernelEx(&cfg, lse_merge_peer_kernel<2>, a, gate, out, out_f16);
  else if (D == 128) err = cudaLaunchKernelEx(&cfg, lse_merge_peer_kernel<4>, a, gate, out, out_f16);
  else if (D == 256) err = cudaLaunchKernelEx(&cfg, lse_merge_peer_kernel<8>, a, gate, out, out_f16);
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
