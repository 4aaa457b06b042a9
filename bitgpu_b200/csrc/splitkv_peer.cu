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

// Rows [8 block, 8 block + 8), one warp per row: merge `nsplit` local partials, store the result
// row into slot (parity, rank) of every rank's gather buffer, then count the row on every rank.
template <int DPL>
__global__ void __launch_bounds__(256) lse_push_kernel(const float *__restrict__ part, uint32_t nsplit, PeerArgs x) {
  constexpr uint32_t D = DPL * 32;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t rows = x.rows, row = blockIdx.x * 8 + warp;
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
    __threadfence_system();  // the row, in every rank, before its counters
    __syncwarp();
    if (lane < x.nranks) atomicAdd_system(x.flags[lane] + (uint64_t)x.rank * rows + row, 1u);
  }
}

// One warp per row: wait for every rank's row of this step, merge, gate, write; the last CTA to
// finish advances the step.
template <int DPL>
__global__ void __launch_bounds__(256) lse_merge_peer_kernel(PeerArgs x, const float *__restrict__ gate, void *out,
                                                             int out_f16) {
  constexpr uint32_t D = DPL * 32;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t rows = x.rows, row = blockIdx.x * 8 + warp;
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
  const uint32_t blocks = (rows + 7) / 8;
  if (D == 64) lse_push_kernel<2><<<blocks, 256, 0, st>>>(partials, nsplit, a);
  else if (D == 128) lse_push_kernel<4><<<blocks, 256, 0, st>>>(partials, nsplit, a);
  else if (D == 256) lse_push_kernel<8><<<blocks, 256, 0, st>>>(partials, nsplit, a);
  else return BG_EUNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int launch_lse_merge_peer(const bg_peer_exchange *x, uint32_t rows, uint32_t D, const float *gate, void *out,
                          int out_f16, cudaStream_t st) {
  const PeerArgs a = peer_args(x, rows);
  const uint32_t blocks = (rows + 7) / 8;
  if (D == 64) lse_merge_peer_kernel<2><<<blocks, 256, 0, st>>>(a, gate, out, out_f16);
  else if (D == 128) lse_merge_peer_kernel<4><<<blocks, 256, 0, st>>>(a, gate, out, out_f16);
  else if (D == 256) lse_merge_peer_kernel<8><<<blocks, 256, 0, st>>>(a, gate, out, out_f16);
  else return BG_EUNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int poll_device_error_peer() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return BG_ELAUNCH;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  return v;
}

}  // namespace bg
