// Log-sum-exp merge of split-KV partial rows and the device view of the peer-memory exchange,
// shared by the merge / push kernels and the fused epilogue of the tensor-core decode kernel.
#pragma once
#include "common.cuh"

namespace bg {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Device view of a bg_peer_exchange: every rank's gather slots [2][nranks][rows][D+2] and per-row
// arrival counters [nranks][rows] (as addressed from this GPU), this rank's step / done counters and
// its per-group tickets.  nranks == 0: no exchange.
struct PeerArgs {
  float *gather[BG_MAX_PEERS];
  uint32_t *flags[BG_MAX_PEERS];
  uint32_t *step, *done, *tickets;
  uint32_t nranks, rank, spin_limit, rows;
};

// Bounded wait until every rank's counter for `row` reaches `target` (system-scope acquire).
// Returns false (and records BG_ETIMEOUT through `err`) when the limit runs out.
__device__ __forceinline__ bool peer_wait_row(const PeerArgs &x, uint32_t row, uint32_t target, int *err) {
  const uint32_t *f = x.flags[x.rank];
  for (uint32_t r = 0; r < x.nranks; ++r) {
    uint32_t it = 0;
    // counters grow by one per step; the signed difference survives wrap-around
    while ((int32_t)(ld_acquire_sys(f + (uint64_t)r * x.rows + row) - target) < 0) {
      if (++it > x.spin_limit) {
        atomicExch(err, BG_ETIMEOUT);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// Whole-warp form: lane r < nranks polls rank r's counter for `row` with relaxed system-scope loads,
// all ranks in parallel, and one acquire fence follows once every counter reached `target`.
// Returns the same value on every lane; false (BG_ETIMEOUT recorded) when a lane's limit ran out.
__device__ __forceinline__ bool peer_wait_row_warp(const PeerArgs &x, uint32_t row, uint32_t target, int *err,
                                                   uint32_t lane) {
  bool ok = true;
  if (lane < x.nranks) {
    const uint32_t *f = x.flags[x.rank] + (uint64_t)lane * x.rows + row;
    uint32_t it = 0, v;
    for (;;) {
      asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if ((int32_t)(v - target) >= 0) break;  // counters grow by one per step (wrap-safe)
      if (++it > x.spin_limit) {
        atomicExch(err, BG_ETIMEOUT);
        ok = false;
        break;
      }
      __nanosleep(32);
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  return ok;
}

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

}  // namespace bg
