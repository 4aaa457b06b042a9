// Causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Path: layer() prefill / PLD verify (src/engine.ts:1580) with an f16 cache and f16 queries --
// query row qi at position posBase+qi attends cache positions 0..posBase+qi.  This is the only
// dense contraction of the attention path, so it runs as a flash-attention forward pass:
//
//   CTA = (head h, block of 256 query rows, sequence b); two 128-row query tiles (a, b) share
//   every K/V tile.  Warp roles (384 threads):
//     warp 0      TMA producer: Q tiles once, then K/V tiles of 128 positions through a 2-stage
//                 ring (4-D tiled loads of the [seq][pos][kv][D] cache, 128B swizzle, no multicast)
//     warp 1      MMA issuer (one thread): S_t = Q_t K^T into TMEM (SS form), then
//                 O_t += P_t V with P read straight from TMEM (TS form); completion is signalled
//                 with tcgen05.commit onto mbarriers
//     warp 2      TMEM allocator (512 columns: S_a, S_b, O_a, O_b; P_t aliases the first 64
//                 columns of S_t as packed f16 pairs)
//     warps 4-7   softmax of tile a, warps 8-11 softmax of tile b: one query row per thread,
//                 the whole 128-column score row read with tcgen05.ld into registers (one wait),
//                 online softmax in log2 units.  The running max used for the exponentials is
//                 raised lazily (only when a row's max grows by more than 2^8), so O is rescaled
//                 in TMEM rarely; P <= 256 stays well inside f16.
//   Epilogue: O / l from TMEM -> f16 (or f32) rows of out[b][q][h][:].
// All mbarrier waits are bounded; on expiry the CTA records BG_ETIMEOUT, stops issuing work, waits
// for what it already issued, frees its TMEM and exits.
#include <cuda.h>
#include <cuda_fp16.h>

#include "prefill.h"
#include "tma.cuh"

namespace bg {
namespace {

constexpr int kRows = 128;    // rows per query tile (UMMA M)
constexpr int kKeys = 128;    // positions per K/V tile (UMMA N of S, K of PV)
constexpr int kD = 128;       // head_dim handled by this kernel
constexpr int kTileBytes = kRows * kD * 2;  // one 128 x 128 f16 tile (two 128B column blocks)
constexpr int kStages = 2;
constexpr int kThreads = 384;
constexpr float kRescaleThreshold = 8.0f;   // log2 units

struct PfParams {
  void *out;
  int out_f16;
  uint32_t S, H, KV, G, posBase, Ltot;
  float sl2;
};

struct PfSmem {  // offsets from the 1024-aligned base
  static constexpr int Q = 0;                        // Q_a, Q_b
  static constexpr int KV = 2 * kTileBytes;          // stages: K then V
  static constexpr int BAR = KV + kStages * 2 * kTileBytes;
  static constexpr int TOTAL = BAR + 256;
};

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) /*sm100 descriptor*/ | (2ull << 61) /*SW128*/;
}

// kind::f16 instruction descriptor: f32 accumulate, f16 A/B, M=128, N=128.
constexpr uint32_t idesc_f16(bool b_mn_major) {
  return (1u << 4) | (b_mn_major ? (1u << 16) : 0u) | ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

#define BG_R32(r) r[0], r[1], r[2], r[3], r[4], r[5], r[6], r[7], r[8], r[9], r[10], r[11], r[12], r[13], r[14], r[15], \
                  r[16], r[17], r[18], r[19], r[20], r[21], r[22], r[23], r[24], r[25], r[26], r[27], r[28], r[29],  \
                  r[30], r[31]

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {  // MUFU exp2; exp2(-inf) = +0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {  // 3-input max (sm_100)
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, PfParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + PfSmem::BAR);
  uint64_t *kv_full = bars;            // [2]
  uint64_t *kv_empty = bars + 2;       // [2]
  uint64_t *q_full = bars + 4;         // [1]
  uint64_t *s_full = bars + 5;         // [2] per tile
  uint64_t *p_full = bars + 7;         // [2]
  uint64_t *o_done = bars + 9;         // [2]
  uint32_t *tmem_base_s = reinterpret_cast<uint32_t *>(bars + 12);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 13);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t h = blockIdx.x;
  const uint32_t qblk = gridDim.y - 1 - blockIdx.y;  // heaviest (latest) query blocks first
  const uint32_t b = blockIdx.z;
  const uint32_t kvh = h / p.G;
  const uint32_t q0 = qblk * 2 * kRows;
  const uint32_t last_key = min(p.posBase + q0 + 2 * kRows, p.Ltot);  // exclusive
  const int ntiles = (int)((last_key + kKeys - 1) / kKeys);

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(q_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {  // TMEM: 512 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_base_s)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  const uint32_t tS[2] = {tmem + 0, tmem + 128};
  const uint32_t tO[2] = {tmem + 256, tmem + 384};
  const uint32_t sQ = smem_u32(sm + PfSmem::Q);
  const uint32_t sKV = smem_u32(sm + PfSmem::KV);

  // Warpgroup 0 (producer, MMA issuer, TMEM owner) runs on 72 registers so the two softmax
  // warpgroups can hold a whole 128-column score row: 128*72 + 256*216 == 384*168 (launch).
  if (warp < 4) asm volatile("setmaxnreg.dec.sync.aligned.u32 72;" ::: "memory");
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_expect_tx(q_full, 2 * kTileBytes);
      for (int t = 0; t < 2; ++t)
        for (int cb = 0; cb < 2; ++cb)
          tma_load_4d(sm + PfSmem::Q + t * kTileBytes + cb * kRows * 128, &tmQ, q_full, cb * 64, (int)h,
                      (int)(q0 + t * kRows), (int)b);
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        if (j >= kStages && !mbar_wait(&kv_empty[st], ((j >> 1) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        unsigned char *kd = sm + PfSmem::KV + st * 2 * kTileBytes;
        mbar_expect_tx(&kv_full[st], 2 * kTileBytes);
        for (int cb = 0; cb < 2; ++cb) {
          tma_load_4d(kd + cb * kKeys * 128, &tmK, &kv_full[st], cb * 64, (int)kvh, j * kKeys, (int)b);
          tma_load_4d(kd + kTileBytes + cb * kKeys * 128, &tmV, &kv_full[st], cb * 64, (int)kvh, j * kKeys, (int)b);
        }
        issued = j + 1;
      }
      // no bulk copy may still be in flight when the CTA exits
      mbar_wait(q_full, 0);
      for (int j = max(0, issued - kStages); j < issued; ++j) mbar_wait(&kv_full[j & 1], (j >> 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // Order per KV tile j:  PV_a(j), S_a(j+1), PV_b(j), S_b(j+1).  S_t(j+1) overwrites the
    // columns PV_t(j) reads P_t(j) from; MMAs issued by one thread execute in order, so it is
    // queued right behind it and the tensor pipe never drains while a softmax runs.  The
    // tcgen05.commit after S_t(j+1) fires only once every earlier MMA (PV_t(j) included) is done,
    // which is what lets the softmax warps touch O_t and P_t after waiting on s_full.
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16(false), idO = idesc_f16(true);
      auto issue_s = [&](int t, uint32_t sK) {
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
          const uint64_t a = umma_desc_sw128(sQ + t * kTileBytes + off, 16, 1024);
          const uint64_t bk = umma_desc_sw128(sK + off, 16, 1024);
          umma_ss(tS[t], a, bk, idS, kk > 0);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, uint32_t sV, int j) {
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          const uint64_t bv = umma_desc_sw128(sV + kk * 16 * 128, kKeys * 128, 1024);
          umma_ts(tO[t], tS[t] + kk * 8, bv, idO, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[t]);
      };
      bool ok = mbar_wait(q_full, 0) && mbar_wait(&kv_full[0], 0);
      tc_fence_after();
      int j = 0;
      if (ok && ntiles > 0) {
        issue_s(0, sKV);
        issue_s(1, sKV);
      }
      for (; ok && j < ntiles; ++j) {
        const int st = j & 1;
        const uint32_t sV = sKV + st * 2 * kTileBytes + kTileBytes;
        const uint32_t sKn = sKV + (st ^ 1) * 2 * kTileBytes;
        const bool more = j + 1 < ntiles;
        if (!mbar_wait(&p_full[0], j & 1)) { ok = false; break; }
        tc_fence_after();
        issue_pv(0, sV, j);
        if (more) {
          if (!mbar_wait(&kv_full[st ^ 1], ((j + 1) >> 1) & 1)) { ok = false; break; }
          tc_fence_after();
          issue_s(0, sKn);
        }
        if (!mbar_wait(&p_full[1], j & 1)) { ok = false; break; }
        tc_fence_after();
        issue_pv(1, sV, j);
        umma_commit(&kv_empty[st]);  // K_j and V_j are free once everything so far has completed
        if (more) issue_s(1, sKn);
      }
      if (!ok) *abort_flag = 1;
      // every MMA this thread issued must complete before the CTA frees TMEM
      if (ntiles > 0)
        for (int t = 0; t < 2; ++t) mbar_wait(&o_done[t], (max(j, 1) - 1) & 1);
    }
  } else if (warp >= 4) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 216;" ::: "memory");
    // ---------------- softmax (one query row per thread) ----------------
    const int t = (warp - 4) >> 2;                 // query tile
    const int row = ((warp & 3) << 5) + lane;      // TMEM lane == tile row
    const uint32_t lane_off = (uint32_t)((warp & 3) << 5) << 16;
    const uint32_t qrow = q0 + t * kRows + row;    // query index within S
    const uint32_t qpos = p.posBase + qrow;
    const float sl2 = p.sl2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (!mbar_wait_warp(&s_full[t], j & 1)) { ok = false; break; }
      tc_fence_after();
      const uint32_t sbase = tS[t] | lane_off;
      const int key0 = j * kKeys;
      // keys of this tile the row may attend: all of them except near the diagonal
      const int nvalid = min(kKeys, max(0, (int)qpos - key0 + 1));
      // the whole 128-column score row in registers: one TMEM wait per tile
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(sbase + c * 32, r[c]);
      tmem_wait_ld();
      const bool full_row = nvalid >= kKeys;
      if (!full_row) {  // keys past the diagonal: -inf scores (exp2 -> 0)
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i >= nvalid) r[c][i] = __float_as_uint(-INFINITY);
      }
      // eight independent max chains (8 deep each) instead of one 64 deep
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int k = (c * 16 + i / 2) & 7;
          mx8[k] = fmax3(mx8[k], __uint_as_float(r[c][i]), __uint_as_float(r[c][i + 1]));
        }
      const float mx = fmaxf(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], fmaxf(mx8[5], fmaxf(mx8[6], mx8[7]))));
      const float mt = mx * sl2;
      // lazy rescale; the TMEM round trip is .sync.aligned, so the branch is taken by the whole
      // warp when any of its rows moved, and rows that did not move use the factor 1
      const bool need = mt > m_used + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need)) {
        if (j > 0) {
          // PV_t(j-1) has completed: the commit we waited on (after S_t(j)) covers it.
          const float f = (need && m_used > -INFINITY) ? ex2_approx(m_used - mt) : 1.0f;
          const uint32_t obase = tO[t] | lane_off;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(obase + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            tmem_st32(obase + c * 32, o);
          }
          l *= f;
        }
        if (need) m_used = mt;
      }
      const float mneg = -m_used;
      // p = exp2(s*sl2 - m_used), packed f16 into the first 64 columns of S_t (masked scores hold
      // -inf -> 0).  Moving a share of these exponentials to the FMA pipe with a polynomial was
      // measured slower (one in eight: -3 %, one in four: -12 %): the softmax is bound by its
      // instruction count and latency more than by MUFU throughput.
      float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
      for (int c = 0; c < 4; c += 2) {
        uint32_t pk0[16], pk1[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(r[c][2 * i]), sl2, mneg));
          const float p1 = ex2_approx(fmaf(__uint_as_float(r[c][2 * i + 1]), sl2, mneg));
          const float p2 = ex2_approx(fmaf(__uint_as_float(r[c + 1][2 * i]), sl2, mneg));
          const float p3 = ex2_approx(fmaf(__uint_as_float(r[c + 1][2 * i + 1]), sl2, mneg));
          ls0 += p0 + p1;
          ls1 += p2 + p3;
          pk0[i] = pack_half2(p0, p1);
          pk1[i] = pack_half2(p2, p3);
        }
        tmem_st16(sbase + c * 16, pk0);
        tmem_st16(sbase + c * 16 + 16, pk1);
      }
      l += ls0 + ls1;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    // epilogue: wait for the last PV of this tile, then O / l -> out
    if (ok && ntiles > 0 && mbar_wait_warp(&o_done[t], (ntiles - 1) & 1)) {
      tc_fence_after();
      const uint32_t obase = tO[t] | lane_off;
      const float inv = 1.0f / l;
      const bool valid = qrow < p.S;
      const uint64_t orow = (((uint64_t)b * p.S + qrow) * p.H + h) * kD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(obase + c * 32, r);
        tmem_wait_ld();
        if (valid) {
          if (p.out_f16) {
            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + orow + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __half2 hv = __floats2half2_rn(__uint_as_float(r[v * 8 + 2 * e]) * inv,
                                               __uint_as_float(r[v * 8 + 2 * e + 1]) * inv);
                w[e] = *reinterpret_cast<uint32_t *>(&hv);
              }
              dst[v] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else {
            float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + orow + c * 32);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_float4(__uint_as_float(r[4 * v]) * inv, __uint_as_float(r[4 * v + 1]) * inv,
                                   __uint_as_float(r[4 * v + 2]) * inv, __uint_as_float(r[4 * v + 3]) * inv);
          }
        }
      }
    } else if (!ok) {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

}  // namespace

bool prefill_tc_supported(int mode, uint32_t D, uint32_t S, int q_f16, bool roll, bool ring) {
  return mode == BG_KV_F16 && D == kD && q_f16 && !roll && !ring && S >= 64;
}

int launch_prefill_tc(const PrefillArgs &a, cudaStream_t st) {
  CUtensorMap tq, tk, tv;
  {
    const uint64_t dims[4] = {kD, a.H, a.S, a.B};
    const uint64_t strides[3] = {kD * 2, (uint64_t)a.H * kD * 2, (uint64_t)a.S * a.H * kD * 2};
    const uint32_t box[4] = {64, 1, kRows, 1};
    if (make_tmap_4d(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return BG_EUNSUPPORTED;
  }
  {
    const uint64_t dims[4] = {kD, a.KV, a.Ltot, a.B};
    const uint64_t strides[3] = {kD * 2, (uint64_t)a.KV * kD * 2, a.seq_stride * a.KV * kD * 2};
    const uint32_t box[4] = {64, 1, kKeys, 1};
    if (make_tmap_4d(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.K, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return BG_EUNSUPPORTED;
    if (make_tmap_4d(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.V, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return BG_EUNSUPPORTED;
  }
  PfParams p;
  p.out = a.out;
  p.out_f16 = a.out_f16;
  p.S = a.S;
  p.H = a.H;
  p.KV = a.KV;
  p.G = a.H / a.KV;
  p.posBase = a.posBase;
  p.Ltot = a.Ltot;
  p.sl2 = a.scale * kLog2e;
  const int smem = PfSmem::TOTAL + 1024;
  if (cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return BG_ELAUNCH;
  dim3 grid(a.H, (a.S + 2 * kRows - 1) / (2 * kRows), a.B);
  prefill_tc_kernel<<<grid, kThreads, smem, st>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int poll_device_error_prefill() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return BG_ELAUNCH;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  return v;
}

}  // namespace bg
