// Causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Path: layer() prefill / PLD verify (src/engine.ts:1580) and the hybrid's gated head_dim-256
// prefill segments (engine.ts:1487-1491): query row qi at position posBase+qi attends cache
// positions 0..posBase+qi.  The engine passes f32 queries (shaders/attention_sg_kv16.wgsl:10,
// attention_sg_kv8.wgsl:10) over an f16 or a q8 cache; f16 queries are accepted as well.  This is
// the only dense contraction of the attention path, so it runs as a flash-attention forward pass
// with both products on the tensor cores in kind::f16 (f32 accumulate):
//
//   head_dim 128: CTA = (head h, 256 query rows, sequence b); two 128-row query tiles (a, b) share
//                 every 128-position K/V tile.  TMEM: S_a, S_b, O_a, O_b (128 columns each).
//   head_dim 256: CTA = (head h, 128 query rows, sequence b); one query tile, 64-position K/V
//                 tiles, S double-buffered so S(j+1) runs on the tensor pipe during softmax(j).
//                 TMEM: S_0, S_1 (64 columns), O (256 columns).
//
//   Warp roles (384 threads):
//     warp 0      TMA producer (f16 cache): Q once (f16 queries), then K/V tiles through a
//                 2-stage ring (4-D tiled loads of the [seq][pos][kv][D] cache, 128B swizzle,
//                 no multicast)
//     warp 1      MMA issuer (one thread): S = Q K^T into TMEM (SS form), O += P V with P read
//                 straight from TMEM (TS form); completion signalled with tcgen05.commit
//     warp 2      TMEM allocator (512 columns)
//     warps 4-7   softmax of tile a (one query row per thread: the whole score row read with
//                 tcgen05.ld into registers, online softmax in log2 units, lazy rescale of O)
//     warps 8-11  softmax of tile b (head_dim 128)
//   q8 cache: the int8 codes and their 32-element block scales are dequantised into the same
//   swizzled f16 operand tiles by producer warps (0, 2, 3 for head_dim 128; 8-11 for head_dim 256)
//   with plain 16-byte loads, then handed to the MMA through the same mbarrier ring.
//   f32 queries: every thread converts a share of the Q tiles to f16 in shared memory at start.
//   Epilogue: O / l from TMEM, the sigmoid gate when given, f16 or f32 rows of out[b][q][h][:].
// All mbarrier waits are bounded; on expiry the CTA records BG_ETIMEOUT, stops issuing work, waits
// for what it already issued, frees its TMEM and exits.
#include <cuda.h>
#include <cuda_fp16.h>

#include "prefill.h"
#include "tma.cuh"
#include "umma.cuh"

namespace bg {
namespace {

constexpr int kRows = 128;    // rows per query tile (UMMA M)
constexpr int kStages = 2;
constexpr int kThreads = 384;
constexpr float kRescaleThreshold = 8.0f;   // log2 units

template <int D>
struct PfCfg {
  static constexpr int NQT = D == 128 ? 2 : 1;       // query tiles per CTA
  static constexpr int KT = D == 128 ? 128 : 64;     // positions per K/V tile
  static constexpr int QTILE = kRows * D * 2;        // bytes of one f16 query tile
  static constexpr int KTILE = KT * D * 2;           // bytes of one f16 K (or V) tile
  static constexpr int Q = 0;
  static constexpr int KVOFF = NQT * QTILE;
  static constexpr int BAR = KVOFF + kStages * 2 * KTILE;
  static constexpr int TOTAL = BAR + 256;
  // TMEM columns
  static constexpr uint32_t S0 = 0, S1 = D == 128 ? 128 : 64;
  static constexpr uint32_t O0 = 256, O1 = 384;       // O1 used by head_dim 128 only
  // q8 producer group
  static constexpr int NPW = D == 128 ? 3 : 4;        // producer warps
};

struct PfParams {
  void *out;
  int out_f16;
  const void *qsrc;       // queries staged by the threads (f32, or f16 over a q8 cache); nullptr: TMA
  int q_f32;
  const float *gate;      // [B][S][H][D] or nullptr
  const int8_t *Kc, *Vc;  // q8 codes
  const float *Ks, *Vs;   // q8 block scales
  uint64_t seq_stride;
  uint32_t S, H, KV, G, posBase, Ltot;
  float sl2;
};

// Byte offset of 16-byte chunk `ch` (8 f16 of one row) of row r in a 128B-swizzled K-major f16
// operand tile of R rows: column blocks of 64 elements, each R rows x 128 B.
template <int R>
__device__ __forceinline__ uint32_t sw128_off(int r, int ch) {
  return (uint32_t)((ch >> 3) * (R * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}


// 16 int8 codes with one block scale (s / 127 as f16x2) -> 16 f16 values code * s / 127.  The
// codes become exact f16 integers through the exponent trick: byte (c + 128) under the f16
// pattern 0x64xx is 1024 + c + 128, minus 1152 leaves c.
__device__ __forceinline__ void dequant16(uint4 w, __half2 sc, uint4 &o0, uint4 &o1) {
  const __half2 bias = __float2half2_rn(1152.0f);
  const uint32_t in[4] = {w.x, w.y, w.z, w.w};
  uint32_t out[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t b = in[i] ^ 0x80808080u;
    uint32_t lo = __byte_perm(b, 0x64646464u, 0x5140), hi = __byte_perm(b, 0x64646464u, 0x5342);
    __half2 l = __hmul2(__hsub2(*reinterpret_cast<__half2 *>(&lo), bias), sc);
    __half2 h = __hmul2(__hsub2(*reinterpret_cast<__half2 *>(&hi), bias), sc);
    out[2 * i] = *reinterpret_cast<uint32_t *>(&l);
    out[2 * i + 1] = *reinterpret_cast<uint32_t *>(&h);
  }
  o0 = make_uint4(out[0], out[1], out[2], out[3]);
  o1 = make_uint4(out[4], out[5], out[6], out[7]);
}

template <int D, bool KVQ8>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, PfParams p) {
  using C = PfCfg<D>;
  constexpr int NQT = C::NQT, KT = C::KT;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + C::BAR);
  uint64_t *kv_full = bars;            // [2] per stage
  uint64_t *kv_empty = bars + 2;       // [2]
  uint64_t *q_full = bars + 4;         // [1]
  uint64_t *s_full = bars + 5;         // [2] per S slot
  uint64_t *p_full = bars + 7;         // [2] per S slot
  uint64_t *o_done = bars + 9;         // [2] per O tile (head_dim 256: [0] only)
  uint64_t *mma_done = bars + 11;      // [1] every MMA of the CTA has completed
  uint32_t *tmem_base_s = reinterpret_cast<uint32_t *>(bars + 12);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 13);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t h = blockIdx.x;
  const uint32_t qblk = gridDim.y - 1 - blockIdx.y;  // heaviest (latest) query blocks first
  const uint32_t b = blockIdx.z;
  const uint32_t kvh = h / p.G;
  const uint32_t q0 = qblk * NQT * kRows;
  const uint32_t last_key = min(p.posBase + q0 + NQT * kRows, p.Ltot);  // exclusive
  const int ntiles = (int)((last_key + KT - 1) / KT);

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], KVQ8 ? C::NPW : 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {  // TMEM: 512 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_base_s)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (p.qsrc) {
    // queries staged by the threads: each converts (f32) or copies (f16) a share of the Q tiles
    // into the swizzled f16 operand layout; rows past S are zero
    constexpr int CPR = D / 8;  // 16-byte chunks per row
    for (int idx = tid; idx < NQT * kRows * CPR; idx += kThreads) {
      const int t = idx / (kRows * CPR), rem = idx % (kRows * CPR), r = rem / CPR, ch = rem % CPR;
      const uint32_t qrow = q0 + t * kRows + r;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (qrow < p.S) {
        const uint64_t e = (((uint64_t)b * p.S + qrow) * p.H + h) * D + ch * 8;
        if (p.q_f32) {
          const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(p.qsrc) + e);
          const float4 a = __ldg(src), c = __ldg(src + 1);
          v = make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(c.x, c.y), pack_half2(c.z, c.w));
        } else {
          v = __ldg(reinterpret_cast<const uint4 *>(static_cast<const __half *>(p.qsrc) + e));
        }
      }
      *reinterpret_cast<uint4 *>(sm + C::Q + t * C::QTILE + sw128_off<kRows>(r, ch)) = v;
    }
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  const uint32_t sQ = smem_u32(sm + C::Q);
  const uint32_t sKV = smem_u32(sm + C::KVOFF);

  // Warpgroup 0 (producer, MMA issuer, TMEM owner) runs on 72 registers so the two softmax
  // warpgroups can hold a whole score row: 128*72 + 256*216 == 384*168 (launch).
  // ---------------- q8 dequantising producer (gtid: thread index within the producer warps) ------
  auto q8_produce = [&](const int gtid) {
    constexpr int GS = C::NPW * 32;
    constexpr int CPR = D / 16;                 // 16-code chunks per row
    constexpr int NCK = 2 * KT * CPR;           // K then V
    constexpr int NIT = (NCK + GS - 1) / GS;
    const uint64_t seq0 = (uint64_t)b * p.seq_stride;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1;
      if (j >= kStages && !mbar_wait_warp(&kv_empty[st], ((j >> 1) - 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
      unsigned char *dst = sm + C::KVOFF + st * 2 * C::KTILE;
#pragma unroll 1
      for (int i0 = 0; i0 < NIT; i0 += 4) {
        uint4 w[4];
        float sc[4];
        int off0[4], off1[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = gtid + (i0 + u) * GS;
          off0[u] = -1;
          w[u] = make_uint4(0, 0, 0, 0);
          sc[u] = 0.f;
          if (i0 + u < NIT && c < NCK) {
            const int which = c / (KT * CPR), rem = c % (KT * CPR), r = rem / CPR, c16 = rem % CPR;
            const uint32_t pos = j * KT + r;
            off0[u] = which * C::KTILE + (int)sw128_off<KT>(r, 2 * c16);
            off1[u] = which * C::KTILE + (int)sw128_off<KT>(r, 2 * c16 + 1);
            if (pos < p.Ltot) {  // rows past Ltot stay zero (0 * garbage could be NaN)
              const uint64_t row = (seq0 + pos) * p.KV + kvh;
              const int8_t *codes = which ? p.Vc : p.Kc;
              const float *scl = which ? p.Vs : p.Ks;
              w[u] = __ldg(reinterpret_cast<const uint4 *>(codes + row * D + c16 * 16));
              sc[u] = __ldg(scl + row * (D / 32) + c16 / 2);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (off0[u] < 0) continue;
          uint4 o0, o1;
          dequant16(w[u], __float2half2_rn(sc[u] * (1.0f / 127.0f)), o0, o1);
          *reinterpret_cast<uint4 *>(dst + off0[u]) = o0;
          *reinterpret_cast<uint4 *>(dst + off1[u]) = o1;
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&kv_full[st]);
    }
  };

  if (warp < 4) asm volatile("setmaxnreg.dec.sync.aligned.u32 72;" ::: "memory");
  if (KVQ8 && D == 128 && warp != 1 && warp < 4) {
    q8_produce((warp == 0 ? 0 : warp - 1) * 32 + lane);
  } else if (warp == 0 && !KVQ8) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      if (!p.qsrc) prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      if (!p.qsrc) {
        mbar_expect_tx(q_full, NQT * C::QTILE);
        for (int t = 0; t < NQT; ++t)
          for (int cb = 0; cb < D / 64; ++cb)
            tma_load_4d(sm + C::Q + t * C::QTILE + cb * kRows * 128, &tmQ, q_full, cb * 64, (int)h,
                        (int)(q0 + t * kRows), (int)b);
      }
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        if (j >= kStages && !mbar_wait(&kv_empty[st], ((j >> 1) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        unsigned char *kd = sm + C::KVOFF + st * 2 * C::KTILE;
        mbar_expect_tx(&kv_full[st], 2 * C::KTILE);
        for (int cb = 0; cb < D / 64; ++cb) {
          tma_load_4d(kd + cb * KT * 128, &tmK, &kv_full[st], cb * 64, (int)kvh, j * KT, (int)b);
          tma_load_4d(kd + C::KTILE + cb * KT * 128, &tmV, &kv_full[st], cb * 64, (int)kvh, j * KT, (int)b);
        }
        issued = j + 1;
      }
      // no bulk copy may still be in flight when the CTA exits
      if (!p.qsrc) mbar_wait(q_full, 0);
      for (int j = max(0, issued - kStages); j < issued; ++j) mbar_wait(&kv_full[j & 1], (j >> 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16(KT, false), idO = idesc_f16(D, true);
      // S_slot = Q_t K^T over D: K-steps of 16 elements (32 B) inside 128 B swizzle atoms
      auto issue_s = [&](int t, uint32_t slot, uint32_t sK) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a = umma_desc_sw128(sQ + t * C::QTILE + (kk >> 2) * (kRows * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bk = umma_desc_sw128(sK + (kk >> 2) * (KT * 128) + (kk & 3) * 32, 16, 1024);
          umma_ss(tmem + slot, a, bk, idS, kk > 0);
        }
      };
      // O_t += P V: P (f16 pairs over the slot's first KT/2 columns) x V (MN-major, N = D)
      auto issue_pv = [&](uint32_t o, uint32_t slot, uint32_t sV, bool acc) {
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
          const uint64_t bv = umma_desc_sw128(sV + kk * 16 * 128, KT * 128, 1024);
          umma_ts(tmem + o, tmem + slot + kk * 8, bv, idO, (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = (p.qsrc || mbar_wait(q_full, 0)) && (ntiles == 0 || mbar_wait(&kv_full[0], 0));
      tc_fence_after();
      int j = 0;
      if constexpr (NQT == 2) {
        // Order per KV tile j:  PV_a(j), S_a(j+1), PV_b(j), S_b(j+1).  S_t(j+1) overwrites the
        // columns PV_t(j) reads P_t(j) from; MMAs issued by one thread execute in order, so it is
        // queued right behind it and the tensor pipe never drains while a softmax runs.  The
        // tcgen05.commit after S_t(j+1) fires only once every earlier MMA (PV_t(j) included) is
        // done, which is what lets the softmax warps touch O_t and P_t after waiting on s_full.
        if (ok && ntiles > 0) {
          issue_s(0, C::S0, sKV);
          umma_commit(&s_full[0]);
          issue_s(1, C::S1, sKV);
          umma_commit(&s_full[1]);
        }
        for (; ok && j < ntiles; ++j) {
          const int st = j & 1;
          const uint32_t sV = sKV + st * 2 * C::KTILE + C::KTILE;
          const uint32_t sKn = sKV + (st ^ 1) * 2 * C::KTILE;
          const bool more = j + 1 < ntiles;
          if (!mbar_wait(&p_full[0], j & 1)) { ok = false; break; }
          tc_fence_after();
          issue_pv(C::O0, C::S0, sV, j > 0);
          umma_commit(&o_done[0]);
          if (more) {
            if (!mbar_wait(&kv_full[st ^ 1], ((j + 1) >> 1) & 1)) { ok = false; break; }
            tc_fence_after();
            issue_s(0, C::S0, sKn);
            umma_commit(&s_full[0]);
          }
          if (!mbar_wait(&p_full[1], j & 1)) { ok = false; break; }
          tc_fence_after();
          issue_pv(C::O1, C::S1, sV, j > 0);
          umma_commit(&o_done[1]);
          umma_commit(&kv_empty[st]);  // K_j and V_j are free once everything so far has completed
          if (more) {
            issue_s(1, C::S1, sKn);
            umma_commit(&s_full[1]);
          }
        }
      } else {
        // One query tile, S double-buffered: S(j+1) is issued as soon as its K tile is in, so it
        // runs while the softmax works on S(j); PV(j) follows P(j).  S(j+1) lands in the slot
        // whose P(j-1) PV(j-1) reads -- queued behind it, in order.
        if (ok && ntiles > 0) {
          issue_s(0, C::S0, sKV);
          umma_commit(&s_full[0]);
        }
        for (; ok && j < ntiles; ++j) {
          const int st = j & 1;
          const uint32_t slot = st ? C::S1 : C::S0;
          if (j + 1 < ntiles) {
            if (!mbar_wait(&kv_full[st ^ 1], ((j + 1) >> 1) & 1)) { ok = false; break; }
            tc_fence_after();
            issue_s(0, st ? C::S0 : C::S1, sKV + (st ^ 1) * 2 * C::KTILE);
            umma_commit(&s_full[st ^ 1]);
          }
          if (!mbar_wait(&p_full[st], (j >> 1) & 1)) { ok = false; break; }
          tc_fence_after();
          issue_pv(C::O0, slot, sKV + st * 2 * C::KTILE + C::KTILE, j > 0);
          umma_commit(&o_done[0]);
          umma_commit(&kv_empty[st]);
        }
      }
      if (!ok) *abort_flag = 1;
      // every MMA this thread issued must complete before the CTA frees TMEM: one more commit
      // tracks all of them
      umma_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
  } else if (warp >= 4) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 216;" ::: "memory");
    if (KVQ8 && D == 256 && warp >= 8) q8_produce((warp - 8) * 32 + lane);
    if (warp >= 4 + 4 * NQT) goto done;
    // ---------------- softmax (one query row per thread) ----------------
    const int t = (warp - 4) >> 2;                 // query tile
    const int row = ((warp & 3) << 5) + lane;      // TMEM lane == tile row
    const uint32_t lane_off = (uint32_t)((warp & 3) << 5) << 16;
    const uint32_t qrow = q0 + t * kRows + row;    // query index within S
    const uint32_t qpos = p.posBase + qrow;
    const uint32_t otile = t ? C::O1 : C::O0;
    const float sl2 = p.sl2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int slot_i = NQT == 2 ? t : (j & 1);
      const uint32_t phase = NQT == 2 ? (j & 1) : ((j >> 1) & 1);
      if (!mbar_wait_warp(&s_full[slot_i], phase)) { ok = false; break; }
      tc_fence_after();
      const uint32_t sbase = (tmem + (slot_i ? C::S1 : C::S0)) | lane_off;
      const int key0 = j * KT;
      // keys of this tile the row may attend: all of them except near the diagonal
      const int nvalid = min(KT, max(0, (int)qpos - key0 + 1));
      // the whole score row in registers: one TMEM wait per tile
      uint32_t r[KT / 32][32];
#pragma unroll
      for (int c = 0; c < KT / 32; ++c) tmem_ld32(sbase + c * 32, r[c]);
      tmem_wait_ld();
      if (nvalid < KT) {  // keys past the diagonal: -inf scores (exp2 -> 0)
#pragma unroll
        for (int c = 0; c < KT / 32; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i >= nvalid) r[c][i] = __float_as_uint(-INFINITY);
      }
      // eight independent max chains instead of one long one
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
#pragma unroll
      for (int c = 0; c < KT / 32; ++c)
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
      // head_dim 128: PV_t(j-1) has completed (the commit we waited on, after S_t(j), covers it).
      // head_dim 256: S(j) was issued before PV(j-1), so PV(j-1) may still run; its o_done phase
      // is consumed exactly once, in order (here, or at the end of this step), so that no wait on
      // o_done can ever be two phases behind the barrier.
      bool pv_prev_done = NQT == 2 || j == 0;
      if (__any_sync(0xffffffffu, need)) {
        if (j > 0) {
          if (!pv_prev_done && !mbar_wait_warp(&o_done[0], (j - 1) & 1)) { ok = false; break; }
          pv_prev_done = true;
          tc_fence_after();
          const float f = (need && m_used > -INFINITY) ? ex2_approx(m_used - mt) : 1.0f;
          const uint32_t obase = (tmem + otile) | lane_off;
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
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
      // p = exp2(s*sl2 - m_used), packed f16 into the first KT/2 columns of the S slot (masked
      // scores hold -inf -> 0).
      float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
      for (int c = 0; c < KT / 32; c += 2) {
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
      if (!pv_prev_done && !mbar_wait_warp(&o_done[0], (j - 1) & 1)) { ok = false; break; }
      tc_fence_before();
      mbar_arrive(&p_full[slot_i]);
    }
    // epilogue: wait for the last PV of this tile, then O / l (x gate) -> out
    if (ok && ntiles > 0 && mbar_wait_warp(&o_done[t], (ntiles - 1) & 1)) {
      tc_fence_after();
      const uint32_t obase = (tmem + otile) | lane_off;
      const float inv = 1.0f / l;
      const bool valid = qrow < p.S;
      const uint64_t orow = (((uint64_t)b * p.S + qrow) * p.H + h) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(obase + c * 32, r);
        tmem_wait_ld();
        if (!valid) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * inv;
        if (p.gate) {
          const float4 *g = reinterpret_cast<const float4 *>(p.gate + orow + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 gv = __ldg(g + i);
            v[4 * i] = v[4 * i] / (1.0f + expf(-gv.x));
            v[4 * i + 1] = v[4 * i + 1] / (1.0f + expf(-gv.y));
            v[4 * i + 2] = v[4 * i + 2] / (1.0f + expf(-gv.z));
            v[4 * i + 3] = v[4 * i + 3] / (1.0f + expf(-gv.w));
          }
        }
        if (p.out_f16) {
          uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + orow + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_half2(v[8 * q], v[8 * q + 1]), pack_half2(v[8 * q + 2], v[8 * q + 3]),
                                pack_half2(v[8 * q + 4], v[8 * q + 5]), pack_half2(v[8 * q + 6], v[8 * q + 7]));
        } else {
          float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + orow + c * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
      }
    } else if (!ok) {
      *abort_flag = 1;
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

template <int D, bool KVQ8>
int launch_cfg(const PrefillArgs &a, cudaStream_t st) {
  using C = PfCfg<D>;
  CUtensorMap tq, tk, tv;
  memset(&tq, 0, sizeof(tq));
  tk = tv = tq;
  if (!a.q_f32 && !KVQ8) {
    const uint64_t dims[4] = {(uint64_t)D, a.H, a.S, a.B};
    const uint64_t strides[3] = {(uint64_t)D * 2, (uint64_t)a.H * D * 2, (uint64_t)a.S * a.H * D * 2};
    const uint32_t box[4] = {64, 1, kRows, 1};
    if (make_tmap_4d(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return BG_EUNSUPPORTED;
  }
  if (!KVQ8) {
    const uint64_t dims[4] = {(uint64_t)D, a.KV, a.Ltot, a.B};
    const uint64_t strides[3] = {(uint64_t)D * 2, (uint64_t)a.KV * D * 2, a.seq_stride * a.KV * D * 2};
    const uint32_t box[4] = {64, 1, (uint32_t)C::KT, 1};
    if (make_tmap_4d(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.K, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return BG_EUNSUPPORTED;
    if (make_tmap_4d(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.V, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return BG_EUNSUPPORTED;
  }
  PfParams p;
  p.out = a.out;
  p.out_f16 = a.out_f16;
  const bool stage_q = a.q_f32 || KVQ8;  // TMA carries f16 queries only next to TMA'd K/V
  p.qsrc = stage_q ? a.q : nullptr;
  p.q_f32 = a.q_f32;
  p.gate = a.gate;
  p.Kc = static_cast<const int8_t *>(a.K);
  p.Vc = static_cast<const int8_t *>(a.V);
  p.Ks = a.Ks;
  p.Vs = a.Vs;
  p.seq_stride = a.seq_stride;
  p.S = a.S;
  p.H = a.H;
  p.KV = a.KV;
  p.G = a.H / a.KV;
  p.posBase = a.posBase;
  p.Ltot = a.Ltot;
  p.sl2 = a.scale * kLog2e;
  const int smem = C::TOTAL + 1024;
  auto kern = prefill_tc_kernel<D, KVQ8>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return BG_ELAUNCH;
  dim3 grid(a.H, (a.S + C::NQT * kRows - 1) / (C::NQT * kRows), a.B);
  kern<<<grid, kThreads, smem, st>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

// q8 cache rows [0, Ltot) of every sequence -> dense f16 [B][Ltot][KV][D] copies of K and V.  One
// thread per 16 codes: value = max(code / 127, -1) * scale in f32 (shaders/attention_sg_kv8.wgsl:40),
// rounded once to f16.  HBM-bound: 144 bytes read and 256 written per 128-element row.
__global__ void __launch_bounds__(256) dequant_q8_kernel(const int8_t *__restrict__ Kc, const int8_t *__restrict__ Vc,
                                                         const float *__restrict__ Ks, const float *__restrict__ Vs,
                                                         uint64_t seq_stride, uint32_t Ltot, uint32_t KV, uint32_t D,
                                                         uint64_t nchunks_side, __half *__restrict__ Ko,
                                                         __half *__restrict__ Vo) {
  const uint32_t cpr = D / 16;
  for (uint64_t c = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; c < 2 * nchunks_side;
       c += (uint64_t)gridDim.x * blockDim.x) {
    const bool v = c >= nchunks_side;
    const uint64_t cc = v ? c - nchunks_side : c;
    const uint64_t drow = cc / cpr;          // ((b*Ltot + pos)*KV + kvh)
    const uint32_t c16 = (uint32_t)(cc % cpr);
    const uint64_t bpos = drow / KV;
    const uint32_t kvh = (uint32_t)(drow % KV);
    const uint64_t b = bpos / Ltot, pos = bpos % Ltot;
    const uint64_t srow = (b * seq_stride + pos) * KV + kvh;
    const uint4 w = __ldg(reinterpret_cast<const uint4 *>((v ? Vc : Kc) + srow * D + c16 * 16));
    const float s = __ldg((v ? Vs : Ks) + srow * (D / 32) + c16 / 2);
    const int8_t *cb = reinterpret_cast<const int8_t *>(&w);
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      o[i] = pack_half2(fmaxf((float)cb[2 * i] / 127.0f, -1.0f) * s, fmaxf((float)cb[2 * i + 1] / 127.0f, -1.0f) * s);
    uint4 *dst = reinterpret_cast<uint4 *>((v ? Vo : Ko) + drow * D + c16 * 16);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

}  // namespace

bool prefill_tc_supported(int mode, uint32_t D, uint32_t S, bool roll, bool ring) {
  const bool shape = (mode == BG_KV_F16 || mode == BG_KV_Q8) ? (D == 128 || D == 256) : (mode == BG_KV_F32 && D == 128);
  return shape && !roll && !ring && S >= 64;
}

int launch_prefill_tc(const PrefillArgs &a, cudaStream_t st) {
  if (a.mode == BG_KV_F32) return launch_prefill_tf32(a, st);
  const bool q8 = a.mode == BG_KV_Q8;
  // q8 with room in the workspace and a prefill that reads every position many times (S large
  // against Ltot): dequantise the cache once into f16 copies, then run the TMA f16 kernel.  The
  // fused form (dequantisation inside every CTA) serves callers without such a workspace.
  const size_t need = prefill_q8_copy_bytes(a.B, a.Ltot, a.KV, a.D);
  if (q8 && a.ws && a.ws_bytes >= need && (uint64_t)a.S * 8 >= a.Ltot) {
    __half *Ko = static_cast<__half *>(a.ws);
    __half *Vo = Ko + (size_t)a.B * a.Ltot * a.KV * a.D;
    const uint64_t nside = (uint64_t)a.B * a.Ltot * a.KV * (a.D / 16);
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t want = (2 * nside + 255) / 256;
    const unsigned grid = (unsigned)(want < (uint64_t)nsm * 8 ? want : (uint64_t)nsm * 8);
    dequant_q8_kernel<<<grid ? grid : 1, 256, 0, st>>>(static_cast<const int8_t *>(a.K), static_cast<const int8_t *>(a.V),
                                                       a.Ks, a.Vs, a.seq_stride, a.Ltot, a.KV, a.D, nside, Ko, Vo);
    if (cudaGetLastError() != cudaSuccess) return BG_ELAUNCH;
    PrefillArgs f = a;
    f.mode = BG_KV_F16;
    f.K = Ko;
    f.V = Vo;
    f.Ks = f.Vs = nullptr;
    f.seq_stride = a.Ltot;
    f.ws = nullptr;
    f.ws_bytes = 0;
    return launch_prefill_tc(f, st);
  }
  if (a.D == 128) return q8 ? launch_cfg<128, true>(a, st) : launch_cfg<128, false>(a, st);
  if (a.D == 256) return q8 ? launch_cfg<256, true>(a, st) : launch_cfg<256, false>(a, st);
  return BG_EUNSUPPORTED;
}

int poll_device_error_prefill() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return BG_ELAUNCH;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  return v;
}

}  // namespace bg
