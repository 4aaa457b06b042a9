// Rope-at-read (sink / rolling-window) decode attention on the tensor cores, sm_100a.
//
// Reference semantics: attention_sg_roll.wgsl:22-62 (f32/f16 K, V) and attention_sg_kv8_roll.wgsl:21-78
// (q8): K is cached unroped and rotated at read by its logical slot j,
//   k'[d] = k[d]*cos[j][d % (D/2)] + rot_half(k)[d]*sin[j][d % (D/2)],
// the cache is a ring of `window` slots behind `sinks` fixed slots (engine.ts:1188-1212 keeps the
// ring head), and the query is already roped.
//
// Design (one CTA per SM, stream-K over (sequence, kv-head group, position)):
//   * a CTA owns HPC kv heads of one sequence at a time (HPC = 8 for the 1.7B shape), one consumer
//     warp per head; the table rows of a tile (cos and sin of 16 logical slots) are shared by all
//     HPC heads, so they are staged once per tile in shared memory instead of being re-read per
//     head from L2;
//   * tiles are 16 logical slots and never straddle a physical discontinuity of the ring (the
//     sink/ring boundary and the ring's wrap point), so every tile is one 4-D TMA box of
//     16 rows x HPC heads x 128 bytes, laid out head-major ([head][slot][128B], 128-byte swizzle)
//     through a tensor map whose kv-head and slot strides are swapped; rows of a short tile past
//     its segment are masked;
//   * the producer warp issues the K/V TMA boxes (lane 0, expect_tx) and cp.async copies of the
//     q8 block scales and of the two table slices (all lanes, arrive.noinc), into an NST-deep
//     mbarrier ring;
//   * the grid is 148 x (resident CTAs per SM); CTA c processes flattened positions
//     [c*W, (c+1)*W) of units x L, so every SM streams the same number of cache rows.  A unit
//     (sequence, head group) cut by CTA boundaries leaves one partial per piece; the CTA holding
//     the unit's first piece marks the unused partial slots empty, and the LSE merge kernel
//     combines them.  When whole units fit per CTA the kernel writes the final rows itself.
// Scores and outputs are computed transposed (S^T = K Q^T, O^T = V^T P^T, m16n8k16) exactly as in
// the plain decode kernel; the rotation runs in f32 on the dequantised K fragment and the rotated
// values are rounded once to f16 for the MMA, with Q split hi + lo.
#include <cuda.h>
#include <cuda_fp16.h>
#include <string.h>

#include "attn.h"
#include "mma.cuh"
#include "tma.cuh"

// 1: rotate in packed f16 (fewer issue slots; errors ~2x the f32 form, far inside tolerance);
// 0: rotate in f32 and round once to f16.
#ifndef BG_ROLL_ROT_F16
#define BG_ROLL_ROT_F16 1
#endif

namespace bg {
namespace {

struct RollParams {
  const void *q;
  int q_f16;
  float *partials;
  uint32_t B, S, H, KV, G, M;
  uint32_t posBase, pos_lo, L;  // attended logical slots [pos_lo, pos_lo + L)
  uint32_t row_offset, nrows_total, nsplit;
  uint32_t units_per_seq;       // KV / HPC
  uint64_t W, total;            // positions per CTA, units * L
  float sl2;
  void *out;
  int out_f16;
  const float *gate;
  const float *cosT, *sinT;
  const float *Ksp, *Vsp;
  uint64_t seq_stride;
  uint32_t sinks, window, ring_head;
};

constexpr int kD = 128;  // head_dim of the rope-at-read kernels

template <int MODE, int HPC>
struct RCfg {
  static constexpr int ES = MODE == BG_KV_F16 ? 2 : 1;
  static constexpr int TP = 16;           // logical slots per tile
  static constexpr int ROWS = HPC * TP;   // smem tile rows, head-major
  static constexpr int ROWB = kD * ES;
  static constexpr int NCB = ROWB / 128;  // 128-byte column blocks per row
  static constexpr int KVT = ROWS * ROWB;
  static constexpr int NB = kD / 32;      // q8 blocks per row
  static constexpr int SCT = MODE == BG_KV_Q8 ? TP * HPC * NB * 4 : 0;
  static constexpr int TBL = TP * (kD / 2) * 4;  // one table's slice for the tile
  static constexpr int STAGE = 2 * KVT + 2 * SCT + 2 * TBL;
  static constexpr int NST_RAW = (220 * 1024) / STAGE;
  static constexpr int NST = NST_RAW < 2 ? 2 : (NST_RAW > 8 ? 8 : NST_RAW);
  static constexpr int THREADS = (HPC + 1) * 32;
  static constexpr int SMEM = NST * STAGE + 1024 + 2 * NST * 8;
};

struct Tile {
  uint32_t ph;  // physical row of the tile's first slot
  uint32_t n;   // slots in the tile (<= 16), all in one physical run
};

// The tile that starts at logical slot `cur` and ends no later than `end`.
__device__ __forceinline__ Tile next_tile(const RollParams &p, uint32_t cur, uint32_t end) {
  uint32_t seg = 0xffffffffu, ph;
  if (p.window == 0 || cur < p.sinks) {
    ph = cur - p.row_offset;
    if (p.window) seg = p.sinks - cur;
  } else {
    uint32_t r = p.ring_head + (cur - p.sinks);  // ring_head < window, cur - sinks < window
    if (r >= p.window) r -= p.window;
    ph = p.sinks + r;
    seg = p.window - r;
  }
  Tile t;
  t.ph = ph;
  t.n = min(min(16u, end - cur), seg);
  return t;
}

// The piece of CTA `c` that starts at flattened position f: unit, logical [a, e), partial slot.
struct Piece {
  uint32_t unit, a, e, slot, count;
};

__device__ __forceinline__ Piece piece_at(const RollParams &p, uint64_t f, uint64_t fend) {
  Piece pc;
  pc.unit = (uint32_t)(f / p.L);
  const uint64_t ubase = (uint64_t)pc.unit * p.L;
  pc.a = p.pos_lo + (uint32_t)(f - ubase);
  pc.e = p.pos_lo + (uint32_t)(min(fend, ubase + p.L) - ubase);
  const uint64_t c_first = ubase / p.W, c_last = (ubase + p.L - 1) / p.W;
  pc.slot = (uint32_t)(f / p.W - c_first);
  pc.count = (uint32_t)(c_last - c_first + 1);
  return pc;
}

template <int MODE, int HPC>
__global__ void __launch_bounds__(RCfg<MODE, HPC>::THREADS, 1)
    attn_roll_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                     RollParams p) {
  using C = RCfg<MODE, HPC>;
  constexpr int TP = C::TP, NST = C::NST, NB = C::NB, ROWS = C::ROWS;
  constexpr int KS = kD / 16;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + NST * C::STAGE);
  uint64_t *empty = full + NST;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint64_t f0 = (uint64_t)blockIdx.x * p.W;
  const uint64_t f1 = min(p.total, f0 + p.W);

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 33);  // lane 0's expect_tx arrival + 32 cp.async arrivals
      mbar_init(&empty[s], HPC);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (f0 >= f1) return;

  if (warp == HPC) {  // ---------------- producer warp ----------------
    if (lane == 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
    }
    bool ok = true;
    uint32_t t = 0;
    for (uint64_t f = f0; f < f1 && ok;) {
      const Piece pc = piece_at(p, f, f1);
      const uint32_t b = pc.unit / p.units_per_seq, kv0 = (pc.unit % p.units_per_seq) * HPC;
      for (uint32_t cur = pc.a; cur < pc.e; ++t) {
        const Tile tl = next_tile(p, cur, pc.e);
        const int s = t % NST;
        if (t >= NST) ok = mbar_wait_warp(&empty[s], ((t / NST) - 1) & 1);
        if (!ok) break;
        unsigned char *st = smem + s * C::STAGE;
        if (lane == 0) {
          mbar_expect_tx(&full[s], 2 * C::KVT);
#pragma unroll
          for (int cb = 0; cb < C::NCB; ++cb) {
            tma_load_4d(st + cb * ROWS * 128, &tmK, &full[s], cb * (128 / C::ES), (int)tl.ph, (int)kv0, (int)b);
            tma_load_4d(st + C::KVT + cb * ROWS * 128, &tmV, &full[s], cb * (128 / C::ES), (int)tl.ph, (int)kv0,
                        (int)b);
          }
        }
        const uint32_t sbase = smem_u32(st + 2 * C::KVT);
        if constexpr (MODE == BG_KV_Q8) {
          // block scales [slot][head][NB] of both caches; slots past the tile are zero-filled
          for (int idx = lane; idx < 2 * TP * HPC; idx += 32) {
            const int which = idx / (TP * HPC), rem = idx % (TP * HPC);
            const int r = rem / HPC, hh = rem % HPC;
            const bool valid = (uint32_t)r < tl.n;
            const uint64_t row = valid ? (((uint64_t)b * p.seq_stride + tl.ph + r) * p.KV + kv0 + hh) : 0;
            const float *src = (which ? p.Vsp : p.Ksp) + row * NB;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sbase + which * C::SCT + rem * 16),
                         "l"(src), "r"(valid ? 16u : 0u)
                         : "memory");
          }
        }
        // cos / sin rows of the tile's logical slots, 16-byte chunks swizzled by (slot & 7)
        const uint32_t tbase = sbase + 2 * C::SCT;
        for (int idx = lane; idx < 2 * TP * 16; idx += 32) {
          const int which = idx / (TP * 16), rem = idx % (TP * 16);
          const int r = rem / 16, c = rem % 16;
          const bool valid = (uint32_t)r < tl.n;
          const float *src = (which ? p.sinT : p.cosT) + (uint64_t)(valid ? cur + r : 0) * (kD / 2) + c * 4;
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(tbase + which * C::TBL +
                                                                            (r * 16 + (c ^ (r & 7))) * 16),
                       "l"(src), "r"(valid ? 16u : 0u)
                       : "memory");
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[s])) : "memory");
        cur += tl.n;
      }
      f = (uint64_t)pc.unit * p.L + (pc.e - p.pos_lo);
    }
    // never leave the CTA with copies in flight: wait (bounded) for the last stages
    if (lane == 0 && ok)
      for (uint32_t u = t > (uint32_t)NST ? t - NST : 0; u < t; ++u) mbar_wait(&full[u % NST], (u / NST) & 1);
    asm volatile("cp.async.wait_all;" ::: "memory");
    return;
  }

  // ---------------- consumer warps: warp w owns kv head kv0 + w ----------------
  const int lrow = (((lane >> 3) & 1) << 3) + (lane & 7);
  const int lhi = lane >> 4;
  const int trow = ((lane >> 4) << 3) + (lane & 7);
  const int tcol = (lane >> 3) & 1;
  const int row0 = warp * TP;
  const int ra = lane >> 2;  // tile-relative slots of the lane's score rows: ra, ra + 8
  bool ok = true;
  uint32_t t = 0;
  for (uint64_t f = f0; f < f1;) {
    const Piece pc = piece_at(p, f, f1);
    f = (uint64_t)pc.unit * p.L + (pc.e - p.pos_lo);
    const uint32_t b = pc.unit / p.units_per_seq, kvh = (pc.unit % p.units_per_seq) * HPC + warp;

    // Q^T fragments of this head's group rows (see the plain decode kernel for the k-slot order)
    uint32_t qh[KS][2], ql[KS][2];
    uint32_t lim[2];
    {
      const uint32_t r = lane >> 2;
      const bool rv = r < p.M;
      const uint32_t qi = rv ? r / p.G : 0, h = kvh * p.G + (rv ? r % p.G : 0);
      const uint64_t qoff = (((uint64_t)b * p.S + qi) * p.H + h) * kD;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int d = MODE == BG_KV_Q8 ? ks * 16 + 4 * (lane & 3) + 2 * half : ks * 16 + 2 * (lane & 3) + 8 * half;
          float x0 = 0.f, x1 = 0.f;
          if (rv) {
            if (p.q_f16) {
              const __half *qp = static_cast<const __half *>(p.q) + qoff + d;
              x0 = __half2float(qp[0]);
              x1 = __half2float(qp[1]);
            } else {
              const float2 v = *reinterpret_cast<const float2 *>(static_cast<const float *>(p.q) + qoff + d);
              x0 = v.x;
              x1 = v.y;
            }
          }
          const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
          qh[ks][half] = pack_f16(__half2float(h0), __half2float(h1));
          ql[ks][half] = pack_f16(x0 - __half2float(h0), x1 - __half2float(h1));
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint32_t rc = 2 * (lane & 3) + j;
        lim[j] = p.posBase + (rc < p.M ? rc / p.G : p.S - 1);
      }
    }

    float m[2] = {kNegBig, kNegBig}, l[2] = {0.f, 0.f};
    float oacc[KS][4];
#pragma unroll
    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) oacc[mt][i] = 0.f;

    for (uint32_t cur = pc.a; cur < pc.e && ok; ++t) {
      const Tile tl = next_tile(p, cur, pc.e);
      const int s = t % NST;
      if (!mbar_wait_warp(&full[s], (t / NST) & 1)) {
        ok = false;
        break;
      }
      const uint32_t sb = smem_u32(smem + s * C::STAGE);
      const uint32_t kb = sb, vb = sb + C::KVT;
      const uint32_t tcos = sb + 2 * C::KVT + 2 * C::SCT, tsin = tcos + C::TBL;
      const float *ksc = reinterpret_cast<const float *>(smem + s * C::STAGE + 2 * C::KVT);
      const uint32_t pa = cur + ra, pb = pa + 8;
      const bool va_ok = (uint32_t)ra < tl.n, vb_ok = (uint32_t)(ra + 8) < tl.n;

      // ---- scores S^T = rot(K) . Q^T, one pair of k steps (dims d, d + D/2) at a time ----
      // four independent accumulators (one per pair of k steps) keep the MMA chains short
      float acc4[KS / 2][4];
#pragma unroll
      for (int c = 0; c < KS / 2; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc4[c][i] = 0.f;
#if BG_ROLL_ROT_F16
      // Packed-f16 rotation: register slot i of an A fragment holds two consecutive dims of row a
      // (i even) or b (i odd); its partner slot in step ks + KS/2 holds the same dims + D/2.
      // cos/sin are read as f32 from the staged slice and packed once per row and slot.
      auto rotate_mma = [&](const uint32_t (&kl)[4], const uint32_t (&kh)[4], int ks) {
        __half2 cs[4], sn[4], nsn[4];
#pragma unroll
        for (int rb = 0; rb < 2; ++rb) {
          const int r = ra + 8 * rb;
          if constexpr (MODE == BG_KV_F16) {
            const int c = ks * 4 + ((lane & 3) >> 1);  // dims d0 = ks*16 + 2*(lane&3) and d0 + 8
            const uint32_t o0 = (r * 16 + (c ^ (r & 7))) * 16 + 8 * (lane & 1);
            const uint32_t o1 = (r * 16 + ((c + 2) ^ (r & 7))) * 16 + 8 * (lane & 1);
            float2 c0, c1, s0, s1;
            asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(c0.x), "=f"(c0.y) : "r"(tcos + o0));
            asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(c1.x), "=f"(c1.y) : "r"(tcos + o1));
            asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(s0.x), "=f"(s0.y) : "r"(tsin + o0));
            asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(s1.x), "=f"(s1.y) : "r"(tsin + o1));
            cs[rb] = __float22half2_rn(c0);
            cs[2 + rb] = __float22half2_rn(c1);
            sn[rb] = __float22half2_rn(s0);
            sn[2 + rb] = __float22half2_rn(s1);
          } else {
            const int c = (ks >> 1) * 8 + (ks & 1) * 4 + (lane & 3);  // dims 4c .. 4c+3
            const uint32_t o = (r * 16 + (c ^ (r & 7))) * 16;
            float4 c4, s4;
            asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                         : "=f"(c4.x), "=f"(c4.y), "=f"(c4.z), "=f"(c4.w)
                         : "r"(tcos + o));
            asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                         : "=f"(s4.x), "=f"(s4.y), "=f"(s4.z), "=f"(s4.w)
                         : "r"(tsin + o));
            cs[rb] = __floats2half2_rn(c4.x, c4.y);
            cs[2 + rb] = __floats2half2_rn(c4.z, c4.w);
            sn[rb] = __floats2half2_rn(s4.x, s4.y);
            sn[2 + rb] = __floats2half2_rn(s4.z, s4.w);
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) nsn[i] = __hneg2(sn[i]);
        uint32_t al[4], ah[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __half2 lo_h = *reinterpret_cast<const __half2 *>(&kl[i]);
          const __half2 hi_h = *reinterpret_cast<const __half2 *>(&kh[i]);
          const __half2 rl = __hfma2(hi_h, nsn[i], __hmul2(lo_h, cs[i]));  // k*cos - k[d+D/2]*sin
          const __half2 rh = __hfma2(lo_h, sn[i], __hmul2(hi_h, cs[i]));   // k*cos + k[d-D/2]*sin
          al[i] = *reinterpret_cast<const uint32_t *>(&rl);
          ah[i] = *reinterpret_cast<const uint32_t *>(&rh);
        }
        float (&acc)[4] = acc4[ks];
        mma16816(acc, al, qh[ks][0], qh[ks][1]);
        mma16816(acc, ah, qh[ks + KS / 2][0], qh[ks + KS / 2][1]);
        mma16816(acc, al, ql[ks][0], ql[ks][1]);
        mma16816(acc, ah, ql[ks + KS / 2][0], ql[ks + KS / 2][1]);
      };
      if constexpr (MODE == BG_KV_F16) {
#pragma unroll
        for (int ks = 0; ks < KS / 2; ++ks) {
          uint32_t a[4], a2[4];
          ldsm_x4(a, swz<ROWS>(kb, row0 + lrow, 2 * ks + lhi));
          ldsm_x4(a2, swz<ROWS>(kb, row0 + lrow, 2 * (ks + KS / 2) + lhi));
          rotate_mma(a, a2, ks);
        }
      } else {
        // snorm8 read: max(code, -127) * (scale/127): the code becomes the exact f16 1152 + code
        // (0x64XX), is clamped and unbiased exactly in f16, then scaled by scale/127 in f16
        const __half2 bias = __float2half2_rn(1152.f), lo127 = __float2half2_rn(1025.f);
        auto deq = [&](uint32_t wx, uint32_t sel, __half2 sc) {
          const uint32_t hb = i8pair_biased(wx, sel);
          const __half2 v = __hmul2(__hsub2(__hmax2(*reinterpret_cast<const __half2 *>(&hb), lo127), bias), sc);
          return *reinterpret_cast<const uint32_t *>(&v);
        };
        const int sa_i = (ra * HPC + warp) * NB, sb_i = ((ra + 8) * HPC + warp) * NB;
#pragma unroll
        for (int bk = 0; bk < NB / 2; ++bk) {
          uint32_t r[4], r2[4];
          ldsm_x4(r, swz<ROWS>(kb, row0 + lrow, 2 * bk + lhi));
          ldsm_x4(r2, swz<ROWS>(kb, row0 + lrow, 2 * (bk + NB / 2) + lhi));
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            r[i] ^= 0x80808080u;
            r2[i] ^= 0x80808080u;
          }
          const __half2 s0 = __float2half2_rn(ksc[sa_i + bk] * (1.0f / 127.0f));
          const __half2 s1 = __float2half2_rn(ksc[sb_i + bk] * (1.0f / 127.0f));
          const __half2 t0 = __float2half2_rn(ksc[sa_i + bk + NB / 2] * (1.0f / 127.0f));
          const __half2 t1 = __float2half2_rn(ksc[sb_i + bk + NB / 2] * (1.0f / 127.0f));
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {  // k step 2bk + h2 from words r[2h2] (row a), r[2h2+1] (row b)
            // a0 = bytes 0,1 of row a; a1 = bytes 0,1 of row b; a2 = bytes 2,3 of row a; a3 = row b
            const uint32_t kl[4] = {deq(r[2 * h2], kSelLo, s0), deq(r[2 * h2 + 1], kSelLo, s1),
                                    deq(r[2 * h2], kSelHi, s0), deq(r[2 * h2 + 1], kSelHi, s1)};
            const uint32_t kh[4] = {deq(r2[2 * h2], kSelLo, t0), deq(r2[2 * h2 + 1], kSelLo, t1),
                                    deq(r2[2 * h2], kSelHi, t0), deq(r2[2 * h2 + 1], kSelHi, t1)};
            rotate_mma(kl, kh, 2 * bk + h2);
          }
        }
      }
#else
      auto rotate_mma = [&](float (&lo_f)[8], float (&hi_f)[8], int ks) {
        float cr_[2][4], sr_[2][4];  // [row a/b][dim slot]
#pragma unroll
        for (int rb = 0; rb < 2; ++rb) {
          const int r = ra + 8 * rb;
          if constexpr (MODE == BG_KV_F16) {
            const int c = ks * 4 + ((lane & 3) >> 1);  // dims d0 = ks*16 + 2*(lane&3) and d0 + 8
            const uint32_t o0 = (r * 16 + (c ^ (r & 7))) * 16 + 8 * (lane & 1);
            const uint32_t o1 = (r * 16 + ((c + 2) ^ (r & 7))) * 16 + 8 * (lane & 1);
            float2 c0, c1, s0, s1;
            asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(c0.x), "=f"(c0.y) : "r"(tcos + o0));
            asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(c1.x), "=f"(c1.y) : "r"(tcos + o1));
            asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(s0.x), "=f"(s0.y) : "r"(tsin + o0));
            asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(s1.x), "=f"(s1.y) : "r"(tsin + o1));
            cr_[rb][0] = c0.x; cr_[rb][1] = c0.y; cr_[rb][2] = c1.x; cr_[rb][3] = c1.y;
            sr_[rb][0] = s0.x; sr_[rb][1] = s0.y; sr_[rb][2] = s1.x; sr_[rb][3] = s1.y;
          } else {
            const int c = (ks >> 1) * 8 + (ks & 1) * 4 + (lane & 3);  // dims 4c .. 4c+3
            const uint32_t o = (r * 16 + (c ^ (r & 7))) * 16;
            float4 c4, s4;
            asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                         : "=f"(c4.x), "=f"(c4.y), "=f"(c4.z), "=f"(c4.w)
                         : "r"(tcos + o));
            asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                         : "=f"(s4.x), "=f"(s4.y), "=f"(s4.z), "=f"(s4.w)
                         : "r"(tsin + o));
            cr_[rb][0] = c4.x; cr_[rb][1] = c4.y; cr_[rb][2] = c4.z; cr_[rb][3] = c4.w;
            sr_[rb][0] = s4.x; sr_[rb][1] = s4.y; sr_[rb][2] = s4.z; sr_[rb][3] = s4.w;
          }
        }
        float rl[8], rh[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          // element e: {a0.x, a0.y, a1.x, a1.y, a2.x, a2.y, a3.x, a3.y}; a1/a3 hold row b
          const int rb = (e >> 1) & 1;
          const int slot = ((e >> 2) & 1) * 2 + (e & 1);
          const float c = cr_[rb][slot], sn = sr_[rb][slot];
          rl[e] = lo_f[e] * c - hi_f[e] * sn;  // d < D/2: k*cos + (-k[d+D/2])*sin
          rh[e] = hi_f[e] * c + lo_f[e] * sn;  // d >= D/2: k*cos + k[d-D/2]*sin
        }
        const uint32_t al[4] = {pack_f16(rl[0], rl[1]), pack_f16(rl[2], rl[3]), pack_f16(rl[4], rl[5]),
                                pack_f16(rl[6], rl[7])};
        const uint32_t ah[4] = {pack_f16(rh[0], rh[1]), pack_f16(rh[2], rh[3]), pack_f16(rh[4], rh[5]),
                                pack_f16(rh[6], rh[7])};
        float (&acc)[4] = acc4[ks];
        mma16816(acc, al, qh[ks][0], qh[ks][1]);
        mma16816(acc, ah, qh[ks + KS / 2][0], qh[ks + KS / 2][1]);
        mma16816(acc, al, ql[ks][0], ql[ks][1]);
        mma16816(acc, ah, ql[ks + KS / 2][0], ql[ks + KS / 2][1]);
      };
      if constexpr (MODE == BG_KV_F16) {
#pragma unroll
        for (int ks = 0; ks < KS / 2; ++ks) {
          uint32_t a[4], a2[4];
          ldsm_x4(a, swz<ROWS>(kb, row0 + lrow, 2 * ks + lhi));
          ldsm_x4(a2, swz<ROWS>(kb, row0 + lrow, 2 * (ks + KS / 2) + lhi));
          float lo_f[8], hi_f[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 x = __half22float2(*reinterpret_cast<const __half2 *>(&a[i]));
            const float2 y = __half22float2(*reinterpret_cast<const __half2 *>(&a2[i]));
            lo_f[2 * i] = x.x;
            lo_f[2 * i + 1] = x.y;
            hi_f[2 * i] = y.x;
            hi_f[2 * i + 1] = y.y;
          }
          rotate_mma(lo_f, hi_f, ks);
        }
      } else {
        // snorm8 read: max(code/127, -1) * scale == max(code, -127) * (scale/127)
        const int sa_i = (ra * HPC + warp) * NB, sb_i = ((ra + 8) * HPC + warp) * NB;
#pragma unroll
        for (int bk = 0; bk < NB / 2; ++bk) {
          uint32_t r[4], r2[4];
          ldsm_x4(r, swz<ROWS>(kb, row0 + lrow, 2 * bk + lhi));
          ldsm_x4(r2, swz<ROWS>(kb, row0 + lrow, 2 * (bk + NB / 2) + lhi));
          const float s0 = ksc[sa_i + bk] * (1.0f / 127.0f), s1 = ksc[sb_i + bk] * (1.0f / 127.0f);
          const float t0 = ksc[sa_i + bk + NB / 2] * (1.0f / 127.0f), t1 = ksc[sb_i + bk + NB / 2] * (1.0f / 127.0f);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {  // k step 2bk + h2 from words r[2h2] (row a), r[2h2+1] (row b)
            const uint32_t wa = r[2 * h2], wb = r[2 * h2 + 1], xa = r2[2 * h2], xb = r2[2 * h2 + 1];
            float lo_f[8], hi_f[8];
            // a0 = bytes 0,1 of row a; a1 = bytes 0,1 of row b; a2 = bytes 2,3 of row a; a3 = row b
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int sh = 8 * ((e & 1) + 2 * (e >> 2));
              const bool rowb = (e >> 1) & 1;
              lo_f[e] = fmaxf((float)(int8_t)(((rowb ? wb : wa) >> sh) & 0xff), -127.f) * (rowb ? s1 : s0);
              hi_f[e] = fmaxf((float)(int8_t)(((rowb ? xb : xa) >> sh) & 0xff), -127.f) * (rowb ? t1 : t0);
            }
            rotate_mma(lo_f, hi_f, 2 * bk + h2);
          }
        }
      }

#endif
      float acc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = (acc4[0][i] + acc4[1][i]) + (acc4[2][i] + acc4[3][i]);

      // ---- online softmax (columns n0 = 2(lane%4), n1 = n0+1; rows pa, pb) ----
      float pr[4], cr[2];
      bool moved = false;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float x0 = (va_ok && pa <= lim[j]) ? acc[j] * p.sl2 : -INFINITY;
        const float x1 = (vb_ok && pb <= lim[j]) ? acc[2 + j] * p.sl2 : -INFINITY;
        float mx = fmaxf(x0, x1);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(m[j], mx);
        const float corr = exp2f(m[j] - mn);
        const float p0 = exp2f(x0 - mn), p1 = exp2f(x1 - mn);
        l[j] = l[j] * corr + p0 + p1;
        m[j] = mn;
        pr[j] = p0;
        pr[2 + j] = p1;
        cr[j] = corr;
        moved |= corr != 1.0f;
      }
      if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
        for (int mt = 0; mt < KS; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) oacc[mt][i] *= cr[i & 1];
      }

      // ---- O^T += V^T . P^T ----
      if constexpr (MODE == BG_KV_F16) {
        const uint32_t pb0 = movm_t(pack_f16(pr[0], pr[1])), pb1 = movm_t(pack_f16(pr[2], pr[3]));
        // slots past a short tile may hold any bits (another run of the ring): zero them so that
        // 0 * NaN cannot reach the accumulator.  Fragment halves: slots 2(lane%4)+{0,1} (+8).
        uint32_t mlo = 0xffffffffu, mhi = 0xffffffffu;
        if (tl.n < (uint32_t)TP) {
          const uint32_t k0 = 2 * (lane & 3);
          mlo = (k0 < tl.n ? 0xffffu : 0u) | (k0 + 1 < tl.n ? 0xffff0000u : 0u);
          mhi = (k0 + 8 < tl.n ? 0xffffu : 0u) | (k0 + 9 < tl.n ? 0xffff0000u : 0u);
        }
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          uint32_t a[4];
          ldsm_x4_t(a, swz<ROWS>(vb, row0 + trow, 2 * mt + tcol));
          a[0] &= mlo;
          a[1] &= mlo;
          a[2] &= mhi;
          a[3] &= mhi;
          mma16816(oacc[mt], a, pb0, pb1);
        }
      } else {
        const float *vsc = ksc + TP * HPC * NB;
        const int sa_i = (ra * HPC + warp) * NB, sb_i = ((ra + 8) * HPC + warp) * NB;
#pragma unroll
        for (int bk = 0; bk < NB; ++bk) {
          const float va = vsc[sa_i + bk] * (1.0f / 127.0f);  // zero-filled past the tile
          const float vbb = vsc[sb_i + bk] * (1.0f / 127.0f);
          const uint32_t pb0 = movm_t(pack_f16(pr[0] * va, pr[1] * va));
          const uint32_t pb1 = movm_t(pack_f16(pr[2] * vbb, pr[3] * vbb));
          uint32_t r[4];
          ldsm_x4_t(r, swz<ROWS>(vb, row0 + lrow, 2 * bk + lhi));
#pragma unroll
          for (int i = 0; i < 4; ++i) r[i] ^= 0x80808080u;
          const uint32_t a0[4] = {i8pair_biased(r[0], kSelEven), i8pair_biased(r[0], kSelOdd),
                                  i8pair_biased(r[1], kSelEven), i8pair_biased(r[1], kSelOdd)};
          const uint32_t a1[4] = {i8pair_biased(r[2], kSelEven), i8pair_biased(r[2], kSelOdd),
                                  i8pair_biased(r[3], kSelEven), i8pair_biased(r[3], kSelOdd)};
          const uint32_t ng = kNeg1152x2();
          const uint32_t aneg[4] = {ng, ng, ng, ng};
          mma16816(oacc[2 * bk], a0, pb0, pb1);
          mma16816(oacc[2 * bk], aneg, pb0, pb1);
          mma16816(oacc[2 * bk + 1], a1, pb0, pb1);
          mma16816(oacc[2 * bk + 1], aneg, pb0, pb1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      cur += tl.n;
    }

    // ---- piece epilogue: this head's rows (columns) to the partial slot or the final output ----
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float lt = l[j];
      lt += __shfl_xor_sync(0xffffffffu, lt, 4);
      lt += __shfl_xor_sync(0xffffffffu, lt, 8);
      lt += __shfl_xor_sync(0xffffffffu, lt, 16);
      const uint32_t n = 2 * (lane & 3) + j;
      if (n >= p.M) continue;
      const uint32_t qi = n / p.G, h = kvh * p.G + n % p.G;
      const uint64_t grow = ((uint64_t)b * p.S + qi) * p.H + h;
      if (p.out) {
        const float inv = 1.0f / lt;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int d = MODE == BG_KV_F16 ? mt * 16 + (lane >> 2) + 8 * hh : mt * 16 + 2 * (lane >> 2) + hh;
            float v = ok ? oacc[mt][2 * hh + j] * inv : 0.f;
            if (p.gate) v = v / (1.0f + expf(-p.gate[grow * kD + d]));
            if (p.out_f16) static_cast<__half *>(p.out)[grow * kD + d] = __float2half_rn(v);
            else static_cast<float *>(p.out)[grow * kD + d] = v;
          }
        }
        continue;
      }
      float *dst = p.partials + ((uint64_t)pc.slot * p.nrows_total + grow) * (kD + 2);
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int d = MODE == BG_KV_F16 ? mt * 16 + (lane >> 2) + 8 * hh : mt * 16 + 2 * (lane >> 2) + hh;
          dst[d] = ok ? oacc[mt][2 * hh + j] : 0.f;
        }
      }
      if (lane < 4) {
        dst[kD] = (ok && lt > 0.f) ? m[j] * kLn2 : -INFINITY;
        dst[kD + 1] = ok ? lt : 0.f;
      }
      // the unit's first piece marks its unused partial slots empty
      if (pc.slot == 0) {
        for (uint32_t sl = pc.count; sl < p.nsplit; ++sl) {
          float *e = p.partials + ((uint64_t)sl * p.nrows_total + grow) * (kD + 2);
          for (int d = lane >> 2; d < kD + 2; d += 8) e[d] = d == kD ? -INFINITY : 0.f;
        }
      }
    }
    if (!ok) break;
  }
}

struct RollSched {
  uint32_t grid, nsplit;
  uint64_t W;
};

template <int MODE, int HPC>
int roll_occupancy() {
  using C = RCfg<MODE, HPC>;
  static int cached = 0;
  if (!cached) {
    int n = 0;
    auto kern = attn_roll_kernel<MODE, HPC>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, C::THREADS, C::SMEM) != cudaSuccess || n < 1) n = 1;
    cached = n;
  }
  return cached;
}

int roll_hpc(uint32_t KV) { return KV % 8 == 0 ? 8 : (KV % 4 == 0 ? 4 : (KV % 2 == 0 ? 2 : 0)); }

int roll_occ(int mode, int hpc) {
  if (mode == BG_KV_F16) return hpc == 8 ? roll_occupancy<BG_KV_F16, 8>() : hpc == 4 ? roll_occupancy<BG_KV_F16, 4>()
                                                                                   : roll_occupancy<BG_KV_F16, 2>();
  return hpc == 8 ? roll_occupancy<BG_KV_Q8, 8>() : hpc == 4 ? roll_occupancy<BG_KV_Q8, 4>()
                                                             : roll_occupancy<BG_KV_Q8, 2>();
}

// Stream-K schedule: W flattened positions per CTA (at least 64), whole units per CTA when there
// are at least as many units as resident CTAs.
RollSched roll_schedule(uint64_t units, uint32_t L, int occ) {
  const uint64_t slots = 148ull * (uint64_t)occ;
  const uint64_t total = units * L;
  RollSched r;
  uint64_t W = (total + slots - 1) / slots;
  if (W < 64) W = 64;
  if (W >= L) {
    const uint64_t per = (W + L - 1) / L;
    r.W = per * L;
    r.grid = (uint32_t)((units + per - 1) / per);
    r.nsplit = 1;
    return r;
  }
  r.W = W;
  r.grid = (uint32_t)((total + W - 1) / W);
  r.nsplit = (uint32_t)((L + W - 1) / W + 1);
  return r;
}

template <int MODE, int HPC>
int launch_roll_cfg(const AttnArgs &a, const RollSched &sc, uint32_t L, cudaStream_t st) {
  using C = RCfg<MODE, HPC>;
  CUtensorMap tk, tv;
  // dims (element, slot, kv head, sequence); the kv-head and slot strides are swapped so a box
  // lands head-major in shared memory and the 128-byte swizzle spreads consecutive slots
  const uint64_t rb = (uint64_t)kD * C::ES;
  uint64_t ext = a.kv.seq_stride;
  if (!a.kv.window) ext = a.pos_hi - a.kv.row_offset;
  const uint64_t dims[4] = {kD, ext, a.KV, a.B};
  const uint64_t strides[3] = {rb * a.KV, rb, rb * a.KV * a.kv.seq_stride};
  const uint32_t box[4] = {128 / C::ES, C::TP, HPC, 1};
  const CUtensorMapDataType dt = MODE == BG_KV_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  if (make_tmap_4d(&tk, dt, a.kv.K, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return BG_EUNSUPPORTED;
  if (make_tmap_4d(&tv, dt, a.kv.V, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return BG_EUNSUPPORTED;
  RollParams p;
  p.q = a.q;
  p.q_f16 = a.q_f16;
  p.partials = a.partials;
  p.B = a.B;
  p.S = a.S;
  p.H = a.H;
  p.KV = a.KV;
  p.G = a.H / a.KV;
  p.M = a.S * p.G;
  p.posBase = a.posBase;
  p.pos_lo = a.pos_lo;
  p.L = L;
  p.row_offset = a.kv.row_offset;
  p.nrows_total = a.B * a.S * a.H;
  p.nsplit = sc.nsplit;
  p.units_per_seq = a.KV / HPC;
  p.W = sc.W;
  p.total = (uint64_t)a.B * p.units_per_seq * L;
  p.sl2 = a.scale * kLog2e;
  p.out = a.out;
  p.out_f16 = a.out_f16;
  p.gate = a.gate;
  p.cosT = a.cosT;
  p.sinT = a.sinT;
  p.Ksp = a.kv.Ks;
  p.Vsp = a.kv.Vs;
  p.seq_stride = a.kv.seq_stride;
  p.sinks = a.kv.sinks;
  p.window = a.kv.window;
  p.ring_head = a.kv.ring_head;
  auto kern = attn_roll_kernel<MODE, HPC>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
    return BG_ELAUNCH;
  kern<<<sc.grid, C::THREADS, C::SMEM, st>>>(tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

}  // namespace

bool attn_roll_supported(int mode, uint32_t D, uint32_t S, uint32_t H, uint32_t KV) {
  return (mode == BG_KV_F16 || mode == BG_KV_Q8) && D == kD && roll_hpc(KV) && S * (H / KV) <= 8;
}

uint32_t attn_roll_num_splits(int mode, uint32_t B, uint32_t KV, uint32_t L) {
  const int hpc = roll_hpc(KV);
  return roll_schedule((uint64_t)B * (KV / hpc), L ? L : 1, roll_occ(mode, hpc)).nsplit;
}

int launch_attn_roll(const AttnArgs &a, cudaStream_t st) {
  if (!attn_roll_supported(a.mode, a.D, a.S, a.H, a.KV) || !a.cosT) return BG_EUNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(a.cosT) % 16 || reinterpret_cast<uintptr_t>(a.sinT) % 16) return BG_EUNSUPPORTED;
  // slots past the last query's position are masked by the causal limit of every row
  const uint32_t L = a.pos_hi > a.pos_lo ? a.pos_hi - a.pos_lo : 0;
  const int hpc = roll_hpc(a.KV);
  const RollSched sc = roll_schedule((uint64_t)a.B * (a.KV / hpc), L ? L : 1, roll_occ(a.mode, hpc));
  if (sc.nsplit != a.nsplit || L == 0) return BG_EUNSUPPORTED;  // caller sized partials differently
  if (a.mode == BG_KV_F16) {
    if (hpc == 8) return launch_roll_cfg<BG_KV_F16, 8>(a, sc, L, st);
    if (hpc == 4) return launch_roll_cfg<BG_KV_F16, 4>(a, sc, L, st);
    return launch_roll_cfg<BG_KV_F16, 2>(a, sc, L, st);
  }
  if (hpc == 8) return launch_roll_cfg<BG_KV_Q8, 8>(a, sc, L, st);
  if (hpc == 4) return launch_roll_cfg<BG_KV_Q8, 4>(a, sc, L, st);
  return launch_roll_cfg<BG_KV_Q8, 2>(a, sc, L, st);
}

int poll_device_error_attn_roll() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return BG_ELAUNCH;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  return v;
}

}  // namespace bg
