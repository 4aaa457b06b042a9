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
//   * three producer warps share the loads of a stage: the K/V TMA boxes (lane 0, expect_tx),
//     the two table slices and the q8 block scales (cp.async, arrive.noinc), into an NST-deep
//     mbarrier ring;
//   * the grid is 148 x (resident CTAs per SM); CTA c processes flattened positions
//     [c*W, (c+1)*W) of units x L, so every SM streams the same number of cache rows.  A unit
//     (sequence, head group) cut by CTA boundaries leaves one partial per piece; the CTA holding
//     the unit's first piece marks the unused partial slots empty, and the LSE merge kernel
//     combines them.  When whole units fit per CTA the kernel writes the final rows itself.
// Scores and outputs are computed transposed (S^T = K Q^T, O^T = V^T P^T, m16n8k16) as in the
// plain decode kernel, but with Q as one f16 operand: the rotated K is itself rounded to f16, so a
// lo half of Q (the plain kernel's hi + lo split) would add MMAs without adding accuracy.  K is
// dequantised and rotated in packed f16 (the operand precision of the MMA; an f32 rotation rounded
// once was measured ~5% slower at half the error, both far inside the 2e-3 gate).  Each consumer
// step takes two tiles when the piece has them, so one max reduction covers 32 slots.
#include <cuda.h>
#include <cuda_fp16.h>
#include <string.h>

#include <type_traits>

#include "attn.h"
#include "mma.cuh"
#include "tma.cuh"

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
  // consumer warps fill whole warpgroups; warp CW of the warpgroup after them is the producer
  static constexpr int CW = HPC < 4 ? 4 : HPC;
  static constexpr int THREADS = (CW + 4) * 32;
  // 384 threads launch at 168 registers (3 warps on some SM sub-partition); the producer
  // warpgroup gives back to 40 and the two consumer warpgroups take 232: 128*40 + 256*232 ==
  // 384*168.  Up to 256 threads need no split (255 registers each).
  static constexpr bool SPLIT_REGS = THREADS > 256;
  static constexpr int SMEM = NST * STAGE + 1024 + 2 * NST * 8;
};

// XOR swizzle of the 16-byte chunks of a staged cos/sin row r.  q8 consumers read 16 bytes per
// lane (one wavefront per quarter warp: rows 2i and 2i+1, four chunks each), f16 consumers 8 bytes
// per lane (one wavefront per half warp: rows 4i..4i+3, two chunks each); these XORs put every
// lane of a wavefront on a distinct 16-byte bank group.
template <int MODE>
__device__ __forceinline__ int tbl_swz(int r) {
  return MODE == BG_KV_F16 ? ((r & 3) << 1) : ((r & 1) << 2);
}

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
      // lane 0's expect_tx arrival + 32 cp.async arrivals per cp.async role (tables; q8 scales)
      mbar_init(&full[s], MODE == BG_KV_Q8 ? 65 : 33);
      mbar_init(&empty[s], HPC);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (f0 >= f1) return;
  static_assert(!C::SPLIT_REGS || C::THREADS == 384, "register split sized for 384 threads");

  if (warp >= C::CW) {  // ---------------- producer warpgroup ----------------
    // role 0: K/V boxes by TMA (lane 0, expect_tx); role 1: cos/sin slices by cp.async; role 2
    // (q8): block scales by cp.async.  Each role walks the same tile sequence and waits for the
    // stage to be released on its own; the cp.async roles arrive with noinc (32 arrivals each).
    if constexpr (C::SPLIT_REGS) asm volatile("setmaxnreg.dec.sync.aligned.u32 40;" ::: "memory");
    const int role = warp - C::CW;
    if (role > (MODE == BG_KV_Q8 ? 2 : 1)) return;
    if (role == 0 && lane == 0) {
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
        const uint32_t sbase = smem_u32(st + 2 * C::KVT);
        if (role == 0) {
          if (lane == 0) {
            mbar_expect_tx(&full[s], 2 * C::KVT);
#pragma unroll
            for (int cb = 0; cb < C::NCB; ++cb) {
              tma_load_4d(st + cb * ROWS * 128, &tmK, &full[s], cb * (128 / C::ES), (int)tl.ph, (int)kv0, (int)b);
              tma_load_4d(st + C::KVT + cb * ROWS * 128, &tmV, &full[s], cb * (128 / C::ES), (int)tl.ph,
                          (int)kv0, (int)b);
            }
          }
        } else if (role == 1) {
          // cos / sin rows of the tile's logical slots; lane: chunk c = lane % 16 of rows
          // lane/16 + 2i, swizzled by tbl_swz
          const int c = lane & 15, r0 = lane >> 4;
          const uint32_t tbase = sbase + 2 * C::SCT;
          const float *cs = p.cosT + (uint64_t)cur * (kD / 2) + c * 4, *sn = p.sinT + (uint64_t)cur * (kD / 2) + c * 4;
#pragma unroll
          for (int i = 0; i < TP / 2; ++i) {
            const int r = r0 + 2 * i;
            const bool valid = (uint32_t)r < tl.n;
            const uint32_t off = valid ? r * (kD / 2) : 0;
            const uint32_t dst = tbase + (r * 16 + (c ^ tbl_swz<MODE>(r))) * 16;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(cs + off),
                         "r"(valid ? 16u : 0u)
                         : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst + C::TBL), "l"(sn + off),
                         "r"(valid ? 16u : 0u)
                         : "memory");
          }
          asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[s])) : "memory");
        } else if constexpr (MODE == BG_KV_Q8) {
          // block scales [head][slot][NB] of both caches (head-major: the 8 slots a consumer warp
          // reads at once are 16 bytes apart); lane: slot lane % 16 of heads lane/16 + 2i; slots
          // past the tile are zero-filled
          const int r = lane & 15, h0 = lane >> 4;
          const bool valid = (uint32_t)r < tl.n;
          const uint64_t row = valid ? ((uint64_t)b * p.seq_stride + tl.ph + r) * p.KV + kv0 : 0;
          const float *ks = p.Ksp + row * NB, *vs = p.Vsp + row * NB;
#pragma unroll
          for (int i = 0; i < HPC / 2; ++i) {
            const int hh = h0 + 2 * i;
            const uint32_t dst = sbase + (hh * TP + r) * 16;
            const uint32_t off = valid ? hh * NB : 0;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(ks + off),
                         "r"(valid ? 16u : 0u)
                         : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst + C::SCT), "l"(vs + off),
                         "r"(valid ? 16u : 0u)
                         : "memory");
          }
          asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[s])) : "memory");
        }
        cur += tl.n;
      }
      f = (uint64_t)pc.unit * p.L + (pc.e - p.pos_lo);
    }
    // never leave the CTA with copies in flight: wait (bounded) for the last stages
    if (role == 0 && lane == 0 && ok)
      for (uint32_t u = t > (uint32_t)NST ? t - NST : 0; u < t; ++u) mbar_wait(&full[u % NST], (u / NST) & 1);
    asm volatile("cp.async.wait_all;" ::: "memory");
    return;
  }

  // ---------------- consumer warps: warp w owns kv head kv0 + w ----------------
  if constexpr (C::SPLIT_REGS) asm volatile("setmaxnreg.inc.sync.aligned.u32 232;" ::: "memory");
  if (warp >= HPC) return;  // idle warps of a padded consumer warpgroup
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
    uint32_t qh[KS][2];
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

    // scores S^T = rot(K) . Q^T of one tile (raw, unscaled), one pair of k steps (dims d and
    // d + D/2) at a time, into four independent accumulators that keep the MMA chains short.
    // The rotation runs in packed f16: register slot i of an A fragment holds two consecutive
    // dims of row a (i even) or b (i odd); its partner slot in step ks + KS/2 holds the same
    // dims + D/2.  cos/sin are read as f32 from the staged slice and packed once per row and slot.
    auto tile_scores = [&](uint32_t sb, const float *ksc, float (&acc)[4]) {
      const uint32_t kb = sb;
      const uint32_t tcos = sb + 2 * C::KVT + 2 * C::SCT, tsin = tcos + C::TBL;
      float acc4[KS / 2][4];
#pragma unroll
      for (int c = 0; c < KS / 2; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc4[c][i] = 0.f;
      auto rotate_mma = [&](const uint32_t (&kl)[4], const uint32_t (&kh)[4], int ks) {
        __half2 cs[4], sn[4];
#pragma unroll
        for (int rb = 0; rb < 2; ++rb) {
          const int r = ra + 8 * rb;
          if constexpr (MODE == BG_KV_F16) {
            const int c = ks * 4 + ((lane & 3) >> 1);  // dims d0 = ks*16 + 2*(lane&3) and d0 + 8
            const uint32_t o0 = (r * 16 + (c ^ tbl_swz<MODE>(r))) * 16 + 8 * (lane & 1);
            const uint32_t o1 = (r * 16 + ((c + 2) ^ tbl_swz<MODE>(r))) * 16 + 8 * (lane & 1);
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
            const uint32_t o = (r * 16 + (c ^ tbl_swz<MODE>(r))) * 16;
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
        uint32_t al[4], ah[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __half2 lo_h = *reinterpret_cast<const __half2 *>(&kl[i]);
          const __half2 hi_h = *reinterpret_cast<const __half2 *>(&kh[i]);
          const __half2 rl = __hfma2(__hneg2(hi_h), sn[i], __hmul2(lo_h, cs[i]));  // k*cos - k[d+D/2]*sin
          const __half2 rh = __hfma2(lo_h, sn[i], __hmul2(hi_h, cs[i]));           // k*cos + k[d-D/2]*sin
          al[i] = *reinterpret_cast<const uint32_t *>(&rl);
          ah[i] = *reinterpret_cast<const uint32_t *>(&rh);
        }
        float (&ac)[4] = acc4[ks];
        mma16816(ac, al, qh[ks][0], qh[ks][1]);
        mma16816(ac, ah, qh[ks + KS / 2][0], qh[ks + KS / 2][1]);
      };
      if constexpr (MODE == BG_KV_F16) {
#pragma unroll
        for (int ks = 0; ks < KS / 2; ++ks) {
          uint32_t x[4], x2[4];
          ldsm_x4(x, swz<ROWS>(kb, row0 + lrow, 2 * ks + lhi));
          ldsm_x4(x2, swz<ROWS>(kb, row0 + lrow, 2 * (ks + KS / 2) + lhi));
          rotate_mma(x, x2, ks);
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
        const int sa_i = (warp * TP + ra) * NB, sb_i = (warp * TP + ra + 8) * NB;
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
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = (acc4[0][i] + acc4[1][i]) + (acc4[2][i] + acc4[3][i]);
    };

    // O^T += V^T . P^T of one tile
    auto tile_pv = [&](uint32_t sb, const float *ksc, uint32_t n, const float (&pr)[4]) {
      const uint32_t vb = sb + C::KVT;
      if constexpr (MODE == BG_KV_F16) {
        const uint32_t pb0 = movm_t(pack_f16(pr[0], pr[1])), pb1 = movm_t(pack_f16(pr[2], pr[3]));
        // slots past a short tile may hold any bits (another run of the ring): zero them so that
        // 0 * NaN cannot reach the accumulator.  Fragment halves: slots 2(lane%4)+{0,1} (+8).
        uint32_t mlo = 0xffffffffu, mhi = 0xffffffffu;
        if (n < (uint32_t)TP) {
          const uint32_t k0 = 2 * (lane & 3);
          mlo = (k0 < n ? 0xffffu : 0u) | (k0 + 1 < n ? 0xffff0000u : 0u);
          mhi = (k0 + 8 < n ? 0xffffu : 0u) | (k0 + 9 < n ? 0xffff0000u : 0u);
        }
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          uint32_t x[4];
          ldsm_x4_t(x, swz<ROWS>(vb, row0 + trow, 2 * mt + tcol));
          x[0] &= mlo;
          x[1] &= mlo;
          x[2] &= mhi;
          x[3] &= mhi;
          mma16816(oacc[mt], x, pb0, pb1);
        }
      } else {
        const float *vsc = ksc + TP * HPC * NB;
        const int sa_i = (warp * TP + ra) * NB, sb_i = (warp * TP + ra + 8) * NB;
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
    };

    // NSUB (1 or 2) consecutive tiles per step: one max reduction and one rescale decision per
    // column for up to 32 slots, and two independent score chains in flight.
    auto step = [&](auto nsub_c, const uint32_t (&cu)[2], const Tile (&tl)[2], const int (&st)[2]) {
      constexpr int NSUB = decltype(nsub_c)::value;
      float acc[NSUB][4];
#pragma unroll
      for (int u = 0; u < NSUB; ++u)
        tile_scores(smem_u32(smem + st[u] * C::STAGE),
                    reinterpret_cast<const float *>(smem + st[u] * C::STAGE + 2 * C::KVT), acc[u]);
      float pr[NSUB][4], cr[2];
      bool moved = false;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float x[NSUB][2];
        float mx = -INFINITY;
#pragma unroll
        for (int u = 0; u < NSUB; ++u) {
          const uint32_t pa = cu[u] + ra;
          x[u][0] = ((uint32_t)ra < tl[u].n && pa <= lim[j]) ? acc[u][j] * p.sl2 : -INFINITY;
          x[u][1] = ((uint32_t)(ra + 8) < tl[u].n && pa + 8 <= lim[j]) ? acc[u][2 + j] * p.sl2 : -INFINITY;
          mx = fmaxf(mx, fmaxf(x[u][0], x[u][1]));
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(m[j], mx);
        const float corr = exp2f(m[j] - mn);
        float ls = 0.f;
#pragma unroll
        for (int u = 0; u < NSUB; ++u) {
          pr[u][j] = exp2f(x[u][0] - mn);
          pr[u][2 + j] = exp2f(x[u][1] - mn);
          ls += pr[u][j] + pr[u][2 + j];
        }
        l[j] = l[j] * corr + ls;
        m[j] = mn;
        cr[j] = corr;
        moved |= corr != 1.0f;
      }
      if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
        for (int mt = 0; mt < KS; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) oacc[mt][i] *= cr[i & 1];
      }
#pragma unroll
      for (int u = 0; u < NSUB; ++u)
        tile_pv(smem_u32(smem + st[u] * C::STAGE),
                reinterpret_cast<const float *>(smem + st[u] * C::STAGE + 2 * C::KVT), tl[u].n, pr[u]);
      __syncwarp();
      if (lane == 0)
#pragma unroll
        for (int u = 0; u < NSUB; ++u) mbar_arrive(&empty[st[u]]);
    };

    for (uint32_t cur = pc.a; cur < pc.e && ok;) {
      Tile tl[2];
      uint32_t cu[2];
      cu[0] = cur;
      tl[0] = next_tile(p, cur, pc.e);
      cu[1] = cur + tl[0].n;
      const bool two = cu[1] < pc.e;
      tl[1] = two ? next_tile(p, cu[1], pc.e) : Tile{0u, 0u};
      const int st[2] = {(int)(t % NST), (int)((t + 1) % NST)};
      if (!mbar_wait_warp(&full[st[0]], (t / NST) & 1) ||
          (two && !mbar_wait_warp(&full[st[1]], ((t + 1) / NST) & 1))) {
        ok = false;
        break;
      }
      if (two) {
        step(std::integral_constant<int, 2>{}, cu, tl, st);
        t += 2;
        cur = cu[1] + tl[1].n;
      } else {
        step(std::integral_constant<int, 1>{}, cu, tl, st);
        t += 1;
        cur = cu[1];
      }
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
