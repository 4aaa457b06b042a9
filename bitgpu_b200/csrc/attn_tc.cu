// Tensor-core split-KV decode attention for f16 and q8 KV caches (sm_100a).
//
// Decode attention is HBM-bound: every cached K/V row is read once per step and the math per row
// is tiny.  The design keeps HBM busy and keeps the per-row math off the issue-bound CUDA-core
// path:
//   * one producer warp streams K/V tiles of 64 positions for one (sequence, kv head) into shared
//     memory with 4-D TMA tiled loads (128-byte swizzle, no multicast), through an NST-deep
//     mbarrier ring (q8 block scales by cp.async; rope-at-read kernels use a ring-aware cp.async
//     producer for everything);
//   * four consumer warps each own 16 positions of a tile.  Scores are computed transposed,
//     S^T = K . Q^T (m16n8k16: positions on M, the GQA group's query rows on N, head_dim on K),
//     so the <= 8 query rows of a group pad only N to 8.  Q (f32) is split hi + lo into two f16
//     operands, so scores keep ~22 bits although K is f16 (or int8 codes);
//   * the output is accumulated transposed too, O^T = V^T . P^T (head_dim on M, rows on N).  The
//     score accumulator of a warp is converted to the P^T operand in registers with movmatrix;
//   * q8: codes enter the MMA as exact f16 integers.  The K block scale (one per 32 values) is
//     applied per block accumulator after the MMA, and the V block scale is folded into P before
//     its f16 conversion, so the q8 math stays exact up to f32/f16 operand rounding of q and p.
// Online softmax in log2 units; the four warps' states are merged in shared memory and written as
// split partials [split][row][D+2] for the LSE merge kernel (shared with the generic path).
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdlib.h>
#include <string.h>

#include "attn.h"
#include "mma.cuh"
#include "tma.cuh"

// CTAs per SM the q8 rope-at-read kernel is compiled for (3: 128 registers, a few spills)
#ifndef BG_ROLL_Q8_MINB
#define BG_ROLL_Q8_MINB 3
#endif

namespace bg {
namespace {

#ifdef BG_TRACE
// Compile-time timing trace (-DBG_TRACE, never in the shipped build): per CTA of the last decode
// launch, 8 u64 records -- [0] entry, [1] first tile ready, [2] last tile consumed, [5] partials
// written (%globaltimer ns); [3] consumer warp 0's cycles waiting on full stages, [4] its cycles in
// the tile loop, [6] SM id, [7] producer cycles waiting on empty stages.  Read with bg_trace_read.
__device__ unsigned long long g_trace[8 * 8192];
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#endif

struct TcParams {
  const void *q;
  int q_f16;
  float *partials;
  uint32_t B, S, H, KV, G, M;
  uint32_t posBase, pos_lo, pos_hi, chunk, row_offset;
  uint32_t nrows_total;
  float sl2;  // softmax scale * log2(e)
  void *out;  // direct mode (single split)
  int out_f16;
  const float *gate;
  // rope-at-read (sink mode): the cp.async producer's view of the cache and the rope tables
  const float *cosT, *sinT;
  const unsigned char *Kp, *Vp;
  const float *Ksp, *Vsp;
  uint64_t seq_stride;
  uint32_t sinks, window, ring_head;
  // peer-exchange step (px.nranks > 0): fused group epilogue, final rows to fout
  PeerArgs px;
  void *fout;
};

// Epilogue of the peer-exchange step, run by the four consumer warps (named barrier 1) of the CTA
// that finished last among the gridDim.x splits of its (sequence, kv head) group:
//   A  merge the group's split partials per row (log-sum-exp) and store each row into slot
//      (step parity, this rank) of every rank's gather buffer over NVLink;
//   B  count each row on every rank (system-scope release after a system fence);
//   C  per row, wait (bounded) until every rank's counter reached this step, merge the nranks rows,
//      apply the gate and write the output;
//   D  free the group's ticket; the last group of this rank to finish advances the step counter.
template <int D>
__device__ __noinline__ void peer_group_epilogue(const TcParams &p, uint32_t b, uint32_t kvh, uint32_t nsplit,
                                                 int tid) {
  constexpr int DPL = D / 32;
  const int warp = tid >> 5, lane = tid & 31;
  const PeerArgs &x = p.px;
  const uint32_t e = *x.step + 1, rows = x.rows;
  auto grow_of = [&](uint32_t n) { return ((uint64_t)b * p.S + n / p.G) * p.H + kvh * p.G + n % p.G; };
  for (uint32_t n = warp; n < p.M; n += 4) {
    const uint64_t g = grow_of(n);
    float acc[DPL], M, L;
    merge_rows<DPL, true>(p.partials + g * (D + 2), (uint64_t)p.nrows_total * (D + 2), nsplit, lane, acc, M, L);
    const uint64_t off = (((uint64_t)(e & 1) * x.nranks + x.rank) * rows + g) * (D + 2);
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
  __threadfence_system();
  asm volatile("bar.sync 1, 128;" ::: "memory");
  for (uint32_t i = tid; i < p.M * x.nranks; i += 128)
    atomicAdd_system(x.flags[i / p.M] + (uint64_t)x.rank * rows + grow_of(i % p.M), 1u);
  for (uint32_t n = warp; n < p.M; n += 4) {
    const uint64_t g = grow_of(n);
    int ok = 1;
    if (lane == 0) ok = peer_wait_row(x, (uint32_t)g, e, &g_device_error);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    float acc[DPL], M = -INFINITY, L = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
    if (ok)
      merge_rows<DPL, true>(x.gather[x.rank] + ((uint64_t)(e & 1) * x.nranks * rows + g) * (D + 2),
                            (uint64_t)rows * (D + 2), x.nranks, lane, acc, M, L);
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const uint64_t i = g * D + lane + 32 * j;
      float o = L > 0.f ? acc[j] / L : 0.f;
      if (p.gate) o = o / (1.0f + expf(-p.gate[i]));
      if (p.out_f16) static_cast<__half *>(p.fout)[i] = __float2half_rn(o);
      else static_cast<float *>(p.fout)[i] = o;
    }
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (tid == 0) {
    x.tickets[blockIdx.y] = 0;
    __threadfence();
    if (atomicAdd(x.done, 1u) == gridDim.y - 1) {
      *x.done = 0;
      __threadfence();
      atomicAdd(x.step, 1u);
    }
  }
}

template <int MODE, int D>
struct Cfg {
  static constexpr int ES = MODE == BG_KV_F16 ? 2 : 1;
  static constexpr int TP = 64;   // positions per tile
  static constexpr int NCW = 4;   // consumer warps, 16 positions each
  static constexpr int ROWB = D * ES;
  static constexpr int NCB = ROWB / 128;       // 128-byte column blocks per row
  static constexpr int KVT = TP * ROWB;        // bytes of the K (or V) tile
  static constexpr int NB = D / 32;            // q8 blocks per row
  static constexpr int SCT = MODE == BG_KV_Q8 ? TP * NB * 4 : 0;
  static constexpr int STAGE = 2 * KVT + 2 * SCT;
  // q8 tiles are half the bytes of f16 ones but need more issue slots per byte: a smaller ring
  // (72 KB) lets 3 CTAs share an SM; f16 keeps 96 KB rings at 2 CTAs per SM.  D = 256 stages are
  // so large that one CTA fills an SM; its ring takes ~200 KB (3 f16 / 5 q8 stages).
  static constexpr int RING = D == 256 ? 204800 : (MODE == BG_KV_Q8 ? 73728 : 98304);
  static constexpr int NST_RAW = RING / STAGE;
  static constexpr int NST = NST_RAW < 2 ? 2 : (NST_RAW > 6 ? 6 : NST_RAW);
  static constexpr int SMEM = NST * STAGE + 1024 /*align*/ + 2 * NST * 8 /*barriers*/ + 16 * NB * 4 /*q8 seeds*/;
};

template <int MODE, int D, int NT, bool ROLL>
__global__ void __launch_bounds__(160, (MODE == BG_KV_Q8 && NT == 1 && D == 128 && !ROLL) ? 3 : (ROLL && NT == 1 ? (MODE == BG_KV_Q8 ? BG_ROLL_Q8_MINB : 2) : 1)) attn_tc_kernel(
                                                      const __grid_constant__ CUtensorMap tmK,
                                                      const __grid_constant__ CUtensorMap tmV,
                                                      const __grid_constant__ CUtensorMap tmKs,
                                                      const __grid_constant__ CUtensorMap tmVs, TcParams p) {
  using C = Cfg<MODE, D>;
  constexpr int TP = C::TP, NST = C::NST, NB = C::NB;
  constexpr int KS = D / 16;  // 16-wide k steps over head_dim
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + NST * C::STAGE);
  uint64_t *empty = full + NST;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t split = blockIdx.x;
  const uint32_t b = blockIdx.y / p.KV, kvh = blockIdx.y % p.KV;
  // No griddepcontrol.launch_dependents: the merge / push kernels are programmatic dependents, but
  // scheduled at this kernel's entry their CTAs sat on the SMs beside the decode and cost ~6 us per
  // 2-GPU config-5b step; with the implicit trigger at exit only their launch overlaps.
  const uint32_t lo = p.pos_lo + split * p.chunk;
  uint32_t hi = min(p.pos_hi, lo + p.chunk);
  hi = min(hi, p.posBase + p.S);
  const int ntiles = hi > lo ? (int)((hi - lo + TP - 1) / TP) : 0;
#ifdef BG_TRACE
  unsigned long long *trc = g_trace + 8 * ((blockIdx.y * gridDim.x + blockIdx.x) & 8191);
  if (tid == 0) {
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    trc[0] = gtime();
    trc[6] = smid;
  }
  long long twait = 0, tloop0 = clock64();
#endif

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      // ROLL: one cp.async arrival per producer lane; q8: lane 0's expect_tx + 32 cp.async arrivals
      mbar_init(&full[s], ROLL ? 32 : (MODE == BG_KV_Q8 ? 33 : 1));
      mbar_init(&empty[s], C::NCW);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == C::NCW && ROLL) {  // ---------------- producer warp (cp.async, ring-aware) ----------------
    // Logical slot -> physical row (sink slots, then the ring); every lane copies 16-byte chunks
    // into the same 128B-swizzled layout TMA would produce; rows past `hi` are zero-filled.
    constexpr int CPR = C::ROWB / 16;  // 16-byte chunks per cache row
    bool ok = true;
    for (int t = 0; t < ntiles && ok; ++t) {
      const int s = t % NST;
      if (t >= NST) ok = mbar_wait_warp(&empty[s], ((t / NST) - 1) & 1);
      if (!ok) break;
      const uint32_t st = smem_u32(smem + s * C::STAGE);
      const uint32_t p0 = lo + t * TP;
      // physical row of tile rows `lane` and `lane + 32` (ring offset < 2*window: one subtraction)
      uint32_t phr[2];
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const uint32_t pl = p0 + lane + 32 * h2;
        uint32_t ph = pl - p.row_offset;
        if (p.window && pl >= p.sinks) {
          uint32_t rel = p.ring_head + (pl - p.sinks);
          if (rel >= p.window) rel -= p.window;
          ph = p.sinks + rel;
        }
        phr[h2] = ph;
      }
      for (int idx = lane; idx < TP * CPR; idx += 32) {
        const int r = idx / CPR, gc = idx % CPR;
        const uint32_t ph = __shfl_sync(0xffffffffu, phr[r >> 5], r & 31);
        const bool valid = p0 + r < hi;
        const uint64_t row = valid ? (((uint64_t)b * p.seq_stride + ph) * p.KV + kvh) : 0;
        const unsigned char *srcK = p.Kp + row * C::ROWB + gc * 16;
        const unsigned char *srcV = p.Vp + row * C::ROWB + gc * 16;
        const uint32_t n = valid ? 16u : 0u;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(swz<TP>(st, r, gc)), "l"(srcK), "r"(n)
                     : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(swz<TP>(st + C::KVT, r, gc)), "l"(srcV),
                     "r"(n)
                     : "memory");
        if constexpr (MODE == BG_KV_Q8) {
          if (gc < NB / 4) {  // the row's block scales: NB floats = NB/4 chunks
            const float *sk = p.Ksp + row * NB + gc * 4, *sv = p.Vsp + row * NB + gc * 4;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(st + 2 * C::KVT + (r * NB + gc * 4) * 4),
                         "l"(sk), "r"(n)
                         : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(st + 2 * C::KVT + C::SCT +
                                                                              (r * NB + gc * 4) * 4),
                         "l"(sv), "r"(n)
                         : "memory");
          }
        }
      }
      asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[s])) : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    return;
  }

  if (warp == C::NCW) {  // ---------------- producer warp ----------------
    // Lane 0 streams the K/V rows with TMA (expect_tx of exactly those bytes).  q8 block scales
    // (16-byte rows) are fetched by all 32 lanes with cp.async and signalled through
    // cp.async.mbarrier.arrive.noinc, so the stage's byte count never depends on how narrow
    // boxes are accounted; rows past the cache extent are zero-filled like TMA's.
    if (ntiles > 0) {
      if (lane == 0) {
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
      }
      bool ok = true;
      for (int t = 0; t < ntiles && ok; ++t) {
        const int s = t % NST;
#ifdef BG_TRACE
        const long long w0 = clock64();
#endif
        if (t >= NST) ok = mbar_wait_warp(&empty[s], ((t / NST) - 1) & 1);
#ifdef BG_TRACE
        twait += clock64() - w0;
#endif
        if (!ok) break;
        unsigned char *st = smem + s * C::STAGE;
        const int z = (int)(lo + t * TP - p.row_offset);
        if (lane == 0) {
          mbar_expect_tx(&full[s], 2 * C::KVT);
#pragma unroll
          for (int cb = 0; cb < C::NCB; ++cb) {
            tma_load_4d(st + cb * TP * 128, &tmK, &full[s], cb * (128 / C::ES), (int)kvh, z, (int)b);
            tma_load_4d(st + C::KVT + cb * TP * 128, &tmV, &full[s], cb * (128 / C::ES), (int)kvh, z, (int)b);
          }
        }
        if constexpr (MODE == BG_KV_Q8) {
          constexpr int CPR = NB / 4;  // 16-byte chunks per scale row
          const uint32_t sbase = smem_u32(st + 2 * C::KVT);
          for (int idx = lane; idx < 2 * TP * CPR; idx += 32) {
            const int which = idx / (TP * CPR), rem = idx % (TP * CPR);
            const int r = rem / CPR, gc = rem % CPR;
            const uint32_t pl = lo + t * TP + r;
            const bool valid = pl < p.pos_hi;
            const uint64_t row = valid ? (((uint64_t)b * p.seq_stride + (pl - p.row_offset)) * p.KV + kvh) : 0;
            const float *src = (which ? p.Vsp : p.Ksp) + row * NB + gc * 4;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sbase + which * C::SCT +
                                                                              (r * NB + gc * 4) * 4),
                         "l"(src), "r"(valid ? 16u : 0u)
                         : "memory");
          }
          asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[s])) : "memory");
        }
      }
      // never leave the CTA with copies in flight: wait (bounded) for the last stages
      if (lane == 0)
        for (int t = max(0, ntiles - NST); t < ntiles; ++t) mbar_wait(&full[t % NST], (t / NST) & 1);
      asm volatile("cp.async.wait_all;" ::: "memory");
#ifdef BG_TRACE
      if (lane == 0) trc[7] = twait;
#endif
    }
    return;
  }

  // ---------------- consumer warps ----------------
  // Q^T operand fragments (B of m16n8k16): column n = lane/4 (query row of the group), k pairs.
  uint32_t qh[NT][KS][2], ql[NT][KS][2];
  uint32_t lim[NT][2];  // last attended position of the lane's two score columns
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const uint32_t r = nt * 8 + (lane >> 2);
    const bool rv = r < p.M;
    const uint32_t qi = rv ? r / p.G : 0, h = kvh * p.G + (rv ? r % p.G : 0);
    const uint64_t qoff = (((uint64_t)b * p.S + qi) * p.H + h) * D;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        // f16 cache: k slots 2j,2j+1 (+8) <-> dims 2j,2j+1 (+8); q8 cache: the byte-pair order of
        // the int8 fragments, dims 4j,4j+1 (half 0) and 4j+2,4j+3 (half 1), j = lane % 4.
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
        qh[nt][ks][half] = pack_f16(__half2float(h0), __half2float(h1));
        ql[nt][ks][half] = pack_f16(x0 - __half2float(h0), x1 - __half2float(h1));
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t rc = nt * 8 + 2 * (lane & 3) + j;
      lim[nt][j] = p.posBase + (rc < p.M ? rc / p.G : p.S - 1);
    }
  }

  // q8: the K accumulators start at -1152 * sum(q over the 32-value block) of their score column,
  // which cancels the +1152 bias of the codes fed to the MMA.  Seeds live in shared memory
  // ([column][block], after the barriers) to keep registers for occupancy.
  float *kcorr_s = reinterpret_cast<float *>(empty + NST);
  if constexpr (MODE == BG_KV_Q8 && !ROLL) {
    for (int idx = tid; idx < NT * 8 * NB; idx += C::NCW * 32) {
      const uint32_t rc = idx / NB, bk = idx % NB;
      float sum = 0.f;
      if (rc < p.M) {
        const uint32_t qi = rc / p.G, h = kvh * p.G + rc % p.G;
        const uint64_t qoff = (((uint64_t)b * p.S + qi) * p.H + h) * D + bk * 32;
        for (int d = 0; d < 32; ++d) {
          const float x = p.q_f16 ? __half2float(static_cast<const __half *>(p.q)[qoff + d])
                                  : static_cast<const float *>(p.q)[qoff + d];
          const float hi = __half2float(__float2half_rn(x));
          sum += hi + __half2float(__float2half_rn(x - hi));
        }
      }
      kcorr_s[idx] = -1152.f * sum;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
  }

  float m[NT][2], l[NT][2];
  float oacc[NT][KS][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m[nt][0] = m[nt][1] = kNegBig;
    l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) oacc[nt][mt][i] = 0.f;
  }

  const int lrow = (((lane >> 3) & 1) << 3) + (lane & 7);  // ldmatrix row for matrices {0,1},{2,3}
  const int lhi = lane >> 4;
  const int trow = ((lane >> 4) << 3) + (lane & 7);         // .trans f16 V: matrices (pos, d) order
  const int tcol = (lane >> 3) & 1;
  bool ok = true;
#ifdef BG_TRACE
  tloop0 = clock64();
#endif
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % NST;
#ifdef BG_TRACE
    const long long w0 = clock64();
#endif
    if (!mbar_wait_warp(&full[s], (t / NST) & 1)) {
      ok = false;
      break;
    }
#ifdef BG_TRACE
    twait += clock64() - w0;
    if (t == 0 && tid == 0) trc[1] = gtime();
#endif
    const uint32_t sb = smem_u32(smem + s * C::STAGE);
    const uint32_t kb = sb, vb = sb + C::KVT;
    const int row0 = warp * 16;
    const uint32_t pa = lo + t * TP + row0 + (lane >> 2), pb = pa + 8;


    // ---- scores S^T[pos][n] ----
    float sc[NT][4];
    if constexpr (ROLL) {
      // rope-at-read by logical slot (attention_sg_roll.wgsl:42-50): dequantise K to f32, rotate
      // each dim with its partner d +- D/2 (held in the same lane and register slot, KS/2 steps
      // away), round to f16 and run the same S^T = K Q^T MMAs.
      constexpr int HALF = D / 2;
      const uint32_t ja = min(pa, hi - 1), jb = min(pb, hi - 1);  // masked tail rows: any valid slot
      const float *ca = p.cosT + (uint64_t)ja * HALF, *sa_ = p.sinT + (uint64_t)ja * HALF;
      const float *cb = p.cosT + (uint64_t)jb * HALF, *sb_ = p.sinT + (uint64_t)jb * HALF;
      // Dims d and d + D/2 of a row sit in k steps ks and ks + KS/2 of the same lane and register
      // slot, so each pair of steps is dequantised, rotated, packed and multiplied before the next
      // pair is touched (keeps ~32 live floats instead of the whole row fragment).
      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
      // element e of a step: {a0.x, a0.y, a1.x, a1.y, a2.x, a2.y, a3.x, a3.y}; a1/a3 hold row b
      auto rotate_mma = [&](float (&lo_f)[8], float (&hi_f)[8], int ks) {
        float cr_[2][4], sr_[2][4];  // [row a/b][dim slot]
        if constexpr (MODE == BG_KV_F16) {
          const int d0 = ks * 16 + 2 * (lane & 3);
#pragma unroll
          for (int rb = 0; rb < 2; ++rb) {
            const float *cc = rb ? cb : ca, *ss = rb ? sb_ : sa_;
            const float2 c0 = __ldg(reinterpret_cast<const float2 *>(cc + d0));
            const float2 c1 = __ldg(reinterpret_cast<const float2 *>(cc + d0 + 8));
            const float2 s0 = __ldg(reinterpret_cast<const float2 *>(ss + d0));
            const float2 s1 = __ldg(reinterpret_cast<const float2 *>(ss + d0 + 8));
            cr_[rb][0] = c0.x; cr_[rb][1] = c0.y; cr_[rb][2] = c1.x; cr_[rb][3] = c1.y;
            sr_[rb][0] = s0.x; sr_[rb][1] = s0.y; sr_[rb][2] = s1.x; sr_[rb][3] = s1.y;
          }
        } else {
          const int d0 = (ks >> 1) * 32 + (ks & 1) * 16 + 4 * (lane & 3);
#pragma unroll
          for (int rb = 0; rb < 2; ++rb) {
            const float4 c4 = __ldg(reinterpret_cast<const float4 *>((rb ? cb : ca) + d0));
            const float4 s4 = __ldg(reinterpret_cast<const float4 *>((rb ? sb_ : sa_) + d0));
            cr_[rb][0] = c4.x; cr_[rb][1] = c4.y; cr_[rb][2] = c4.z; cr_[rb][3] = c4.w;
            sr_[rb][0] = s4.x; sr_[rb][1] = s4.y; sr_[rb][2] = s4.z; sr_[rb][3] = s4.w;
          }
        }
        float rl[8], rh[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
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
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma16816(acc[nt], al, qh[nt][ks][0], qh[nt][ks][1]);
          mma16816(acc[nt], al, ql[nt][ks][0], ql[nt][ks][1]);
          mma16816(acc[nt], ah, qh[nt][ks + KS / 2][0], qh[nt][ks + KS / 2][1]);
          mma16816(acc[nt], ah, ql[nt][ks + KS / 2][0], ql[nt][ks + KS / 2][1]);
        }
      };
      if constexpr (MODE == BG_KV_F16) {
#pragma unroll
        for (int ks = 0; ks < KS / 2; ++ks) {
          uint32_t a[4], a2[4];
          ldsm_x4(a, swz<TP>(kb, row0 + lrow, 2 * ks + lhi));
          ldsm_x4(a2, swz<TP>(kb, row0 + lrow, 2 * (ks + KS / 2) + lhi));
          float lo_f[8], hi_f[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&a[i]));
            const float2 g = __half22float2(*reinterpret_cast<const __half2 *>(&a2[i]));
            lo_f[2 * i] = f.x;
            lo_f[2 * i + 1] = f.y;
            hi_f[2 * i] = g.x;
            hi_f[2 * i + 1] = g.y;
          }
          rotate_mma(lo_f, hi_f, ks);
        }
      } else {
        const float *ksc = reinterpret_cast<const float *>(smem + s * C::STAGE + 2 * C::KVT);
        // snorm8 read: max(code/127, -1) * scale == max(code, -127) * (scale/127); the code is
        // turned into an exact f16 by the 0x64XX trick (value 1152 + code) and unbiased in f16.
        const __half2 bias = __half2(__float2half_rn(1152.f), __float2half_rn(1152.f));
        const __half2 lo127 = __half2(__float2half_rn(-127.f), __float2half_rn(-127.f));
        auto deq = [&](uint32_t w, uint32_t sel) {
          const uint32_t hb = i8pair_biased(w ^ 0x80808080u, sel);
          return __half22float2(__hmax2(__hsub2(*reinterpret_cast<const __half2 *>(&hb), bias), lo127));
        };
#pragma unroll
        for (int bk = 0; bk < NB / 2; ++bk) {
          uint32_t r[4], r2[4];
          ldsm_x4(r, swz<TP>(kb, row0 + lrow, 2 * bk + lhi));
          ldsm_x4(r2, swz<TP>(kb, row0 + lrow, 2 * (bk + NB / 2) + lhi));
          const int ra = (row0 + (lane >> 2)) * NB;
          const float s0 = ksc[ra + bk] * (1.0f / 127.0f), s1 = ksc[ra + 8 * NB + bk] * (1.0f / 127.0f);
          const float t0 = ksc[ra + bk + NB / 2] * (1.0f / 127.0f),
                      t1 = ksc[ra + 8 * NB + bk + NB / 2] * (1.0f / 127.0f);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {  // k step 2bk + h2 from words r[2h2] (row a), r[2h2+1] (row b)
            float lo_f[8], hi_f[8];
            // a0 = bytes 0,1 of row a; a1 = bytes 0,1 of row b; a2 = bytes 2,3 of row a; a3 = row b
            const float2 x0 = deq(r[2 * h2], kSelLo), x1 = deq(r[2 * h2 + 1], kSelLo);
            const float2 x2 = deq(r[2 * h2], kSelHi), x3 = deq(r[2 * h2 + 1], kSelHi);
            const float2 y0 = deq(r2[2 * h2], kSelLo), y1 = deq(r2[2 * h2 + 1], kSelLo);
            const float2 y2 = deq(r2[2 * h2], kSelHi), y3 = deq(r2[2 * h2 + 1], kSelHi);
            lo_f[0] = x0.x * s0; lo_f[1] = x0.y * s0; lo_f[2] = x1.x * s1; lo_f[3] = x1.y * s1;
            lo_f[4] = x2.x * s0; lo_f[5] = x2.y * s0; lo_f[6] = x3.x * s1; lo_f[7] = x3.y * s1;
            hi_f[0] = y0.x * t0; hi_f[1] = y0.y * t0; hi_f[2] = y1.x * t1; hi_f[3] = y1.y * t1;
            hi_f[4] = y2.x * t0; hi_f[5] = y2.y * t0; hi_f[6] = y3.x * t1; hi_f[7] = y3.y * t1;
            rotate_mma(lo_f, hi_f, 2 * bk + h2);
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[nt][i] = acc[nt][i] * p.sl2;
    } else if constexpr (MODE == BG_KV_F16) {
      // hi and lo halves of Q accumulate into separate chains (D = 256 would otherwise chain
      // 32 dependent MMAs per tile)
      float acc[NT][4], acl[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][i] = acl[nt][i] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t a[4];
        ldsm_x4(a, swz<TP>(kb, row0 + lrow, 2 * ks + lhi));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma16816(acc[nt], a, qh[nt][ks][0], qh[nt][ks][1]);
          mma16816(acl[nt], a, ql[nt][ks][0], ql[nt][ks][1]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[nt][i] = (acc[nt][i] + acl[nt][i]) * p.sl2;
    } else {
      const float *ksc = reinterpret_cast<const float *>(smem + s * C::STAGE + 2 * C::KVT);
      float acc[NT][NB][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int bk = 0; bk < NB; ++bk)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[nt][bk][i] = kcorr_s[(nt * 8 + 2 * (lane & 3) + (i & 1)) * NB + bk];
#pragma unroll
      for (int bk = 0; bk < NB; ++bk) {
        uint32_t r[4];
        ldsm_x4(r, swz<TP>(kb, row0 + lrow, 2 * bk + lhi));
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] ^= 0x80808080u;
        const uint32_t a0[4] = {i8pair_biased(r[0], kSelLo), i8pair_biased(r[1], kSelLo),
                                i8pair_biased(r[0], kSelHi), i8pair_biased(r[1], kSelHi)};
        const uint32_t a1[4] = {i8pair_biased(r[2], kSelLo), i8pair_biased(r[3], kSelLo),
                                i8pair_biased(r[2], kSelHi), i8pair_biased(r[3], kSelHi)};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma16816(acc[nt][bk], a0, qh[nt][2 * bk][0], qh[nt][2 * bk][1]);
          mma16816(acc[nt][bk], a0, ql[nt][2 * bk][0], ql[nt][2 * bk][1]);
          mma16816(acc[nt][bk], a1, qh[nt][2 * bk + 1][0], qh[nt][2 * bk + 1][1]);
          mma16816(acc[nt][bk], a1, ql[nt][2 * bk + 1][0], ql[nt][2 * bk + 1][1]);
        }
      }
      float sa[NB], sbv[NB];
#pragma unroll
      for (int bk = 0; bk < NB; ++bk) {
        sa[bk] = ksc[(row0 + (lane >> 2)) * NB + bk] * (p.sl2 * (1.0f / 127.0f));
        sbv[bk] = ksc[(row0 + (lane >> 2) + 8) * NB + bk] * (p.sl2 * (1.0f / 127.0f));
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int bk = 0; bk < NB; ++bk) {
          s0 = fmaf(acc[nt][bk][0], sa[bk], s0);
          s1 = fmaf(acc[nt][bk][1], sa[bk], s1);
          s2 = fmaf(acc[nt][bk][2], sbv[bk], s2);
          s3 = fmaf(acc[nt][bk][3], sbv[bk], s3);
        }
        sc[nt][0] = s0;
        sc[nt][1] = s1;
        sc[nt][2] = s2;
        sc[nt][3] = s3;
      }
    }

    // ---- online softmax (columns n0 = 2(lane%4), n1 = n0+1; rows pa, pb) ----
    float pr[NT][4], cr[NT][2];
    bool moved = false;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float x0 = (pa < hi && pa <= lim[nt][j]) ? sc[nt][j] : -INFINITY;
        float x1 = (pb < hi && pb <= lim[nt][j]) ? sc[nt][2 + j] : -INFINITY;
        float mx = fmaxf(x0, x1);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(m[nt][j], mx);
        const float corr = exp2f(m[nt][j] - mn);
        const float p0 = exp2f(x0 - mn), p1 = exp2f(x1 - mn);
        l[nt][j] = l[nt][j] * corr + p0 + p1;
        m[nt][j] = mn;
        pr[nt][j] = p0;
        pr[nt][2 + j] = p1;
        cr[nt][j] = corr;
        moved |= corr != 1.0f;
      }
    }
    // rescale the output only when some running max of this warp moved (rare after the first
    // tiles of a long context)
    if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int mt = 0; mt < KS; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) oacc[nt][mt][i] *= cr[nt][i & 1];
    }

    // ---- O^T += V^T . P^T ----
    if constexpr (MODE == BG_KV_F16) {
      uint32_t pb0[NT], pb1[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        pb0[nt] = movm_t(pack_f16(pr[nt][0], pr[nt][1]));
        pb1[nt] = movm_t(pack_f16(pr[nt][2], pr[nt][3]));
      }
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
        uint32_t a[4];
        ldsm_x4_t(a, swz<TP>(vb, row0 + trow, 2 * mt + tcol));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816(oacc[nt][mt], a, pb0[nt], pb1[nt]);
      }
    } else {
      const float *vsc = reinterpret_cast<const float *>(smem + s * C::STAGE + 2 * C::KVT + C::SCT);
#pragma unroll
      for (int bk = 0; bk < NB; ++bk) {
        const float va = vsc[(row0 + (lane >> 2)) * NB + bk] * (1.0f / 127.0f);
        const float vbb = vsc[(row0 + (lane >> 2) + 8) * NB + bk] * (1.0f / 127.0f);
        uint32_t pb0[NT], pb1[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          pb0[nt] = movm_t(pack_f16(pr[nt][0] * va, pr[nt][1] * va));
          pb1[nt] = movm_t(pack_f16(pr[nt][2] * vbb, pr[nt][3] * vbb));
        }
        uint32_t r[4];
        ldsm_x4_t(r, swz<TP>(vb, row0 + lrow, 2 * bk + lhi));
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] ^= 0x80808080u;
        const uint32_t a0[4] = {i8pair_biased(r[0], kSelEven), i8pair_biased(r[0], kSelOdd),
                                i8pair_biased(r[1], kSelEven), i8pair_biased(r[1], kSelOdd)};
        const uint32_t a1[4] = {i8pair_biased(r[2], kSelEven), i8pair_biased(r[2], kSelOdd),
                                i8pair_biased(r[3], kSelEven), i8pair_biased(r[3], kSelOdd)};
        const uint32_t ng = kNeg1152x2();
        const uint32_t aneg[4] = {ng, ng, ng, ng};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma16816(oacc[nt][2 * bk], a0, pb0[nt], pb1[nt]);
          mma16816(oacc[nt][2 * bk], aneg, pb0[nt], pb1[nt]);
          mma16816(oacc[nt][2 * bk + 1], a1, pb0[nt], pb1[nt]);
          mma16816(oacc[nt][2 * bk + 1], aneg, pb0[nt], pb1[nt]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

#ifdef BG_TRACE
  if (tid == 0) {
    trc[2] = gtime();
    trc[3] = twait;
    trc[4] = clock64() - tloop0;
  }
#endif
  // ---- merge the four warps' states; write split partials ----
  // (1) each warp's (m, l) per column; (2) every lane rescales its own o by exp2(m_warp - M) once
  // per column and stores it, warp 0 keeps the merged (M, L) per column; (3) each output element
  // is the plain sum of the four scaled values, four columns per thread.  Row stride D + 4 keeps
  // the stores of (2) on distinct banks.
  constexpr int NN = NT * 8, DP = D + 4;
  asm volatile("bar.sync 1, 128;" ::: "memory");  // all consumers done with the stages
  float *ep = reinterpret_cast<float *>(smem);     // [NCW][NN][DP] scaled o
  float *mw = ep + C::NCW * NN * DP;               // [NCW][NN] m (log2 units)
  float *lw = mw + C::NCW * NN;                    // [NCW][NN] l
  float *mrow = lw + C::NCW * NN, *lsrow = mrow + NN;  // [NN] merged M, L
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float lt = l[nt][j];
      lt += __shfl_xor_sync(0xffffffffu, lt, 4);
      lt += __shfl_xor_sync(0xffffffffu, lt, 8);
      lt += __shfl_xor_sync(0xffffffffu, lt, 16);
      const int n = nt * 8 + 2 * (lane & 3) + j;
      if (lane < 4) {
        mw[warp * NN + n] = ok ? m[nt][j] : kNegBig;
        lw[warp * NN + n] = ok ? lt : 0.f;  // timed out: an empty partial
      }
    }
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = nt * 8 + 2 * (lane & 3) + j;
      float M = kNegBig;
#pragma unroll
      for (int w = 0; w < C::NCW; ++w) M = fmaxf(M, mw[w * NN + n]);
      const float f = ok ? exp2f(mw[warp * NN + n] - M) : 0.f;
      if (warp == 0 && lane < 4) {
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < C::NCW; ++w) L = fmaf(lw[w * NN + n], exp2f(mw[w * NN + n] - M), L);
        mrow[n] = M;
        lsrow[n] = L;
      }
      float *mine = ep + (warp * NN + n) * DP;
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int d = MODE == BG_KV_F16 ? mt * 16 + (lane >> 2) + 8 * hh : mt * 16 + 2 * (lane >> 2) + hh;
          mine[d] = oacc[nt][mt][2 * hh + j] * f;
        }
      }
    }
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  for (int idx = tid; idx < (int)p.M * (D / 4); idx += C::NCW * 32) {
    const int n = idx / (D / 4), d = (idx % (D / 4)) * 4;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < C::NCW; ++w) {
      const float4 x = *reinterpret_cast<const float4 *>(ep + (w * NN + n) * DP + d);
      o.x += x.x; o.y += x.y; o.z += x.z; o.w += x.w;
    }
    const float M = mrow[n], L = lsrow[n];
    const uint32_t qi = n / p.G, h = kvh * p.G + n % p.G;
    const uint64_t grow = ((uint64_t)b * p.S + qi) * p.H + h;
    if (p.out) {  // single split: final output
      const float inv = L > 0.f ? 1.0f / L : 0.f;  // L == 0 only after a timed-out wait (BG_ETIMEOUT)
      float v[4] = {o.x * inv, o.y * inv, o.z * inv, o.w * inv};
      if (p.gate) {
        const float4 g = *reinterpret_cast<const float4 *>(p.gate + grow * D + d);
        const float gg[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = v[i] / (1.0f + expf(-gg[i]));
      }
      if (p.out_f16) {
        const uint2 hv = make_uint2(pack_f16(v[0], v[1]), pack_f16(v[2], v[3]));
        *reinterpret_cast<uint2 *>(static_cast<__half *>(p.out) + grow * D + d) = hv;
      } else {
        *reinterpret_cast<float4 *>(static_cast<float *>(p.out) + grow * D + d) = make_float4(v[0], v[1], v[2], v[3]);
      }
      continue;
    }
    float *dst = p.partials + ((uint64_t)split * p.nrows_total + grow) * (D + 2);
    *reinterpret_cast<float2 *>(dst + d) = make_float2(o.x, o.y);
    *reinterpret_cast<float2 *>(dst + d + 2) = make_float2(o.z, o.w);
    if (d == 0) *reinterpret_cast<float2 *>(dst + D) = make_float2(L > 0.f ? M * kLn2 : -INFINITY, L);
  }
#ifdef BG_TRACE
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (tid == 0) trc[5] = gtime();
#endif
  if constexpr (!ROLL) {
    if (p.px.nranks) {
      // the group's last CTA (a ticket per (sequence, kv head)) finishes the whole step
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      volatile int *last = reinterpret_cast<volatile int *>(smem);  // ep is no longer read
      if (tid == 0) *last = atomicAdd(p.px.tickets + blockIdx.y, 1u) == gridDim.x - 1;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (*last) {
        __threadfence();
        peer_group_epilogue<D>(p, b, kvh, gridDim.x, tid);
      }
    }
  }
}

template <int MODE, int D, int NT, bool ROLL>
int launch_cfg(const AttnArgs &a, cudaStream_t st) {
  using C = Cfg<MODE, D>;
  CUtensorMap tk, tv, tks, tvs;
  if (!ROLL) {
  const uint64_t Lvalid = a.pos_hi - a.kv.row_offset;
  const uint64_t dims[4] = {a.D, a.KV, Lvalid, a.B};
  const uint64_t rb = (uint64_t)a.D * C::ES;
  const uint64_t strides[3] = {rb, rb * a.KV, rb * a.KV * a.kv.seq_stride};
  const uint32_t box[4] = {128 / C::ES, 1, C::TP, 1};
  const CUtensorMapDataType dt = MODE == BG_KV_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  if (make_tmap_4d(&tk, dt, a.kv.K, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return BG_EUNSUPPORTED;
  if (make_tmap_4d(&tv, dt, a.kv.V, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return BG_EUNSUPPORTED;
  tks = tk;  // the q8 block scales travel by cp.async (see the producer), not TMA
  tvs = tv;
  } else {
    memset(&tk, 0, sizeof(tk));  // the cp.async producer of the ROLL kernels uses no tensor map
    tv = tks = tvs = tk;
  }
  // the epilogue stores four columns at once: 16-byte aligned rows of out / gate, 8-byte partials
  if (((uintptr_t)a.out | (uintptr_t)a.gate) & 15 || (uintptr_t)a.partials & 7) return BG_EUNSUPPORTED;
  TcParams p;
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
  p.pos_hi = a.pos_hi;
  p.chunk = a.chunk;
  p.row_offset = a.kv.row_offset;
  p.nrows_total = a.B * a.S * a.H;
  p.sl2 = a.scale * kLog2e;
  p.out = a.out;
  p.out_f16 = a.out_f16;
  p.gate = a.gate;
  p.cosT = a.cosT;
  p.sinT = a.sinT;
  p.Kp = static_cast<const unsigned char *>(a.kv.K);
  p.Vp = static_cast<const unsigned char *>(a.kv.V);
  p.Ksp = a.kv.Ks;
  p.Vsp = a.kv.Vs;
  p.seq_stride = a.kv.seq_stride;
  p.sinks = a.kv.sinks;
  p.window = a.kv.window;
  p.ring_head = a.kv.ring_head;
  p.px = a.px;
  p.fout = a.fout;
  auto kern = attn_tc_kernel<MODE, D, NT, ROLL>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
    return BG_ELAUNCH;
  kern<<<dim3(a.nsplit, a.B * a.KV), 160, C::SMEM, st>>>(tk, tv, tks, tvs, p);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

template <int MODE, int D, int NT, bool ROLL = false>
int occupancy() {
  using C = Cfg<MODE, D>;
  static int cached = 0;
  if (!cached) {
    int n = 0;
    auto kern = attn_tc_kernel<MODE, D, NT, ROLL>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, 160, C::SMEM) != cudaSuccess || n < 1) n = 1;
    cached = n;
  }
  return cached;
}

template <int MODE>
int launch_mode(const AttnArgs &a, uint32_t M, cudaStream_t st) {
  const bool roll = a.cosT != nullptr || a.kv.window != 0;
  if (roll) {
    if (a.D != 128 || !a.cosT) return BG_EUNSUPPORTED;  // ring without rope-at-read: generic path
    return M <= 8 ? launch_cfg<MODE, 128, 1, true>(a, st) : launch_cfg<MODE, 128, 2, true>(a, st);
  }
  if (a.D == 128) return M <= 8 ? launch_cfg<MODE, 128, 1, false>(a, st) : launch_cfg<MODE, 128, 2, false>(a, st);
  if (a.D == 256 && M <= 8) return launch_cfg<MODE, 256, 1, false>(a, st);
  return BG_EUNSUPPORTED;
}

}  // namespace

bool attn_tc_supported(int mode, uint32_t D, uint32_t S, uint32_t H, uint32_t KV, bool roll, bool ring) {
  if (mode != BG_KV_F16 && mode != BG_KV_Q8) return false;
  const uint32_t M = S * (H / KV);
  if (roll || ring) return roll && D == 128 && M <= 16;  // rope-at-read kernels (cp.async producer)
  if (D == 128) return M <= 16;
  if (D == 256) return M <= 8;
  return false;
}

int attn_tc_ctas_per_sm(int mode, uint32_t D, uint32_t M, bool roll) {
  if (roll) {
    if (mode == BG_KV_F16) return M <= 8 ? occupancy<BG_KV_F16, 128, 1, true>() : occupancy<BG_KV_F16, 128, 2, true>();
    return M <= 8 ? occupancy<BG_KV_Q8, 128, 1, true>() : occupancy<BG_KV_Q8, 128, 2, true>();
  }
  if (mode == BG_KV_F16) {
    if (D == 256) return occupancy<BG_KV_F16, 256, 1>();
    return M <= 8 ? occupancy<BG_KV_F16, 128, 1>() : occupancy<BG_KV_F16, 128, 2>();
  }
  if (D == 256) return occupancy<BG_KV_Q8, 256, 1>();
  return M <= 8 ? occupancy<BG_KV_Q8, 128, 1>() : occupancy<BG_KV_Q8, 128, 2>();
}

bool roll_legacy() {
  static const bool v = [] {
    const char *e = getenv("BGATTN_ROLL_LEGACY");  // one-head-per-CTA rope-at-read kernel (A/B)
    return e && *e == '1';
  }();
  return v;
}

int launch_attn_tc(const AttnArgs &a, cudaStream_t st) {
  if (!attn_tc_supported(a.mode, a.D, a.S, a.H, a.KV, a.cosT != nullptr, a.kv.window != 0)) return BG_EUNSUPPORTED;
  if (a.cosT && !roll_legacy()) {
    const int rc = launch_attn_roll(a, st);
    if (rc != BG_EUNSUPPORTED) return rc;
  }
  const uint32_t M = a.S * (a.H / a.KV);
  return a.mode == BG_KV_F16 ? launch_mode<BG_KV_F16>(a, M, st) : launch_mode<BG_KV_Q8>(a, M, st);
}

int poll_device_error_attn_tc() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return BG_ELAUNCH;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  return v;
}

}  // namespace bg

#ifdef BG_TRACE
extern "C" int bg_trace_read(unsigned long long *dst, size_t n) {
  return cudaMemcpyFromSymbol(dst, bg::g_trace, n * sizeof(unsigned long long)) == cudaSuccess ? 0 : -1;
}
#endif
