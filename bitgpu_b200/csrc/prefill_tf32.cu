// Causal prefill attention over an f32 KV cache on the tensor cores in 3xTF32 (tcgen05 kind::tf32).
//
// Path: layer() prefill (src/engine.ts:1580) with the f32 cache (shaders/attention_sg.wgsl /
// attention_wg.wgsl: f32 queries, f32 K/V, f32 math).  A plain TF32 product keeps 11 significant
// bits of each operand; the split x = hi + lo with hi = tf32(x), lo = x - hi keeps ~22, and the
// three largest partial products give the f32-class result:
//   S  = Qhi Khi^T + Qlo Khi^T + Qhi Klo^T        (48 MMAs of 128 x 32 x 8 per key tile)
//   O += Phi Vhi + Phi Vlo + Plo Vhi              (12 MMAs of 128 x 128 x 8)
// head_dim 128.  CTA = (head h, 128 query rows, sequence b); key tiles of 32 positions.
//   TMEM (512 columns): Qhi [0,128), Qlo [128,256), O [256,384), S0 [384,416), S1 [416,448),
//                       Plo0 [448,480), Plo1 [480,512).  The S products read Q straight from
//                       tensor memory (TS form); P hi overwrites its S slot, P lo sits beside it.
//   warp 1      MMA issuer (one thread); S double-buffered, S(j+1) overlaps softmax(j)
//   warp 2      TMEM allocator
//   warps 4-7   Q -> (hi, lo) into TMEM at start, then the softmax (one query row per thread)
//   warps 8-11  operand split: each thread loads its share of the next K/V tile from global memory
//               into registers while it writes the current one into a 3-stage operand ring -- K hi /
//               lo K-major as stored, V hi / lo transposed to K-major [d][key] (the B operand of
//               P V).  Rows past Ltot are zero.
// All mbarrier waits are bounded; on expiry the CTA records BG_ETIMEOUT, stops issuing work, waits
// for what it already issued, frees its TMEM and exits.
#include "prefill.h"
#include "tma.cuh"
#include "umma.cuh"

namespace bg {
namespace {

constexpr int kD = 128;
constexpr int kRows = 128;
constexpr int kKT = 32;                    // positions per key tile
constexpr int kThreads = 384;
constexpr int kTile = kKT * kD * 4;        // 16 KB: one f32 32 x 128 tile
constexpr float kRescaleThreshold = 8.0f;  // log2 units

constexpr int kOpStages = 3;

struct Tf32Smem {
  // operand ring: Khi, Klo, VhiT, VloT per stage
  static constexpr int KHI = 0, KLO = kTile, VHI = 2 * kTile, VLO = 3 * kTile, OP_STAGE = 4 * kTile;
  static constexpr int BAR = kOpStages * OP_STAGE;
  static constexpr int TOTAL = BAR + 256;
};

constexpr uint32_t kTQhi = 0, kTQlo = 128, kTO = 256, kTS0 = 384, kTS1 = 416, kTPlo0 = 448, kTPlo1 = 480;

struct Tf32Params {
  const float *K, *V;
  uint64_t seq_stride;
  uint32_t KV;
  const void *q;
  int q_f32;
  const float *gate;
  void *out;
  int out_f16;
  uint32_t S, H, G, posBase, Ltot;
  float sl2;
};

__device__ __forceinline__ float tf32_rna(float x) {  // round to the nearest tf32 (ties away)
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_tf32_kernel(Tf32Params p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + Tf32Smem::BAR);
  uint64_t *conv_full = bars + 6;   // [3] split operands written
  uint64_t *kv_empty = bars + 3;    // [3] operand stage free (MMAs done)
  uint64_t *s_full = bars + 10;     // [2]
  uint64_t *p_full = bars + 12;     // [2]
  uint64_t *o_done = bars + 14;     // [1]
  uint64_t *q_full = bars + 15;     // [1] Q hi / lo in TMEM
  uint64_t *mma_done = bars + 16;   // [1]
  uint32_t *tmem_base_s = reinterpret_cast<uint32_t *>(bars + 17);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 18);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t h = blockIdx.x;
  const uint32_t qblk = gridDim.y - 1 - blockIdx.y;  // heaviest query blocks first
  const uint32_t b = blockIdx.z;
  const uint32_t kvh = h / p.G;
  const uint32_t q0 = qblk * kRows;
  const uint32_t last_key = min(p.posBase + q0 + kRows, p.Ltot);
  const int ntiles = (int)((last_key + kKT - 1) / kKT);

  if (tid == 0) {
    for (int i = 0; i < kOpStages; ++i) {
      mbar_init(&conv_full[i], 4);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
    }
    mbar_init(o_done, 1);
    mbar_init(q_full, 128);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_base_s)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 72;" ::: "memory");
    if (warp == 1 && lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idS = idesc_tf32(kKT), idO = idesc_tf32(kD);
      const uint32_t s0 = smem_u32(sm);
      auto issue_s = [&](uint32_t slot, uint32_t sb) {
        // (A from TMEM, B = K tile K-major) x 3 terms, 16 K-steps of 8 elements (32 B) each
#pragma unroll
        for (int term = 0; term < 3; ++term) {
          const uint32_t qa = tmem + (term == 1 ? kTQlo : kTQhi);
          const uint32_t kb = sb + (term == 2 ? Tf32Smem::KLO : Tf32Smem::KHI);
#pragma unroll
          for (int kk = 0; kk < kD / 8; ++kk) {
            const uint64_t bd = umma_desc_sw128(kb + (kk >> 2) * (kKT * 128) + (kk & 3) * 32, 16, 1024);
            umma_ts_tf32(tmem + slot, qa + kk * 8, bd, idS, (term > 0 || kk > 0) ? 1u : 0u);
          }
        }
      };
      auto issue_pv = [&](uint32_t slot, uint32_t plo, uint32_t sb, bool acc) {
        // Phi Vhi, Phi Vlo, Plo Vhi
#pragma unroll
        for (int term = 0; term < 3; ++term) {
          const uint32_t vb = sb + (term == 1 ? Tf32Smem::VLO : Tf32Smem::VHI);
          const uint32_t pa = tmem + (term == 2 ? plo : slot);
#pragma unroll
          for (int kk = 0; kk < kKT / 8; ++kk) {
            const uint64_t bd = umma_desc_sw128(vb + kk * 32, 16, 1024);
            umma_ts_tf32(tmem + kTO, pa + kk * 8, bd, idO, (acc || term > 0 || kk > 0) ? 1u : 0u);
          }
        }
      };
      bool ok = mbar_wait(q_full, 0) && mbar_wait(&conv_full[0], 0);
      tc_fence_after();
      int j = 0;
      if (ok && ntiles > 0) {
        issue_s(kTS0, s0);
        umma_commit(&s_full[0]);
      }
      for (; ok && j < ntiles; ++j) {
        const int st = j & 1, os = j % kOpStages, os1 = (j + 1) % kOpStages;
        if (j + 1 < ntiles) {
          if (!mbar_wait(&conv_full[os1], ((j + 1) / kOpStages) & 1)) { ok = false; break; }
          tc_fence_after();
          issue_s(st ? kTS0 : kTS1, s0 + os1 * Tf32Smem::OP_STAGE);
          umma_commit(&s_full[st ^ 1]);
        }
        if (!mbar_wait(&p_full[st], (j >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
        issue_pv(st ? kTS1 : kTS0, st ? kTPlo1 : kTPlo0, s0 + os * Tf32Smem::OP_STAGE, j > 0);
        umma_commit(o_done);
        umma_commit(&kv_empty[os]);
      }
      if (!ok) *abort_flag = 1;
      umma_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
  } else if (warp >= 8) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 216;" ::: "memory");
    // ---------------- operand split ----------------
    // thread ct: K chunks idx = ct + 128*i (key idx/32, 16-byte chunk idx%32 of the 512-byte row),
    // coalesced; V: key ct%32, d-group (ct/32) + 4*i, one row per lane (the transposed write is
    // then conflict-free across the warp).
    const int ct = tid - 256;
    const int vkey = ct & 31;
    float4 kr[8], vr[8];
    auto load_tile = [&](int j) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = ct + 128 * i, key = idx >> 5, c4 = idx & 31;
        const uint32_t pos = j * kKT + key;
        kr[i] = pos < p.Ltot ? __ldg(reinterpret_cast<const float4 *>(
                                   p.K + (((uint64_t)b * p.seq_stride + pos) * p.KV + kvh) * kD + c4 * 4))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        const uint32_t vpos = j * kKT + vkey;
        const int d4 = (ct >> 5) + 4 * i;
        vr[i] = vpos < p.Ltot ? __ldg(reinterpret_cast<const float4 *>(
                                    p.V + (((uint64_t)b * p.seq_stride + vpos) * p.KV + kvh) * kD + d4 * 4))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    };
    if (ntiles > 0) load_tile(0);
    for (int j = 0; j < ntiles; ++j) {
      const int os = j % kOpStages;
      if (j >= kOpStages && !mbar_wait_warp(&kv_empty[os], ((j / kOpStages) - 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      unsigned char *ob = sm + os * Tf32Smem::OP_STAGE;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = ct + 128 * i, key = idx >> 5, c4 = idx & 31;
        const uint32_t o = (c4 >> 3) * (kKT * 128) + key * 128 + (((c4 & 7) ^ (key & 7)) << 4);
        const float4 x = kr[i];
        const float4 hi = make_float4(tf32_rna(x.x), tf32_rna(x.y), tf32_rna(x.z), tf32_rna(x.w));
        *reinterpret_cast<float4 *>(ob + Tf32Smem::KHI + o) = hi;
        *reinterpret_cast<float4 *>(ob + Tf32Smem::KLO + o) = make_float4(x.x - hi.x, x.y - hi.y, x.z - hi.z, x.w - hi.w);
        const int d = 4 * ((ct >> 5) + 4 * i);
        const float xs[4] = {vr[i].x, vr[i].y, vr[i].z, vr[i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int dd = d + e;
          const uint32_t ov = dd * 128 + ((((vkey >> 2) ^ (dd & 7))) << 4) + (vkey & 3) * 4;
          const float hv = tf32_rna(xs[e]);
          *reinterpret_cast<float *>(ob + Tf32Smem::VHI + ov) = hv;
          *reinterpret_cast<float *>(ob + Tf32Smem::VLO + ov) = xs[e] - hv;
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv_full[os]);
      if (j + 1 < ntiles) load_tile(j + 1);  // in flight while the next stage frees up
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 216;" ::: "memory");
    // ---------------- Q split into TMEM, then the softmax (one query row per thread) ----------
    const int row = ((warp & 3) << 5) + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) << 5) << 16;
    const uint32_t qrow = q0 + row;
    const uint32_t qpos = p.posBase + qrow;
    {
      const uint64_t e0 = (((uint64_t)b * p.S + qrow) * p.H + h) * kD;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
          if (qrow < p.S) {
            if (p.q_f32) {
              x = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(p.q) + e0 + c * 32 + i));
            } else {
              const uint2 hv = __ldg(reinterpret_cast<const uint2 *>(static_cast<const __half *>(p.q) + e0 + c * 32 + i));
              const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&hv.x));
              const float2 bb = __half22float2(*reinterpret_cast<const __half2 *>(&hv.y));
              x = make_float4(a.x, a.y, bb.x, bb.y);
            }
          }
          const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float hv = tf32_rna(xs[e]);
            hi[i + e] = __float_as_uint(hv);
            lo[i + e] = __float_as_uint(xs[e] - hv);
          }
        }
        tmem_st32((tmem + kTQhi + c * 32) | lane_off, hi);
        tmem_st32((tmem + kTQlo + c * 32) | lane_off, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(q_full);
    }
    const float sl2 = p.sl2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1;
      if (!mbar_wait_warp(&s_full[st], (j >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      const uint32_t sbase = (tmem + (st ? kTS1 : kTS0)) | lane_off;
      const int nvalid = min(kKT, max(0, (int)qpos - j * kKT + 1));
      uint32_t r[32];
      tmem_ld32(sbase, r);
      tmem_wait_ld();
      if (nvalid < kKT) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i >= nvalid) r[i] = __float_as_uint(-INFINITY);
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < 32; i += 2) mx4[(i >> 1) & 3] = fmax3(mx4[(i >> 1) & 3], __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
      const float mt = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;
      const bool need = mt > m_used + kRescaleThreshold;
      // S(j) was issued before PV(j-1), so PV(j-1) may still run.  Its o_done phase is consumed
      // exactly once, in order (before touching O, or at the end of this step), so that no wait
      // on o_done can be two phases behind the barrier.
      bool pv_prev_done = j == 0;
      if (__any_sync(0xffffffffu, need)) {
        if (j > 0) {
          if (!mbar_wait_warp(o_done, (j - 1) & 1)) { ok = false; break; }
          pv_prev_done = true;
          tc_fence_after();
          const float f = (need && m_used > -INFINITY) ? ex2_approx(m_used - mt) : 1.0f;
          const uint32_t obase = (tmem + kTO) | lane_off;
#pragma unroll 1
          for (int c = 0; c < kD / 32; ++c) {
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
      float ls0 = 0.f, ls1 = 0.f;
      uint32_t plo[32];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(r[i]), sl2, mneg));
        const float p1 = ex2_approx(fmaf(__uint_as_float(r[i + 1]), sl2, mneg));
        ls0 += p0;
        ls1 += p1;
        const float h0 = tf32_rna(p0), h1 = tf32_rna(p1);
        r[i] = __float_as_uint(h0);
        r[i + 1] = __float_as_uint(h1);
        plo[i] = __float_as_uint(p0 - h0);
        plo[i + 1] = __float_as_uint(p1 - h1);
      }
      tmem_st32(sbase, r);
      tmem_st32((tmem + (st ? kTPlo1 : kTPlo0)) | lane_off, plo);
      l += ls0 + ls1;
      tmem_wait_st();
      if (!pv_prev_done && !mbar_wait_warp(o_done, (j - 1) & 1)) { ok = false; break; }
      tc_fence_before();
      mbar_arrive(&p_full[st]);
    }
    if (ok && ntiles > 0 && mbar_wait_warp(o_done, (ntiles - 1) & 1)) {
      tc_fence_after();
      const uint32_t obase = (tmem + kTO) | lane_off;
      const float inv = 1.0f / l;
      const bool valid = qrow < p.S;
      const uint64_t orow = (((uint64_t)b * p.S + qrow) * p.H + h) * kD;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

}  // namespace

int launch_prefill_tf32(const PrefillArgs &a, cudaStream_t st) {
  if (a.D != kD) return BG_EUNSUPPORTED;
  Tf32Params p;
  p.K = static_cast<const float *>(a.K);
  p.V = static_cast<const float *>(a.V);
  p.seq_stride = a.seq_stride;
  p.KV = a.KV;
  p.q = a.q;
  p.q_f32 = a.q_f32;
  p.gate = a.gate;
  p.out = a.out;
  p.out_f16 = a.out_f16;
  p.S = a.S;
  p.H = a.H;
  p.G = a.H / a.KV;
  p.posBase = a.posBase;
  p.Ltot = a.Ltot;
  p.sl2 = a.scale * kLog2e;
  const int smem = Tf32Smem::TOTAL + 1024;
  if (cudaFuncSetAttribute(prefill_tf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return BG_ELAUNCH;
  dim3 grid(a.H, (a.S + kRows - 1) / kRows, a.B);
  prefill_tf32_kernel<<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int poll_device_error_prefill_tf32() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return BG_ELAUNCH;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  return v;
}

}  // namespace bg
