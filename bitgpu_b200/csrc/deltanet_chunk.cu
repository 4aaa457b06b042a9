// Chunked (WY) gated-DeltaNet prefill: the chunk-parallel form of the delta rule that bitgpu's
// numpy oracle implements as tools/qwen35_numpy.py:144-187 (_delta_chunk, == HF
// torch_chunk_gated_delta_rule), extended with an initial state.  The recurrent kernel
// (deltanet.cu) is sequential over every token; here only the state hand-off between chunks of
// C = 64 tokens is sequential, everything inside a chunk is dense f32 arithmetic.
//
//   norm kernel   Kn = l2norm(k), Qn = l2norm(q)/sqrt(DK) once per (token, key head)
//   prep kernel   one CTA per (chunk, value head), all independent:
//                 g/beta from a/b (fused gbeta), gc = cumsum(g) within the chunk,
//                 M[i][j] = -beta_i (Kn_i . Kn_j) exp(gc_i - gc_j)   (j < i),
//                 Aqk[i][j] = (Qn_i . Kn_j) exp(gc_i - gc_j)   (j <= i),
//                 U = (I - M)^-1 (beta V),  W = (I - M)^-1 (beta exp(gc) Kn) by forward
//                 substitution (the reference forms T = (I - M)^-1 by a row recurrence,
//                 qwen35_numpy.py:168-173, then multiplies)  -> workspace {U, W, Aqk, gc}
//   scan kernel   one CTA per (value head, 64 state columns), chunks in order:
//                 Vn = U - W S;  O = (Qn exp(gc)) S + Aqk Vn;
//                 S  = S exp(gc_last) + (Kn exp(gc_last - gc))^T Vn      (qwen35_numpy.py:177-185)
// Value head h reads key/query head h % HK (tile GQA, shaders/deltanet_recur.wgsl:27).
// Arithmetic is f32 on the CUDA cores (the reference computes in float32).
#include <math.h>
#include <stdlib.h>

#include <cuda.h>

#include "kv.h"
#include "tma.cuh"
#include "umma.cuh"

namespace bg {
namespace {

constexpr int C = 64;    // chunk length (the reference's chunk=64)
constexpr int DKc = 128; // key / value head dims this path is built for
constexpr int DVc = 128;

struct ChunkArgs {
  uint32_t S, H, HK, nc;
  const float *q, *k, *v, *a, *b, *a_neg, *dt_bias;
  const float *state_in;
  float *state_out, *core;
  float *U, *W, *Aqk, *gcum;  // workspace, per (head, chunk)
  float *KT;                  // workspace: (Kn exp(gc_last - gc))^T per (head, chunk), [DK][C]
  float *QN, *KN;             // workspace: l2-normalised q (x 1/sqrt(DK)) and k, [S][HK][DK]
};

__device__ __forceinline__ float softplus_s(float x) { return fmaxf(x, 0.f) + logf(1.0f + expf(-fabsf(x))); }

// One warp per (token, key head): Kn = l2norm(k), Qn = l2norm(q) / sqrt(DK)  (qwen35_numpy.py:66-68,131)
__global__ void dn_norm_qk(ChunkArgs p) {
  const uint64_t row = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= (uint64_t)p.S * p.HK) return;
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const float *src = (w ? p.q : p.k) + row * DKc + lane * 4;
    const float4 v = *reinterpret_cast<const float4 *>(src);
    float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    ss = warp_sum(ss);
    const float inv = (1.0f / sqrtf(ss + 1e-6f)) * (w ? 1.0f / sqrtf((float)DKc) : 1.0f);
    *reinterpret_cast<float4 *>((w ? p.QN : p.KN) + row * DKc + lane * 4) =
        make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
  }
}

__device__ __forceinline__ void cp16(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(valid ? 16u : 0u)
               : "memory");
}

constexpr int KP = DKc + 4;   // row stride (floats) of 128-wide tiles: 16-byte rows, 4-bank skew
constexpr int CP = C + 4;     // row stride of 64-wide tiles

__device__ __forceinline__ float4 lds4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

// Per (chunk, value head), 256 threads.
//   K Kn^T and Qn Kn^T: 4 x 4 register tiles (rows 4*(tid/16) + u, cols tid%16 + 16*v), float4
//   loads along dk; the epilogue applies the decays and beta:
//     M[i][j]   = -beta_i (Kn_i . Kn_j) exp(gc_i - gc_j)   (j < i, else 0)
//     Aqk[i][j] =  (Qn_i . Kn_j) exp(gc_i - gc_j)           (j <= i, else 0)
//   U = (I - M)^-1 (beta V) and W = (I - M)^-1 (beta exp(gc) Kn) by forward substitution over the
//   64 rows: thread = one column of U (tid < 128) or of W, its 64 rows in registers, M rows read as
//   warp broadcasts; no barrier inside.  (I - M)^-1 is the T of qwen35_numpy.py:168-173: its row
//   recurrence computes T' = M + M T', i.e. T = T' + I = (I - M)^-1.
__global__ void __launch_bounds__(256, 2) dn_chunk_prep(ChunkArgs p) {
  extern __shared__ __align__(16) float sm[];
  float *kn = sm;              // [C][KP]
  float *qn = kn + C * KP;     // [C][KP]
  float *M = qn + C * KP;      // [C][CP]
  float *gc = M + C * CP;      // [C]
  float *beta = gc + C;        // [C]
  const uint32_t c = blockIdx.x, hk = blockIdx.y;
  const uint32_t t0 = c * C;
  const int tid = threadIdx.x;

  for (int idx = tid; idx < C * (DKc / 4); idx += blockDim.x) {
    const int r = idx / (DKc / 4), c4 = idx % (DKc / 4);
    const uint32_t t = t0 + r;
    const uint64_t off = ((uint64_t)(t < p.S ? t : 0) * p.HK + hk) * DKc + c4 * 4;
    cp16(kn + r * KP + c4 * 4, p.KN + off, t < p.S);
    cp16(qn + r * KP + c4 * 4, p.QN + off, t < p.S);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  // Kn Kn^T and Qn Kn^T depend on the key head only: computed once, kept in registers, and
  // reused for every value head h = hk + j*HK that reads this key head ("tile" pairing)
  const int i0 = (tid / 16) * 4, jb = tid % 16;
  float kk[4][4] = {}, qk[4][4] = {};
  {
#pragma unroll 2
    for (int d = 0; d < DKc; d += 4) {
      float4 ki[4], qi[4], kj[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        ki[u] = lds4(kn + (i0 + u) * KP + d);
        qi[u] = lds4(qn + (i0 + u) * KP + d);
        kj[u] = lds4(kn + (jb + 16 * u) * KP + d);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          kk[u][v] = fmaf(ki[u].x, kj[v].x, fmaf(ki[u].y, kj[v].y, fmaf(ki[u].z, kj[v].z, fmaf(ki[u].w, kj[v].w, kk[u][v]))));
          qk[u][v] = fmaf(qi[u].x, kj[v].x, fmaf(qi[u].y, kj[v].y, fmaf(qi[u].z, kj[v].z, fmaf(qi[u].w, kj[v].w, qk[u][v]))));
        }
    }
  }
  for (uint32_t h = hk; h < p.H; h += p.HK) {
  if (h != hk) __syncthreads();  // the previous value head is done with M, gc, beta
  // g / beta (deltanet_gbeta.wgsl:20-24); padded rows: g = 0, beta = 0 (as the reference pads)
  if (tid < C) {
    const uint32_t t = t0 + tid;
    float g = 0.f, bt = 0.f;
    if (t < p.S) {
      const uint64_t i = (uint64_t)t * p.H + h;
      g = p.a_neg[h] * softplus_s(p.a[i] + p.dt_bias[h]);
      bt = 1.0f / (1.0f + expf(-p.b[i]));
    }
    gc[tid] = g;
    beta[tid] = bt;
  }
  __syncthreads();
  if (tid < 32) {  // inclusive cumsum of g over the chunk (two values per lane)
    float a0 = gc[2 * tid], a1 = gc[2 * tid + 1];
    float sacc = a0 + a1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, sacc, o);
      if (tid >= o) sacc += y;
    }
    const float excl = sacc - (a0 + a1);
    gc[2 * tid] = excl + a0;
    gc[2 * tid + 1] = excl + a0 + a1;
  }
  __syncthreads();
  float *Aqk_out = p.Aqk + ((uint64_t)h * p.nc + c) * C * C;
  {
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int i = i0 + u, j = jb + 16 * v;
        const float dec = j <= i ? expf(gc[i] - gc[j]) : 0.f;
        M[i * CP + j] = j < i ? -(beta[i] * kk[u][v]) * dec : 0.f;
        Aqk_out[i * C + j] = qk[u][v] * dec;
      }
  }
  __syncthreads();
  {
    // forward substitution: x_r = b_r + sum_{m<r} M[r][m] x_m, column `col` of U or W
    const int col = tid % DVc, which = tid / DVc;  // 0: U (beta V), 1: W (beta exp(gc) Kn)
    float x[C];
    if (which == 0) {
#pragma unroll
      for (int r = 0; r < C; ++r) {
        const uint32_t t = t0 + r;
        x[r] = t < p.S ? p.v[((uint64_t)t * p.H + h) * DVc + col] * beta[r] : 0.f;
      }
    } else {
#pragma unroll
      for (int r = 0; r < C; ++r) x[r] = beta[r] * expf(gc[r]) * kn[r * KP + col];
    }
#pragma unroll
    for (int r = 1; r < C; ++r) {
      float acc0 = x[r], acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;  // four independent chains
#pragma unroll
      for (int m = 0; m + 4 <= r; m += 4) {
        const float4 mr = lds4(M + r * CP + m);
        acc0 = fmaf(mr.x, x[m], acc0);
        acc1 = fmaf(mr.y, x[m + 1], acc1);
        acc2 = fmaf(mr.z, x[m + 2], acc2);
        acc3 = fmaf(mr.w, x[m + 3], acc3);
      }
#pragma unroll
      for (int m = r & ~3; m < r; ++m) acc0 = fmaf(M[r * CP + m], x[m], acc0);
      x[r] = (acc0 + acc1) + (acc2 + acc3);
    }
    float *dst = (which ? p.W : p.U) + ((uint64_t)h * p.nc + c) * C * DVc;
#pragma unroll
    for (int r = 0; r < C; ++r) dst[r * DVc + col] = x[r];
  }
  if (tid < C) p.gcum[((uint64_t)h * p.nc + c) * C + tid] = gc[tid];
  // decayed keys, transposed for the tensor-core scan: KT[dk][t] = Kn[t][dk] exp(gc_last - gc_t);
  // the 64 decay factors once per value head (in beta's slot: beta is no longer read)
  if (p.KT) {
    __syncthreads();  // every solve thread is done with beta
    if (tid < C) beta[tid] = expf(gc[C - 1] - gc[tid]);
    __syncthreads();
    float *kt = p.KT + ((uint64_t)h * p.nc + c) * DKc * C;
    for (int idx = tid; idx < DKc * C; idx += blockDim.x) {
      const int dk = idx / C, t = idx % C;
      kt[idx] = kn[t * KP + dk] * beta[t];
    }
  }
  }
}

// Per (value head, 64 state columns), 512 threads, chunks in order; the next chunk's W and Qn
// (and U columns) are staged by cp.async while this chunk's second phase runs, and this chunk's
// Kn and Aqk while its first phase runs.
//   phase 1 (rows 2*(tid/16) + {0,1}, cols 4*(tid%16) + {0..3}):
//       Vn = U - W S  (-> shared),  QS = Qn S  (registers)
//   phase 2: O = exp(gc) QS + Aqk Vn  (Aqk zero above the diagonal)           -> core
//            S = exp(gc_last) S + (Kn exp(gc_last - gc))^T Vn   (rows 4*(tid/16) + {0..3})
// (qwen35_numpy.py:177-185)
constexpr int SG = 64;  // state columns per scan CTA

__global__ void __launch_bounds__(512) dn_chunk_scan(ChunkArgs p) {
  extern __shared__ __align__(16) float sm[];
  float *Wt = sm;                // [C][KP]
  float *Qt = Wt + C * KP;       // [C][KP]
  float *Kt = Qt + C * KP;       // [C][KP]
  float *Aq = Kt + C * KP;       // [C][CP]
  float *Uc = Aq + C * CP;       // [C][CP] (SG columns)
  float *Vn = Uc + C * CP;       // [C][CP]
  float *Ss = Vn + C * CP;       // [DK][CP] state columns
  float *gc = Ss + DKc * CP;     // [C]
  const uint32_t grp = blockIdx.x, h = blockIdx.y, hk = h % p.HK;
  const int tid = threadIdx.x;
  const uint32_t col0 = grp * SG;
  const int rp = tid / 16, cb = tid % 16;  // phase-1 / O tiles: rows 2rp, 2rp+1; cols 4cb..4cb+3
  const int r0 = 2 * rp, c0 = 4 * cb;

  auto stage_wq = [&](uint32_t c) {
    const uint32_t t0 = c * C;
    const float *W = p.W + ((uint64_t)h * p.nc + c) * C * DKc;
    const float *Ug = p.U + ((uint64_t)h * p.nc + c) * C * DVc;
    for (int idx = tid; idx < C * (DKc / 4); idx += blockDim.x) {
      const int r = idx / (DKc / 4), c4 = idx % (DKc / 4);
      const uint32_t t = t0 + r;
      cp16(Wt + r * KP + c4 * 4, W + r * DKc + c4 * 4, true);
      cp16(Qt + r * KP + c4 * 4, p.QN + ((uint64_t)(t < p.S ? t : 0) * p.HK + hk) * DKc + c4 * 4, t < p.S);
    }
    for (int idx = tid; idx < C * (SG / 4); idx += blockDim.x) {
      const int r = idx / (SG / 4), c4 = idx % (SG / 4);
      cp16(Uc + r * CP + c4 * 4, Ug + r * DVc + col0 + c4 * 4, true);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  auto stage_ka = [&](uint32_t c) {
    const uint32_t t0 = c * C;
    const float *A = p.Aqk + ((uint64_t)h * p.nc + c) * C * C;
    for (int idx = tid; idx < C * (DKc / 4); idx += blockDim.x) {
      const int r = idx / (DKc / 4), c4 = idx % (DKc / 4);
      const uint32_t t = t0 + r;
      cp16(Kt + r * KP + c4 * 4, p.KN + ((uint64_t)(t < p.S ? t : 0) * p.HK + hk) * DKc + c4 * 4, t < p.S);
    }
    for (int idx = tid; idx < C * (C / 4); idx += blockDim.x) {
      const int r = idx / (C / 4), c4 = idx % (C / 4);
      cp16(Aq + r * CP + c4 * 4, A + r * C + c4 * 4, true);
    }
    if (tid < C / 4) cp16(gc + tid * 4, p.gcum + ((uint64_t)h * p.nc + c) * C + tid * 4, true);
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  for (int idx = tid; idx < DKc * SG; idx += blockDim.x) {
    const int dk = idx / SG, cc = idx % SG;
    Ss[dk * CP + cc] = p.state_in ? p.state_in[((uint64_t)h * DKc + dk) * DVc + col0 + cc] : 0.f;
  }
  stage_wq(0);
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  for (uint32_t c = 0; c < p.nc; ++c) {
    const uint32_t t0 = c * C;
    stage_ka(c);
    // ---- phase 1: Vn = U - W S, QS = Qn S ----
    float vw[2][4], qs[2][4];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        vw[u][v] = Uc[(r0 + u) * CP + c0 + v];
        qs[u][v] = 0.f;
      }
#pragma unroll 2
    for (int d = 0; d < DKc; d += 4) {
      const float4 w0 = lds4(Wt + r0 * KP + d), w1 = lds4(Wt + (r0 + 1) * KP + d);
      const float4 q0 = lds4(Qt + r0 * KP + d), q1 = lds4(Qt + (r0 + 1) * KP + d);
      const float wa[2][4] = {{w0.x, w0.y, w0.z, w0.w}, {w1.x, w1.y, w1.z, w1.w}};
      const float qa[2][4] = {{q0.x, q0.y, q0.z, q0.w}, {q1.x, q1.y, q1.z, q1.w}};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 sv = lds4(Ss + (d + k) * CP + c0);
        const float sa[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            vw[u][v] = fmaf(-wa[u][k], sa[v], vw[u][v]);
            qs[u][v] = fmaf(qa[u][k], sa[v], qs[u][v]);
          }
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u)
      *reinterpret_cast<float4 *>(Vn + (r0 + u) * CP + c0) = make_float4(vw[u][0], vw[u][1], vw[u][2], vw[u][3]);
    asm volatile("cp.async.wait_all;" ::: "memory");  // this chunk's Kn, Aqk, gc
    __syncthreads();                                  // Vn complete; Wt / Qt / Uc free
    if (c + 1 < p.nc) stage_wq(c + 1);
    // ---- phase 2a: O = exp(gc) QS + Aqk Vn ----
    {
      float o[2][4];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float e = expf(gc[r0 + u]);
#pragma unroll
        for (int v = 0; v < 4; ++v) o[u][v] = qs[u][v] * e;
      }
      for (int j = 0; j <= r0 + 1; j += 4) {
        const float4 a0 = lds4(Aq + r0 * CP + j), a1 = lds4(Aq + (r0 + 1) * CP + j);
        const float aa[2][4] = {{a0.x, a0.y, a0.z, a0.w}, {a1.x, a1.y, a1.z, a1.w}};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float4 vv = lds4(Vn + (j + k) * CP + c0);
          const float va[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
          for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int v = 0; v < 4; ++v) o[u][v] = fmaf(aa[u][k], va[v], o[u][v]);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint32_t t = t0 + r0 + u;
        if (t < p.S)
          *reinterpret_cast<float4 *>(p.core + ((uint64_t)t * p.H + h) * DVc + col0 + c0) =
              make_float4(o[u][0], o[u][1], o[u][2], o[u][3]);
      }
    }
    // ---- phase 2b: S = exp(gc_last) S + (Kn exp(gc_last - gc))^T Vn, rows 4*rp .. +3 ----
    {
      const float gl = gc[C - 1], el = expf(gl);
      const int d0 = 4 * rp;
      float sacc[4][4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 sv = lds4(Ss + (d0 + u) * CP + c0);
        sacc[u][0] = sv.x * el; sacc[u][1] = sv.y * el; sacc[u][2] = sv.z * el; sacc[u][3] = sv.w * el;
      }
#pragma unroll 4
      for (int i = 0; i < C; ++i) {
        const float ek = expf(gl - gc[i]);
        const float4 kv = lds4(Kt + i * KP + d0);
        const float4 vv = lds4(Vn + i * CP + c0);
        const float ka[4] = {kv.x * ek, kv.y * ek, kv.z * ek, kv.w * ek};
        const float va[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int v = 0; v < 4; ++v) sacc[u][v] = fmaf(ka[u], va[v], sacc[u][v]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<float4 *>(Ss + (d0 + u) * CP + c0) =
            make_float4(sacc[u][0], sacc[u][1], sacc[u][2], sacc[u][3]);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // next chunk's W, Qn, U
    __syncthreads();
  }
  for (int idx = tid; idx < DKc * SG; idx += blockDim.x) {
    const int dk = idx / SG, cc = idx % SG;
    p.state_out[((uint64_t)h * DKc + dk) * DVc + col0 + cc] = Ss[dk * CP + cc];
  }
}

// ---------------------------------------------------------------------------------------------
// Tensor-core scan (tcgen05, kind::tf32 in 3xTF32: x = hi + lo, the three largest products).
// One CTA per value head; the state is held TRANSPOSED in tensor memory, S^T [dv lanes][dk cols],
// as the accumulator of its own update -- and split into hi / lo copies it is the A operand of the
// next chunk's products, so it never leaves the SM.  Per chunk (transposed forms of
// qwen35_numpy.py:177-185; B operands K-major in 128B-swizzled shared memory):
//   T1 = S^T W^T       [dv][t]   (A = S^T hi/lo from TMEM, B = W [t][dk])
//   T2 = S^T Qn^T      [dv][t]   (B = Qn [t][dk])
//   Vn^T = U^T - T1    (state warps, into TMEM as hi / lo: the A operand of T3 and T4)
//   T4: S^T = exp(gc_last) S^T + Vn^T Kd    (B = Kd^T [dk][t], the prep kernel's decayed keys)
//   T3 = Vn^T Aqk^T    [dv][t]   (B = Aqk [i][j])
//   O^T = exp(gc_t) T2 + T3   -> core
// The products issue as two MMA groups per chunk: [T1 | T2] with W and Qn stacked in one B tile
// (N = 128), and [T4 | T3] with Kd^T and Aqk stacked (N = 192, accumulating: the state warps zero
// the T3 columns first).
// TMEM (512 columns): S hi [0,128), S lo [128,256), S^T [256,384), T1 / T3 [384,448), T2 [448,512);
// Vn hi / lo reuse [0,64) / [128,192) once T1 and T2 are done.
// Warps: 0 TMA producer (W, Qn, Aqk, Kd^T f32 tiles into the hi buffers), 1 MMA issuer, 2 TMEM
// owner, 4-7 state warps (TMEM lane = dv), 8-11 split warps (hi in place, lo beside it).
// All mbarrier waits are bounded (BG_ETIMEOUT on expiry).
namespace sc {
// B tile 1: per 32-column block of dk, rows 0-63 = W, rows 64-127 = Qn  (4 blocks x 16 KB)
// B tile 2: per 32-column block of t,  rows 0-127 = Kd^T, rows 128-191 = Aqk  (2 blocks x 24 KB)
constexpr int B1 = 128 * 128, B1T = 4 * B1, B2 = 192 * 128, B2T = 2 * B2;
constexpr int WQ = C * DKc * 4, AQ = C * C * 4, KTB = DKc * C * 4;  // bytes TMA brings per tile
constexpr int H1 = 0, L1 = B1T, H2 = 2 * B1T, L2 = H2 + B2T, BAR = L2 + B2T, EG = BAR + 256, TOTAL = EG + 800;
constexpr uint32_t TSHI = 0, TSLO = 128, TS = 256, TT1 = 384, TT2 = 448;
}  // namespace sc

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

struct ScanMaps {
  CUtensorMap W, Q, A, K;
};

__global__ void __launch_bounds__(384, 1) dn_chunk_scan_tc(const __grid_constant__ ScanMaps mp, ChunkArgs p) {
  using namespace sc;
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + BAR);
  uint64_t *wq_raw = bars, *wq_full = bars + 1, *wq_empty = bars + 2;
  uint64_t *ak_raw = bars + 3, *ak_full = bars + 4, *ak_empty = bars + 5;
  uint64_t *s_ready = bars + 6, *t2_done = bars + 7, *vn_ready = bars + 8, *t4_done = bars + 9;
  uint64_t *t3_done = bars + 10, *out_read = bars + 11, *mma_done = bars + 12;
  uint32_t *tmem_s = reinterpret_cast<uint32_t *>(bars + 13);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 14);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t h = blockIdx.x, hk = h % p.HK, nc = p.nc;
  if (tid == 0) {
    mbar_init(wq_raw, 1); mbar_init(wq_full, 4); mbar_init(wq_empty, 1);
    mbar_init(ak_raw, 1); mbar_init(ak_full, 4); mbar_init(ak_empty, 1);
    mbar_init(s_ready, 128); mbar_init(t2_done, 1); mbar_init(vn_ready, 128); mbar_init(t4_done, 1);
    mbar_init(t3_done, 1); mbar_init(out_read, 128); mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_s)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_s;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 72;" ::: "memory");
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer ----------------
      prefetch_tmap(&mp.W); prefetch_tmap(&mp.Q); prefetch_tmap(&mp.A); prefetch_tmap(&mp.K);
      for (uint32_t c = 0; c < nc; ++c) {
        const int rowW = (int)((h * nc + c) * C), rowK = (int)((h * nc + c) * DKc);
        if (c > 0 && !mbar_wait(wq_empty, (c - 1) & 1)) { *abort_flag = 1; break; }
        if (*abort_flag) break;
        mbar_expect_tx(wq_raw, 2 * WQ);
        for (int cb = 0; cb < DKc / 32; ++cb) {
          tma_load_4d(sm + H1 + cb * B1, &mp.W, wq_raw, cb * 32, rowW, 0, 0);
          tma_load_4d(sm + H1 + cb * B1 + C * 128, &mp.Q, wq_raw, cb * 32, (int)hk, (int)(c * C), 0);
        }
        if (c > 0 && !mbar_wait(ak_empty, (c - 1) & 1)) { *abort_flag = 1; break; }
        mbar_expect_tx(ak_raw, AQ + KTB);
        for (int cb = 0; cb < C / 32; ++cb) {
          tma_load_4d(sm + H2 + cb * B2, &mp.K, ak_raw, cb * 32, rowK, 0, 0);
          tma_load_4d(sm + H2 + cb * B2 + DKc * 128, &mp.A, ak_raw, cb * 32, rowW, 0, 0);
        }
      }
      // no bulk copy in flight at exit: the last chunk's loads were consumed by the split warps
      if (nc) { mbar_wait(wq_raw, (nc - 1) & 1); mbar_wait(ak_raw, (nc - 1) & 1); }
    } else if (warp == 1 && lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t s0 = smem_u32(sm);
      constexpr uint32_t id128 = idesc_tf32(128), id192 = idesc_tf32(192);
      // D[dv][n] (+)= A (TMEM, K columns) x B (K-major smem tile of `rows` rows, K = 32 per 128B block)
      auto prod = [&](uint32_t d, uint32_t ahi, uint32_t alo, uint32_t bhi, uint32_t blo, int ksteps, int rows,
                      uint32_t idesc, bool acc) {
#pragma unroll 1
        for (int term = 0; term < 3; ++term) {
          const uint32_t a = term == 1 ? alo : ahi, bb = term == 2 ? blo : bhi;
#pragma unroll 4
          for (int kk = 0; kk < ksteps; ++kk) {
            const uint64_t bd = umma_desc_sw128(bb + (kk >> 2) * (rows * 128) + (kk & 3) * 32, 16, 1024);
            umma_ts_tf32(d, a + kk * 8, bd, idesc, (acc || term > 0 || kk > 0) ? 1u : 0u);
          }
        }
      };
      bool ok = true;
      uint32_t c = 0;
      for (; ok && c < nc; ++c) {
        const uint32_t ph = c & 1;
        if (!mbar_wait(s_ready, ph) || !mbar_wait(wq_full, ph) || (c > 0 && !mbar_wait(out_read, (c - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // [T1 | T2] = S^T [W ; Qn]^T into columns [384, 512)
        prod(tmem + TT1, tmem + TSHI, tmem + TSLO, s0 + H1, s0 + L1, DKc / 8, 128, id128, false);
        umma_commit(t2_done);
        umma_commit(wq_empty);
        if (!mbar_wait(vn_ready, ph) || !mbar_wait(ak_full, ph)) { ok = false; break; }
        tc_fence_after();
        // [T4 | T3] = Vn^T [Kd^T ; Aqk]^T accumulated into columns [256, 448): S^T (pre-scaled)
        // and the zeroed T3 columns
        prod(tmem + TS, tmem + TSHI, tmem + TSLO, s0 + H2, s0 + L2, C / 8, 192, id192, true);
        umma_commit(t3_done);
        umma_commit(t4_done);
        umma_commit(ak_empty);
      }
      if (!ok) *abort_flag = 1;
      umma_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
  } else if (warp >= 8) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 216;" ::: "memory");
    // ---------------- split warps: hi in place, lo beside it (same swizzled offsets) ----------------
    const int ct = tid - 256;
    auto split = [&](int hi, int lo, int bytes) {
#pragma unroll 4
      for (int i = ct; i < bytes / 16; i += 128) {
        float4 *hp = reinterpret_cast<float4 *>(sm + hi + i * 16);
        const float4 x = *hp;
        const float4 y = make_float4(tf32_rna(x.x), tf32_rna(x.y), tf32_rna(x.z), tf32_rna(x.w));
        *hp = y;
        *reinterpret_cast<float4 *>(sm + lo + i * 16) = make_float4(x.x - y.x, x.y - y.y, x.z - y.z, x.w - y.w);
      }
    };
    for (uint32_t c = 0; c < nc; ++c) {
      if (!mbar_wait_warp(wq_raw, c & 1)) { *abort_flag = 1; break; }
      split(H1, L1, B1T);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(wq_full);
      if (!mbar_wait_warp(ak_raw, c & 1)) { *abort_flag = 1; break; }
      split(H2, L2, B2T);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(ak_full);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 216;" ::: "memory");
    // ---------------- state warps: TMEM lane = value column dv ----------------
    const uint32_t dv = (uint32_t)((warp & 3) * 32 + lane);
    const uint32_t loff = (uint32_t)((warp & 3) * 32) << 16;
    // S^T from state_in [h][dk][dv] (zero without one)
#pragma unroll 1
    for (int cb = 0; cb < DKc / 32; ++cb) {
      uint32_t r[32];
#pragma unroll
      for (int i = 0; i < 32; ++i)
        r[i] = __float_as_uint(p.state_in ? p.state_in[((uint64_t)h * DKc + cb * 32 + i) * DVc + dv] : 0.f);
      tmem_st32((tmem + TS + cb * 32) | loff, r);
    }
    tmem_wait_st();
    bool ok = true;
    // Decay factors a chunk ahead, in shared memory (no global load on the chain): eg[c % 3][t] =
    // exp(gc_t) of chunk c, el[c % 3] = exp(gc_last) of chunk c.  State thread t < 64 computes them
    // one iteration ahead; three slots keep the writer of chunk c+1 clear of readers of chunk c-1.
    float *eg = reinterpret_cast<float *>(sm + EG);  // [3][C]
    float *elv = eg + 3 * C;                         // [3]
    auto decays = [&](uint32_t cc) {
      if (cc < nc && dv < C) {
        const float g = __ldg(p.gcum + ((uint64_t)h * nc + cc) * C + dv);
        eg[(cc % 3) * C + dv] = expf(g);
        if (dv == C - 1) elv[cc % 3] = expf(g);
      }
    };
    decays(0);
    asm volatile("bar.sync 2, 128;" ::: "memory");
    // output of chunk oc: O^T = exp(gc_t) T2 + T3 read into registers (then the T columns are free)
    auto read_out = [&](uint32_t oc, float (&o)[C]) {
      const float *e = eg + (oc % 3) * C;
#pragma unroll
      for (int cb = 0; cb < C / 32; ++cb) {
        uint32_t a[32], b3[32];
        tmem_ld32((tmem + TT2 + cb * 32) | loff, a);
        tmem_ld32((tmem + TT1 + cb * 32) | loff, b3);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[cb * 32 + i] = fmaf(__uint_as_float(a[i]), e[cb * 32 + i], __uint_as_float(b3[i]));
      }
    };
    auto store_out = [&](uint32_t oc, const float (&o)[C]) {
#pragma unroll
      for (int t = 0; t < C; ++t) {
        const uint32_t tt = oc * C + t;
        if (tt < p.S) p.core[((uint64_t)tt * p.H + h) * DVc + dv] = o[t];
      }
    };
    float o[C];
    for (uint32_t c = 0; c < nc && ok; ++c) {
      const uint32_t ph = c & 1;
      if (c > 0) {  // T3 and T4 of the previous chunk are done with Vn and S^T
        if (!mbar_wait_warp(t4_done, (c - 1) & 1)) { ok = false; break; }
        tc_fence_after();
      }
      // (1) S hi / lo for T1, T2; S^T scaled by exp(gc_last) for T4
      const float el = elv[c % 3];
#pragma unroll 1
      for (int cb = 0; cb < DKc / 32; ++cb) {
        uint32_t x[32], hi[32], lo[32];
        tmem_ld32((tmem + TS + cb * 32) | loff, x);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float v = __uint_as_float(x[i]), vh = tf32_rna(v);
          hi[i] = __float_as_uint(vh);
          lo[i] = __float_as_uint(v - vh);
          x[i] = __float_as_uint(v * el);
        }
        tmem_st32((tmem + TSHI + cb * 32) | loff, hi);
        tmem_st32((tmem + TSLO + cb * 32) | loff, lo);
        tmem_st32((tmem + TS + cb * 32) | loff, x);
      }
      tmem_wait_st();
      // the previous chunk's output: read its accumulators, free them, then finish it while this
      // chunk's T1 / T2 run
      tc_fence_before();
      mbar_arrive(s_ready);
      if (c > 0) {
        read_out(c - 1, o);
        tc_fence_before();
        mbar_arrive(out_read);
        store_out(c - 1, o);
      }
      // (3) Vn^T = U^T - T1, split into hi / lo over the S hi / lo columns (T1, T2 are done)
      const float *U = p.U + ((uint64_t)h * nc + c) * C * DVc;
      float u[C];
#pragma unroll
      for (int t = 0; t < C; ++t) u[t] = __ldg(U + t * DVc + dv);
      decays(c + 1);  // slot (c+1) % 3: last read by read_out(c - 2), before the previous barrier
      if (!mbar_wait_warp(t2_done, ph)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int cb = 0; cb < C / 32; ++cb) {
        uint32_t x[32], hi[32], lo[32];
        tmem_ld32((tmem + TT1 + cb * 32) | loff, x);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float v = u[cb * 32 + i] - __uint_as_float(x[i]), vh = tf32_rna(v);
          hi[i] = __float_as_uint(vh);
          lo[i] = __float_as_uint(v - vh);
          x[i] = 0u;
        }
        tmem_st32((tmem + TSHI + cb * 32) | loff, hi);
        tmem_st32((tmem + TSLO + cb * 32) | loff, lo);
        tmem_st32((tmem + TT1 + cb * 32) | loff, x);  // T3 accumulates onto zero
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(vn_ready);
      asm volatile("bar.sync 2, 128;" ::: "memory");  // decays(c + 1) visible to every state thread
    }
    if (ok && nc) {  // the last chunk's output
      if (mbar_wait_warp(t4_done, (nc - 1) & 1)) {
        tc_fence_after();
        read_out(nc - 1, o);
        store_out(nc - 1, o);
      } else {
        ok = false;
      }
    }
    if (ok && nc) {
#pragma unroll 1
      for (int cb = 0; cb < DKc / 32; ++cb) {
        uint32_t r[32];
        tmem_ld32((tmem + TS + cb * 32) | loff, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) p.state_out[((uint64_t)h * DKc + cb * 32 + i) * DVc + dv] = __uint_as_float(r[i]);
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

int launch_scan_tc(const ChunkArgs &p, cudaStream_t st) {
  ScanMaps mp;
  const uint64_t nrow = (uint64_t)p.H * p.nc;
  {
    const uint64_t dims[4] = {DKc, nrow * C, 1, 1}, strides[3] = {DKc * 4, nrow * C * DKc * 4, nrow * C * DKc * 4};
    const uint32_t box[4] = {32, C, 1, 1};
    if (make_tmap_4d(&mp.W, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.W, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return BG_EUNSUPPORTED;
  }
  {
    const uint64_t dims[4] = {DKc, p.HK, p.S, 1};
    const uint64_t strides[3] = {DKc * 4, (uint64_t)p.HK * DKc * 4, (uint64_t)p.S * p.HK * DKc * 4};
    const uint32_t box[4] = {32, 1, C, 1};
    if (make_tmap_4d(&mp.Q, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.QN, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return BG_EUNSUPPORTED;
  }
  {
    const uint64_t dims[4] = {C, nrow * C, 1, 1}, strides[3] = {C * 4, nrow * C * C * 4, nrow * C * C * 4};
    const uint32_t box[4] = {32, C, 1, 1};
    if (make_tmap_4d(&mp.A, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.Aqk, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return BG_EUNSUPPORTED;
  }
  {
    const uint64_t dims[4] = {C, nrow * DKc, 1, 1}, strides[3] = {C * 4, nrow * DKc * C * 4, nrow * DKc * C * 4};
    const uint32_t box[4] = {32, DKc, 1, 1};
    if (make_tmap_4d(&mp.K, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.KT, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return BG_EUNSUPPORTED;
  }
  const int smem = sc::TOTAL + 1024;
  if (cudaFuncSetAttribute(dn_chunk_scan_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return BG_ELAUNCH;
  dn_chunk_scan_tc<<<p.H, 384, smem, st>>>(mp, p);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

// BGATTN_DN_SCAN=cuda keeps the CUDA-core scan (A/B checks)
bool scan_tc_enabled() {
  static const bool v = [] {
    const char *e = getenv("BGATTN_DN_SCAN");
    return !(e && e[0] == 'c');
  }();
  return v;
}

}  // namespace

size_t deltanet_chunk_workspace(uint32_t S, uint32_t H) {
  const uint64_t nc = (S + C - 1) / C;
  return (size_t)H * nc * (C * DVc + C * DKc + C * C + C + DKc * C) * sizeof(float) +
         2 * (size_t)S * H * DKc * sizeof(float);
}

int launch_deltanet_chunked(const DeltaArgs &d, void *ws, size_t ws_bytes, cudaStream_t st) {
  if (d.DK != DKc || d.DV != DVc) return BG_EUNSUPPORTED;
  if (d.S == 0) return BG_OK;
  if (!ws || ws_bytes < deltanet_chunk_workspace(d.S, d.H)) return BG_ENOMEM;
  ChunkArgs p;
  p.S = d.S;
  p.H = d.H;
  p.HK = d.HK;
  p.nc = (d.S + C - 1) / C;
  p.q = d.q;
  p.k = d.k;
  p.v = d.v;
  p.a = d.a;
  p.b = d.b;
  p.a_neg = d.a_neg;
  p.dt_bias = d.dt_bias;
  p.state_in = d.loadState ? d.state_in : nullptr;
  p.state_out = d.state_out;
  p.core = d.core;
  float *w = static_cast<float *>(ws);
  const uint64_t per = (uint64_t)d.H * p.nc;
  p.U = w;
  p.W = p.U + per * C * DVc;
  p.Aqk = p.W + per * C * DKc;
  p.gcum = p.Aqk + per * C * C;
  p.QN = p.gcum + per * C;               // [S][HK][DK] (H >= HK rows reserved)
  p.KN = p.QN + (uint64_t)d.S * d.H * DKc;
  p.KT = scan_tc_enabled() ? p.KN + (uint64_t)d.S * d.H * DKc : nullptr;  // [H][nc][DK][C]
  const int smem_prep = (2 * C * KP + C * CP + 2 * C) * sizeof(float);
  const int smem_scan = (3 * C * KP + 3 * C * CP + DKc * CP + C) * sizeof(float);
  if (cudaFuncSetAttribute(dn_chunk_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_prep) != cudaSuccess ||
      cudaFuncSetAttribute(dn_chunk_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_scan) != cudaSuccess)
    return BG_ELAUNCH;
  const uint64_t nrows = (uint64_t)d.S * d.HK;
  dn_norm_qk<<<(unsigned)((nrows * 32 + 255) / 256), 256, 0, st>>>(p);
  dn_chunk_prep<<<dim3(p.nc, d.HK), 256, smem_prep, st>>>(p);
  if (p.KT) {
    if (cudaGetLastError() != cudaSuccess) return BG_ELAUNCH;
    return launch_scan_tc(p, st);
  }
  dn_chunk_scan<<<dim3(DVc / SG, d.H), 512, smem_scan, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int poll_device_error_dnchunk() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return BG_ELAUNCH;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  return v;
}

}  // namespace bg
