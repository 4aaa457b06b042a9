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

#include "kv.h"

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
__global__ void __launch_bounds__(256) dn_chunk_prep(ChunkArgs p) {
  extern __shared__ __align__(16) float sm[];
  float *kn = sm;              // [C][KP]
  float *qn = kn + C * KP;     // [C][KP]
  float *M = qn + C * KP;      // [C][CP]
  float *gc = M + C * CP;      // [C]
  float *beta = gc + C;        // [C]
  const uint32_t c = blockIdx.x, h = blockIdx.y, hk = h % p.HK;
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
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  float *Aqk_out = p.Aqk + ((uint64_t)h * p.nc + c) * C * C;
  {
    const int i0 = (tid / 16) * 4, jb = tid % 16;
    float kk[4][4] = {}, qk[4][4] = {};
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
      float acc0 = x[r], acc1 = 0.f;
#pragma unroll
      for (int m = 0; m + 4 <= r; m += 4) {
        const float4 mr = lds4(M + r * CP + m);
        acc0 = fmaf(mr.x, x[m], acc0);
        acc1 = fmaf(mr.y, x[m + 1], acc1);
        acc0 = fmaf(mr.z, x[m + 2], acc0);
        acc1 = fmaf(mr.w, x[m + 3], acc1);
      }
#pragma unroll
      for (int m = r & ~3; m < r; ++m) acc0 = fmaf(M[r * CP + m], x[m], acc0);
      x[r] = acc0 + acc1;
    }
    float *dst = (which ? p.W : p.U) + ((uint64_t)h * p.nc + c) * C * DVc;
#pragma unroll
    for (int r = 0; r < C; ++r) dst[r * DVc + col] = x[r];
  }
  if (tid < C) p.gcum[((uint64_t)h * p.nc + c) * C + tid] = gc[tid];
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

}  // namespace

size_t deltanet_chunk_workspace(uint32_t S, uint32_t H) {
  const uint64_t nc = (S + C - 1) / C;
  return (size_t)H * nc * (C * DVc + C * DKc + C * C + C) * sizeof(float) + 2 * (size_t)S * H * DKc * sizeof(float);
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
  const int smem_prep = (2 * C * KP + C * CP + 2 * C) * sizeof(float);
  const int smem_scan = (3 * C * KP + 3 * C * CP + DKc * CP + C) * sizeof(float);
  if (cudaFuncSetAttribute(dn_chunk_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_prep) != cudaSuccess ||
      cudaFuncSetAttribute(dn_chunk_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_scan) != cudaSuccess)
    return BG_ELAUNCH;
  const uint64_t nrows = (uint64_t)d.S * d.HK;
  dn_norm_qk<<<(unsigned)((nrows * 32 + 255) / 256), 256, 0, st>>>(p);
  dn_chunk_prep<<<dim3(p.nc, d.H), 256, smem_prep, st>>>(p);
  dn_chunk_scan<<<dim3(DVc / SG, d.H), 512, smem_scan, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

}  // namespace bg
