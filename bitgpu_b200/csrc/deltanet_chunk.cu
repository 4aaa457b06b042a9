// Chunked (WY) gated-DeltaNet prefill: the chunk-parallel form of the delta rule that bitgpu's
// numpy oracle implements as tools/qwen35_numpy.py:144-187 (_delta_chunk, == HF
// torch_chunk_gated_delta_rule), extended with an initial state.  The recurrent kernel
// (deltanet.cu) is sequential over every token; here only the state hand-off between chunks of
// C = 64 tokens is sequential, everything inside a chunk is dense f32 arithmetic.
//
//   prep kernel   one CTA per (chunk, value head), all independent:
//                 Kn = l2norm(k), Qn = l2norm(q)/sqrt(DK), g/beta from a/b (fused gbeta),
//                 gc = cumsum(g) within the chunk,
//                 A[i][j] = -beta_i (Kn_i . Kn_j) exp(gc_i - gc_j)   (j < i),
//                 T = the reference's row recurrence on A, plus I   (qwen35_numpy.py:168-172),
//                 U = T (beta V),  W = T (beta exp(gc) Kn),
//                 Aqk[i][j] = (Qn_i . Kn_j) exp(gc_i - gc_j)   (j <= i)
//                 -> workspace {U, W, Aqk, gc}
//   scan kernel   one CTA per (value head, 16 state columns), chunks in order:
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
constexpr int GRP = 16;  // state columns per scan CTA
constexpr int PAD = DKc + 1;   // prep: conflict-free row-pair dot products
constexpr int SPAD = DKc;      // scan: rows read as warp broadcasts, no padding needed

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

// rows t0 .. t0+63 of a normalised [S][HK][DK] tensor into smem (row stride `pad`), zero past S
__device__ __forceinline__ void load_rows(float *dst, int pad, const float *src, uint32_t S, uint32_t HK,
                                          uint32_t hk, uint32_t t0) {
  for (int idx = threadIdx.x; idx < C * (DKc / 4); idx += blockDim.x) {
    const int r = idx / (DKc / 4), c4 = idx % (DKc / 4);
    const uint32_t t = t0 + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < S) v = *reinterpret_cast<const float4 *>(src + ((uint64_t)t * HK + hk) * DKc + c4 * 4);
    float *d = dst + r * pad + c4 * 4;
    d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
  }
}

__device__ __forceinline__ void cp16(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(valid ? 16u : 0u)
               : "memory");
}

__global__ void __launch_bounds__(256) dn_chunk_prep(ChunkArgs p) {
  extern __shared__ float sm[];
  float *kn = sm;                  // [C][PAD]
  float *qn = kn + C * PAD;        // [C][PAD]
  float *vb = qn;                  // [C][PAD]  beta * v, loaded once Qn is no longer needed
  float *T = qn + C * PAD;         // [C][C+1]
  float *gc = T + C * (C + 1);     // [C]
  float *beta = gc + C;            // [C]
  float *newrow = beta + C;        // [C]
  float *bge = newrow + C;         // [C] beta * exp(gc)
  const uint32_t c = blockIdx.x, h = blockIdx.y, hk = h % p.HK;
  const uint32_t t0 = c * C;
  const int tid = threadIdx.x;

  load_rows(kn, PAD, p.KN, p.S, p.HK, hk, t0);
  load_rows(qn, PAD, p.QN, p.S, p.HK, hk, t0);
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
    float s = a0 + a1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, s, o);
      if (tid >= o) s += y;
    }
    const float excl = s - (a0 + a1);
    gc[2 * tid] = excl + a0;
    gc[2 * tid + 1] = excl + a0 + a1;
  }
  __syncthreads();
  // A (strictly lower) and Aqk (lower incl. diagonal)
  float *Aqk_out = p.Aqk + ((uint64_t)h * p.nc + c) * C * C;
  {
    // 4 x 4 tile of (i, j) per thread: 12 shared loads feed 32 FMAs per d
    const int i0 = (tid / 16) * 4, j0 = (tid % 16) * 4;
    float kk[4][4] = {}, qk[4][4] = {};
    if (j0 <= i0 + 3) {
      for (int d = 0; d < DKc; ++d) {
        float ki[4], qi[4], kj[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          ki[u] = kn[(i0 + u) * PAD + d];
          qi[u] = qn[(i0 + u) * PAD + d];
          kj[u] = kn[(j0 + u) * PAD + d];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            kk[u][v] = fmaf(ki[u], kj[v], kk[u][v]);
            qk[u][v] = fmaf(qi[u], kj[v], qk[u][v]);
          }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int i = i0 + u, j = j0 + v;
        const float dec = j <= i ? expf(gc[i] - gc[j]) : 0.f;
        T[i * (C + 1) + j] = j < i ? -(beta[i] * kk[u][v]) * dec : 0.f;
        Aqk_out[i * C + j] = qk[u][v] * dec;
      }
  }
  __syncthreads();
  // Qn is consumed: its buffer now takes beta * V
  for (int idx = tid; idx < C * DVc; idx += blockDim.x) {
    const int r = idx / DVc, d = idx % DVc;
    const uint32_t t = t0 + r;
    vb[r * PAD + d] = t < p.S ? p.v[((uint64_t)t * p.H + h) * DVc + d] * beta[r] : 0.f;
  }
  // row recurrence of the reference: row_i[:i] += row_i[:i] @ T[:i,:i] with rows < i final
  for (int i = 1; i < C; ++i) {
    if (tid < i) {
      float acc = T[i * (C + 1) + tid];
      for (int m = tid + 1; m < i; ++m) acc = fmaf(T[i * (C + 1) + m], T[m * (C + 1) + tid], acc);
      newrow[tid] = acc;
    }
    __syncthreads();
    if (tid < i) T[i * (C + 1) + tid] = newrow[tid];
    __syncthreads();
  }
  if (tid < C) {
    T[tid * (C + 1) + tid] = 1.0f;
    bge[tid] = beta[tid] * expf(gc[tid]);
  }
  __syncthreads();
  // U = T (beta V), W = T (beta exp(gc) Kn): rows i, sum over m <= i
  float *U = p.U + ((uint64_t)h * p.nc + c) * C * DVc;
  float *W = p.W + ((uint64_t)h * p.nc + c) * C * DKc;
  {
    // thread -> one dim d and 32 rows; T is zero above the diagonal, so the m loop is dense
    const int d = tid % DVc, ib = (tid / DVc) * 32;
    float u[32], w[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) u[r] = w[r] = 0.f;
    for (int m = 0; m < ib + 32; ++m) {
      const float vm = vb[m * PAD + d], km = bge[m] * kn[m * PAD + d];
#pragma unroll
      for (int r = 0; r < 32; ++r) {
        const float tm = T[(ib + r) * (C + 1) + m];
        u[r] = fmaf(tm, vm, u[r]);
        w[r] = fmaf(tm, km, w[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      U[(ib + r) * DVc + d] = u[r];
      W[(ib + r) * DKc + d] = w[r];
    }
  }
  if (tid < C) p.gcum[((uint64_t)h * p.nc + c) * C + tid] = gc[tid];
}

__global__ void __launch_bounds__(256) dn_chunk_scan(ChunkArgs p) {
  extern __shared__ float sm[];
  float *Ws = sm;                 // [C][SPAD]
  float *qn = Ws + C * SPAD;      // [C][SPAD]
  float *kn = qn + C * SPAD;      // [C][SPAD]
  float *Uc = kn + C * SPAD;      // [C][GRP] this CTA's columns of U
  float *Ss = Uc + C * GRP;       // [DK][GRP] state columns
  float *Vn = Ss + DKc * GRP;     // [C][GRP]
  float *gc = Vn + C * GRP;       // [C]
  float *ek = gc + C;             // [C] exp(gc_last - gc)
  const uint32_t grp = blockIdx.x, h = blockIdx.y, hk = h % p.HK;
  const int tid = threadIdx.x;
  const uint32_t col0 = grp * GRP;
  for (int idx = tid; idx < DKc * GRP; idx += blockDim.x) {
    const int dk = idx / GRP, cc = idx % GRP;
    Ss[idx] = p.state_in ? p.state_in[((uint64_t)h * DKc + dk) * DVc + col0 + cc] : 0.f;
  }
  for (uint32_t c = 0; c < p.nc; ++c) {
    const uint32_t t0 = c * C;
    __syncthreads();  // previous chunk fully consumed
    // stage this chunk with cp.async: every copy in flight at once, one wait
    const float *W = p.W + ((uint64_t)h * p.nc + c) * C * DKc;
    const float *A = p.Aqk + ((uint64_t)h * p.nc + c) * C * C;
    const float *Ug = p.U + ((uint64_t)h * p.nc + c) * C * DVc;
    for (int idx = tid; idx < C * (DKc / 4); idx += blockDim.x) {
      const int r = idx / (DKc / 4), c4 = idx % (DKc / 4);
      const uint32_t t = t0 + r;
      const uint64_t qk_off = ((uint64_t)(t < p.S ? t : 0) * p.HK + hk) * DKc + c4 * 4;
      cp16(Ws + r * SPAD + c4 * 4, W + r * DKc + c4 * 4, true);
      cp16(qn + r * SPAD + c4 * 4, p.QN + qk_off, t < p.S);
      cp16(kn + r * SPAD + c4 * 4, p.KN + qk_off, t < p.S);
    }
    for (int idx = tid; idx < C * (GRP / 4); idx += blockDim.x)
      cp16(Uc + (idx / (GRP / 4)) * GRP + (idx % (GRP / 4)) * 4,
           Ug + (idx / (GRP / 4)) * DVc + col0 + (idx % (GRP / 4)) * 4, true);
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (tid < C) gc[tid] = p.gcum[((uint64_t)h * p.nc + c) * C + tid];
    __syncthreads();
    if (tid < C) ek[tid] = expf(gc[C - 1] - gc[tid]);
    // Vn = U - W S    (C x GRP outputs, 4 per thread)
    const int cc = tid % GRP, rb = tid / GRP;  // column and row group (16 groups)
    {  // Vn = U - W S: rows rb + 16u, four independent accumulators
      float acc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[u] = Uc[(rb + 16 * u) * GRP + cc];
#pragma unroll 4
      for (int d = 0; d < DKc; ++d) {
        const float sv = Ss[d * GRP + cc];
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[u] = fmaf(-Ws[(rb + 16 * u) * SPAD + d], sv, acc[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) Vn[(rb + 16 * u) * GRP + cc] = acc[u];
    }
    __syncthreads();
    {  // O = exp(gc) (Qn S) + Aqk Vn   (Aqk is zero above the diagonal)
      float qs[4] = {0.f, 0.f, 0.f, 0.f}, av[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
      for (int d = 0; d < DKc; ++d) {
        const float sv = Ss[d * GRP + cc];
#pragma unroll
        for (int u = 0; u < 4; ++u) qs[u] = fmaf(qn[(rb + 16 * u) * SPAD + d], sv, qs[u]);
      }
#pragma unroll 4
      for (int j = 0; j < C; ++j) {
        const float vv = Vn[j * GRP + cc];
#pragma unroll
        for (int u = 0; u < 4; ++u) av[u] = fmaf(__ldg(A + (rb + 16 * u) * C + j), vv, av[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = rb + 16 * u;
        const uint32_t t = t0 + i;
        if (t < p.S) p.core[((uint64_t)t * p.H + h) * DVc + col0 + cc] = fmaf(qs[u], expf(gc[i]), av[u]);
      }
    }
    __syncthreads();
    {  // S = S exp(gc_last) + (Kn exp(gc_last - gc))^T Vn: state rows rb + 16u, u < 8
      const float el = expf(gc[C - 1]);
      float acc[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc[u] = Ss[(rb + 16 * u) * GRP + cc] * el;
#pragma unroll 4
      for (int i = 0; i < C; ++i) {
        const float vv = Vn[i * GRP + cc] * ek[i];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[u] = fmaf(kn[i * SPAD + rb + 16 * u], vv, acc[u]);
      }
      __syncthreads();  // every thread has read the old state
#pragma unroll
      for (int u = 0; u < 8; ++u) Ss[(rb + 16 * u) * GRP + cc] = acc[u];
    }
  }
  __syncthreads();
  for (int idx = tid; idx < DKc * GRP; idx += blockDim.x) {
    const int dk = idx / GRP, cc = idx % GRP;
    p.state_out[((uint64_t)h * DKc + dk) * DVc + col0 + cc] = Ss[idx];
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
  const int smem_prep = (2 * C * PAD + C * (C + 1) + 4 * C) * sizeof(float);
  const int smem_scan = (3 * C * SPAD + C * GRP + DKc * GRP + C * GRP + 2 * C) * sizeof(float);
  if (cudaFuncSetAttribute(dn_chunk_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_prep) != cudaSuccess ||
      cudaFuncSetAttribute(dn_chunk_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_scan) != cudaSuccess)
    return BG_ELAUNCH;
  const uint64_t nrows = (uint64_t)d.S * d.HK;
  dn_norm_qk<<<(unsigned)((nrows * 32 + 255) / 256), 256, 0, st>>>(p);
  dn_chunk_prep<<<dim3(p.nc, d.H), 256, smem_prep, st>>>(p);
  dn_chunk_scan<<<dim3(DVc / GRP, d.H), 256, smem_scan, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

}  // namespace bg
