// CUDA-core split-KV GQA attention over f32 / f16 / q8 / q8r caches, with optional rope-at-read
// (rolling-window mode) and ring-mapped slots.  It is the production path for the f32 cache
// and for rope-at-read, and the reference path every other kernel is cross-checked against.
//
// Math per query row (shaders/attention_sg.wgsl:31-44): online softmax over the row's cache
// positions, scores (q.k)*scale, f32 throughout.  Scores are carried in log2 units (scale is
// pre-multiplied by log2 e) so the exponentials are exp2f.
//
// Work decomposition: one CTA per (KV split, sequence x kv head, chunk of RB query rows).  All
// rows of a chunk share the CTA's K/V reads (a row is (query token, head of the GQA group)), so a
// cache row is read once per group instead of once per head as in the reference.  4 warps walk
// interleaved positions; a lane owns D/32 contiguous dims (vector loads); per-warp states are
// merged through shared memory and written as split partials for bg::launch_lse_merge.
#include <math.h>

#include "attn.h"

namespace bg {
namespace {

template <int MODE, int DPL>
__device__ __forceinline__ void load_row(const KVView &kv, bool is_v, uint64_t row, int lane,
                                         float (&x)[DPL]) {
  constexpr int D = DPL * 32;
  const uint64_t off = row * D + (uint64_t)lane * DPL;
  if constexpr (MODE == BG_KV_F32) {
    load_f32<DPL>(static_cast<const float *>(is_v ? kv.V : kv.K) + off, x);
  } else if constexpr (MODE == BG_KV_F16) {
    load_f16<DPL>(static_cast<const __half *>(is_v ? kv.V : kv.K) + off, x);
  } else {
    int8_t c[DPL];
    load_i8<DPL>(static_cast<const int8_t *>(is_v ? kv.V : kv.K) + off, c);
    const float *sc = is_v ? kv.Vs : kv.Ks;
    if constexpr (MODE == BG_KV_Q8) {
      const float s = sc[row * (D / 32) + (lane * DPL) / 32];
#pragma unroll
      for (int i = 0; i < DPL; ++i) x[i] = snorm8(c[i]) * s;
    } else {  // q8r: one absmax/127 scale per 128 elements
      const float s = sc[row * (D / 128) + (lane * DPL) / 128];
#pragma unroll
      for (int i = 0; i < DPL; ++i) x[i] = (float)c[i] * s;
    }
  }
}

template <int MODE, int D, bool ROLL, int RB>
__global__ void __launch_bounds__(128) attn_generic_kernel(AttnArgs a) {
  constexpr int DPL = D / 32;
  constexpr int NW = 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t split = blockIdx.x;
  const uint32_t b = blockIdx.y / a.KV, kvh = blockIdx.y % a.KV;
  const uint32_t G = a.H / a.KV;
  const uint32_t rows = a.S * G;
  const uint32_t r0 = blockIdx.z * RB;

  // rows of this CTA: r -> (qi = r / G, head = kvh*G + r % G)
  float q[RB][DPL];
  uint32_t lastpos[RB];
  uint32_t maxlast = 0;
  const float sl2 = a.scale * kLog2e;
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    const uint32_t rr = r0 + r;
    if (rr < rows) {
      const uint32_t qi = rr / G, h = kvh * G + rr % G;
      const uint64_t qoff = (((uint64_t)b * a.S + qi) * a.H + h) * D + lane * DPL;
      if (a.q_f16) load_f16<DPL>(static_cast<const __half *>(a.q) + qoff, q[r]);
      else load_f32<DPL>(static_cast<const float *>(a.q) + qoff, q[r]);
#pragma unroll
      for (int i = 0; i < DPL; ++i) q[r][i] *= sl2;
      lastpos[r] = a.posBase + qi;
      maxlast = max(maxlast, lastpos[r]);
    } else {
#pragma unroll
      for (int i = 0; i < DPL; ++i) q[r][i] = 0.f;
      lastpos[r] = 0;
    }
  }
  const bool row_valid_any = r0 < rows;
  uint32_t lo = a.pos_lo + split * a.chunk;
  uint32_t hi = min(a.pos_hi, lo + a.chunk);
  hi = min(hi, maxlast + 1);

  float m[RB], l[RB], acc[RB][DPL];
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    m[r] = kNegBig;
    l[r] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[r][i] = 0.f;
  }

  if (row_valid_any) {
    for (uint32_t j = lo + warp; j < hi; j += NW) {
      const uint64_t row = cache_row(a.kv, b, j, kvh);
      float k[DPL], v[DPL];
      load_row<MODE, DPL>(a.kv, false, row, lane, k);
      load_row<MODE, DPL>(a.kv, true, row, lane, v);
      if constexpr (ROLL) {
        // rope-at-read by logical slot j (attention_sg_roll.wgsl:42-50): partner dim d +- D/2
        // is held by lane ^ 16; rotate_half gives -k[d+half] below half, +k[d-half] above.
        constexpr int HALF = D / 2;
        const float *cs = a.cosT + (uint64_t)j * HALF + (lane & 15) * DPL;
        const float *sn = a.sinT + (uint64_t)j * HALF + (lane & 15) * DPL;
        float c[DPL], s[DPL];
        load_f32<DPL>(cs, c);
        load_f32<DPL>(sn, s);
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const float p = __shfl_xor_sync(0xffffffffu, k[i], 16);
          const float rot = lane < 16 ? -p : p;
          k[i] = k[i] * c[i] + rot * s[i];
        }
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        float part = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) part = fmaf(q[r][i], k[i], part);
        float sc = warp_sum(part);
        if (j > lastpos[r]) sc = -INFINITY;
        const float mn = fmaxf(m[r], sc);
        const float corr = exp2f(m[r] - mn);
        const float p = exp2f(sc - mn);
        l[r] = l[r] * corr + p;
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[r][i] = fmaf(acc[r][i], corr, p * v[i]);
        m[r] = mn;
      }
    }
  }

  // merge the 4 warps' states: shared [NW][RB][D + 2]
  extern __shared__ float sh[];
  float *mine = sh + (size_t)warp * RB * (D + 2);
#pragma unroll
  for (int r = 0; r < RB; ++r) {
#pragma unroll
    for (int i = 0; i < DPL; ++i) mine[r * (D + 2) + lane * DPL + i] = acc[r][i];
    if (lane == 0) {
      mine[r * (D + 2) + D] = m[r];
      mine[r * (D + 2) + D + 1] = l[r];
    }
  }
  __syncthreads();
  const uint32_t nrows_total = a.B * a.S * a.H;
  for (int idx = threadIdx.x; idx < RB * D; idx += blockDim.x) {
    const int r = idx / D, d = idx % D;
    const uint32_t rr = r0 + r;
    if (rr >= rows) continue;
    float M = kNegBig;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sh[(w * RB + r) * (D + 2) + D]);
    float o = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float *st = sh + (w * RB + r) * (D + 2);
      const float f = exp2f(st[D] - M);
      o = fmaf(st[d], f, o);
      L = fmaf(st[D + 1], f, L);
    }
    const uint32_t qi = rr / G, h = kvh * G + rr % G;
    const uint64_t grow = ((uint64_t)b * a.S + qi) * a.H + h;
    if (a.out) {  // single split: final output
      float v = o / L;
      if (a.gate) v = v / (1.0f + expf(-a.gate[grow * D + d]));
      if (a.out_f16) static_cast<__half *>(a.out)[grow * D + d] = __float2half_rn(v);
      else static_cast<float *>(a.out)[grow * D + d] = v;
      continue;
    }
    float *dst = a.partials + ((uint64_t)split * nrows_total + grow) * (D + 2);
    dst[d] = o;
    if (d == 0) {
      dst[D] = L > 0.f ? M * kLn2 : -INFINITY;
      dst[D + 1] = L;
    }
  }
}

// Combine split partials [nsplit][rows][D+2] -> out[rows][D], optional sigmoid gate (or, with
// out_f16 < 0, into one partial row (o, m, l) for split-KV slices).  One block per row: the split
// weights exp(m_s - M) are computed in parallel with block reductions, then thread (d, group)
// sums a strided subset of the splits for dim d and the groups are added in shared memory.
__device__ __forceinline__ float block_reduce(float v, float *scratch, bool is_max) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float x = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, x) : v + x;
  }
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = is_max ? -INFINITY : 0.f;
  for (int w = 0; w < nw; ++w) r = is_max ? fmaxf(r, scratch[w]) : r + scratch[w];
  return r;
}

__global__ void lse_merge_kernel(const float *__restrict__ part, uint32_t nsplit, uint32_t rows,
                                 uint32_t D, const float *__restrict__ gate, void *out, int out_f16) {
  const uint32_t row = blockIdx.x;
  extern __shared__ float sm[];  // [nsplit] weights, then [groups][D] partial sums
  float *w = sm;
  float *acc = sm + nsplit;
  __shared__ float red[32];
  const uint64_t stride = (uint64_t)rows * (D + 2);
  const float *base = part + (uint64_t)row * (D + 2);
  float M = -INFINITY;
  for (uint32_t s = threadIdx.x; s < nsplit; s += blockDim.x)
    if (base[s * stride + D + 1] > 0.f) M = fmaxf(M, base[s * stride + D]);
  M = block_reduce(M, red, true);
  float L = 0.f;
  for (uint32_t s = threadIdx.x; s < nsplit; s += blockDim.x) {
    const float l = base[s * stride + D + 1];
    const float f = l > 0.f ? expf(base[s * stride + D] - M) : 0.f;
    w[s] = f;
    L = fmaf(l, f, L);
  }
  L = block_reduce(L, red, false);  // (its barriers also publish w[])
  const uint32_t groups = blockDim.x / D;
  const uint32_t d = threadIdx.x % D, g = threadIdx.x / D;
  if (g < groups) {
    float o = 0.f;
    for (uint32_t s = g; s < nsplit; s += groups) {
      const float f = w[s];
      if (f != 0.f) o = fmaf(base[s * stride + d], f, o);
    }
    acc[g * D + d] = o;
  }
  __syncthreads();
  if (threadIdx.x >= D) return;
  float o = 0.f;
  for (uint32_t k = 0; k < groups; ++k) o += acc[k * D + d];
  if (out_f16 < 0) {
    float *dst = static_cast<float *>(out) + (uint64_t)row * (D + 2);
    dst[d] = o;
    if (d == 0) {
      dst[D] = L > 0.f ? M : -INFINITY;
      dst[D + 1] = L;
    }
    return;
  }
  o = o / L;
  if (gate) o = o / (1.0f + expf(-gate[(uint64_t)row * D + d]));
  if (out_f16) static_cast<__half *>(out)[(uint64_t)row * D + d] = __float2half_rn(o);
  else static_cast<float *>(out)[(uint64_t)row * D + d] = o;
}

// Warp-parallel LSE merge: WPR warps per output row (WPR in {1,2,4,8}), warp k of a row takes
// splits k, k + WPR, ... (at most kMergeSpw each, up to 64 splits).  Every warp loads its o values
// first, then all (m, l) of the row (lane j: splits j, j+32), so a row costs one global round
// trip; the WPR partial sums are combined through shared memory.
constexpr int kMergeSpw = 8;

template <int DPL>
__global__ void __launch_bounds__(256) lse_merge_warp_kernel(const float *__restrict__ part, uint32_t nsplit,
                                                             uint32_t rows, uint32_t wpr,
                                                             const float *__restrict__ gate, void *out,
                                                             int out_f16) {
  constexpr uint32_t D = DPL * 32;
  __shared__ float red[8][D];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t row = blockIdx.x * (8 / wpr) + warp / wpr, k = warp % wpr;
  const bool live = row < rows;
  const uint64_t stride = (uint64_t)rows * (D + 2);
  const float *base = part + (uint64_t)(live ? row : 0) * (D + 2);
  float vals[kMergeSpw][DPL];
#pragma unroll
  for (int i = 0; i < kMergeSpw; ++i) {
    const uint32_t sp = k + i * wpr;
#pragma unroll
    for (int j = 0; j < DPL; ++j) vals[i][j] = (live && sp < nsplit) ? __ldg(base + sp * stride + lane + 32 * j) : 0.f;
  }
  float mv[2], lv[2];
  float M = -INFINITY;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const uint32_t sp = lane + 32 * c;
    mv[c] = -INFINITY;
    lv[c] = 0.f;
    if (live && sp < nsplit) {
      lv[c] = __ldg(base + sp * stride + D + 1);
      mv[c] = __ldg(base + sp * stride + D);
      if (lv[c] > 0.f) M = fmaxf(M, mv[c]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float L = 0.f, f[2];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    f[c] = lv[c] > 0.f ? expf(mv[c] - M) : 0.f;
    L = fmaf(lv[c], f[c], L);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  float acc[DPL];
#pragma unroll
  for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
#pragma unroll
  for (int i = 0; i < kMergeSpw; ++i) {
    const uint32_t sp = k + i * wpr;  // warp-uniform
    const float fs = __shfl_sync(0xffffffffu, sp < 32 ? f[0] : f[1], sp & 31);
    const bool use = sp < nsplit && fs != 0.f;  // empty slots may hold any bits
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[j] = use ? fmaf(vals[i][j], fs, acc[j]) : acc[j];
  }
  if (wpr > 1) {
#pragma unroll
    for (int j = 0; j < DPL; ++j) red[warp][lane + 32 * j] = acc[j];
    __syncthreads();
    if (k != 0) return;
    for (uint32_t w = 1; w < wpr; ++w)
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[j] += red[warp + w][lane + 32 * j];
  }
  if (!live) return;
  if (out_f16 < 0) {
    float *dst = static_cast<float *>(out) + (uint64_t)row * (D + 2);
#pragma unroll
    for (int j = 0; j < DPL; ++j) dst[lane + 32 * j] = acc[j];
    if (lane == 0) {
      dst[D] = L > 0.f ? M : -INFINITY;
      dst[D + 1] = L;
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < DPL; ++j) {
    const uint32_t d = lane + 32 * j;
    float o = acc[j] / L;
    if (gate) o = o / (1.0f + expf(-gate[(uint64_t)row * D + d]));
    if (out_f16) static_cast<__half *>(out)[(uint64_t)row * D + d] = __float2half_rn(o);
    else static_cast<float *>(out)[(uint64_t)row * D + d] = o;
  }
}

// LSE merge for many splits: CTA (row, 64-column slice), its 8 warps take splits w, w + 8, ...;
// each warp reduces (m, l) of every split (lane-strided), then loads its splits' 64 o values in
// batches of 8 before any arithmetic, and the 8 partial sums meet in shared memory.  Launched as a
// programmatic dependent of the decode kernel: its start-up overlaps that kernel's tail.
constexpr int kWideCols = 64;

__global__ void __launch_bounds__(256) lse_merge_wide_kernel(const float *__restrict__ part, uint32_t nsplit,
                                                             uint32_t rows, uint32_t D, const float *__restrict__ gate,
                                                             void *out, int out_f16) {
  __shared__ float red[8][kWideCols];
  __shared__ float lsum[8];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t row = blockIdx.x, c0 = blockIdx.y * kWideCols;
  const uint64_t stride = (uint64_t)rows * (D + 2);
  const float *base = part + (uint64_t)row * (D + 2);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float M = -INFINITY;
  for (uint32_t s = lane; s < nsplit; s += 32) {
    const float l = __ldcg(base + s * stride + D + 1), m = __ldcg(base + s * stride + D);
    if (l > 0.f) M = fmaxf(M, m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float a0 = 0.f, a1 = 0.f, L = 0.f;
  for (uint32_t s0 = warp; s0 < nsplit; s0 += 64) {
    float v0[8], v1[8], f[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t s = s0 + 8 * i;
      const bool in = s < nsplit;
      const float *src = base + (uint64_t)(in ? s : 0) * stride;
      const float l = in ? __ldcg(src + D + 1) : 0.f, m = in ? __ldcg(src + D) : 0.f;
      f[i] = l > 0.f ? expf(m - M) : 0.f;  // empty slots may hold any bits
      L = fmaf(l > 0.f ? l : 0.f, f[i], L);
      v0[i] = in ? __ldcg(src + c0 + lane) : 0.f;
      v1[i] = in ? __ldcg(src + c0 + 32 + lane) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (f[i] != 0.f) {
        a0 = fmaf(v0[i], f[i], a0);
        a1 = fmaf(v1[i], f[i], a1);
      }
    }
  }
  red[warp][lane] = a0;
  red[warp][lane + 32] = a1;
  if (lane == 0) lsum[warp] = L;
  __syncthreads();
  if (warp != 0) return;
#pragma unroll
  for (int w = 1; w < 8; ++w) {
    a0 += red[w][lane];
    a1 += red[w][lane + 32];
  }
  L = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) L += lsum[w];
  if (out_f16 < 0) {
    float *dst = static_cast<float *>(out) + (uint64_t)row * (D + 2);
    dst[c0 + lane] = a0;
    dst[c0 + 32 + lane] = a1;
    if (c0 == 0 && lane == 0) {
      dst[D] = L > 0.f ? M : -INFINITY;
      dst[D + 1] = L;
    }
    return;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t d = c0 + lane + 32 * h;
    float o = (h ? a1 : a0) / L;
    if (gate) o = o / (1.0f + expf(-gate[(uint64_t)row * D + d]));
    if (out_f16) static_cast<__half *>(out)[(uint64_t)row * D + d] = __float2half_rn(o);
    else static_cast<float *>(out)[(uint64_t)row * D + d] = o;
  }
}

template <int MODE, int D, bool ROLL>
int launch_rb(const AttnArgs &a, cudaStream_t st) {
  const uint32_t rows = a.S * (a.H / a.KV);
  constexpr int RBMAX = D >= 256 ? 4 : 8;
  auto go = [&](auto rbc) -> int {
    constexpr int RB = decltype(rbc)::value;
    dim3 grid(a.nsplit, a.B * a.KV, (rows + RB - 1) / RB);
    const size_t smem = (size_t)4 * RB * (D + 2) * sizeof(float);
    auto kern = attn_generic_kernel<MODE, D, ROLL, RB>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, 128, smem, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
  };
  if (rows <= 1) return go(std::integral_constant<int, 1>{});
  if (rows <= 2) return go(std::integral_constant<int, 2>{});
  if (rows <= 4 || RBMAX == 4) return go(std::integral_constant<int, (RBMAX < 4 ? RBMAX : 4)>{});
  return go(std::integral_constant<int, RBMAX>{});
}

template <int MODE, int D>
int launch_roll(const AttnArgs &a, cudaStream_t st) {
  return a.cosT ? launch_rb<MODE, D, true>(a, st) : launch_rb<MODE, D, false>(a, st);
}

template <int MODE>
int launch_d(const AttnArgs &a, cudaStream_t st) {
  switch (a.D) {
    case 64: return launch_roll<MODE, 64>(a, st);
    case 128: return launch_roll<MODE, 128>(a, st);
    case 256: return launch_roll<MODE, 256>(a, st);
    default: return BG_EUNSUPPORTED;
  }
}

}  // namespace

namespace {

template <int MODE, int D, bool ROLL, int RB>
int generic_occ() {
  static int cached = 0;
  if (!cached) {
    int n = 0;
    const int smem = 4 * RB * (D + 2) * (int)sizeof(float);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_generic_kernel<MODE, D, ROLL, RB>, 128, smem) !=
            cudaSuccess ||
        n < 1)
      n = 1;
    cached = n;
  }
  return cached;
}

template <int MODE, int D>
int generic_occ_rb(uint32_t rows, bool roll) {
  constexpr int RBMAX = D >= 256 ? 4 : 8;
  auto pick = [&](auto rbc) -> int {
    constexpr int RB = decltype(rbc)::value;
    return roll ? generic_occ<MODE, D, true, RB>() : generic_occ<MODE, D, false, RB>();
  };
  if (rows <= 1) return pick(std::integral_constant<int, 1>{});
  if (rows <= 2) return pick(std::integral_constant<int, 2>{});
  if (rows <= 4 || RBMAX == 4) return pick(std::integral_constant<int, (RBMAX < 4 ? RBMAX : 4)>{});
  return pick(std::integral_constant<int, RBMAX>{});
}

template <int MODE>
int generic_occ_d(uint32_t D, uint32_t rows, bool roll) {
  switch (D) {
    case 64: return generic_occ_rb<MODE, 64>(rows, roll);
    case 128: return generic_occ_rb<MODE, 128>(rows, roll);
    default: return generic_occ_rb<MODE, 256>(rows, roll);
  }
}

uint32_t kv_row_bytes(int mode, uint32_t D) {
  switch (mode) {
    case BG_KV_F32: return 4 * D;
    case BG_KV_F16: return 2 * D;
    case BG_KV_Q8: return D + D / 8;
    default: return D + D / 32;
  }
}

}  // namespace

int attn_generic_ctas_per_sm(int mode, uint32_t D, uint32_t rows, bool roll) {
  switch (mode) {
    case BG_KV_F32: return generic_occ_d<BG_KV_F32>(D, rows, roll);
    case BG_KV_F16: return generic_occ_d<BG_KV_F16>(D, rows, roll);
    case BG_KV_Q8: return generic_occ_d<BG_KV_Q8>(D, rows, roll);
    default: return D % 128 ? 1 : generic_occ_d<BG_KV_Q8R>(D, rows, roll);
  }
}

// Split count from a small cost model in units of bytes moved at full HBM rate:
//   waves(n) * slots * (bytes of one CTA's slice + pipeline ramp)  +  n * partial-row traffic,
// where a CTA's slice is the unit's cache bytes / n and `slots` = resident CTAs on 148 SMs.
// The first term rewards filling the last wave; the second charges the split partials'
// write + merge read.  Splits never get shorter than 256 positions.
uint32_t attn_num_splits(uint32_t B, uint32_t S, uint32_t H, uint32_t KV, uint32_t D, uint32_t L, int mode, bool tc,
                         bool roll) {
  if (tc && roll && attn_roll_supported(mode, D, S, H, KV) && !roll_legacy()) return attn_roll_num_splits(mode, B, KV, L);
  const uint32_t G = H / KV;
  const uint32_t M = S * G;
  const uint32_t rb = D >= 256 ? 4 : 8;
  const uint64_t rowchunks = tc ? 1 : (M + rb - 1) / rb;
  const uint64_t units = (uint64_t)B * KV * rowchunks;
  const int per_sm = tc ? attn_tc_ctas_per_sm(mode, D, M, roll) : attn_generic_ctas_per_sm(mode, D, M, roll);
  const double slots = 148.0 * per_sm;
  const double unit_bytes = 2.0 * L * kv_row_bytes(mode, D);
  const double ramp = 2.0 * 64 * 2 * kv_row_bytes(mode, D);
  const double split_bytes = (double)B * S * H * (D + 2) * 8.0;
  uint64_t maxs = (L + 255) / 256;
  if (maxs > 128) maxs = 128;
  if (maxs < 1) maxs = 1;
  uint32_t best = 1;
  double best_cost = 0;
  for (uint64_t n = 1; n <= maxs; ++n) {
    const double waves = (double)((units * n + (uint64_t)slots - 1) / (uint64_t)slots);
    const double cost = waves * slots * (unit_bytes / n + ramp) + n * split_bytes;
    if (n == 1 || cost < best_cost * 0.999) {
      best = (uint32_t)n;
      best_cost = cost;
    }
  }
  return best;
}

uint32_t attn_max_splits(uint32_t B, uint32_t S, uint32_t H, uint32_t KV, uint32_t D, uint32_t L) {
  uint32_t m = 1;
  for (int mode = BG_KV_F32; mode <= BG_KV_Q8R; ++mode) {
    if (mode == BG_KV_Q8R && D % 128) continue;
    const uint32_t a = attn_num_splits(B, S, H, KV, D, L, mode, false);
    m = a > m ? a : m;
    for (int roll = 0; roll < 2; ++roll) {
      if (attn_tc_supported(mode, D, S, H, KV, roll, false)) {
        const uint32_t t = attn_num_splits(B, S, H, KV, D, L, mode, true, roll);
        m = t > m ? t : m;
      }
      const uint32_t g = attn_num_splits(B, S, H, KV, D, L, mode, false, roll);
      m = g > m ? g : m;
    }
  }
  return m;
}

int launch_attn_generic(const AttnArgs &a, cudaStream_t st) {
  switch (a.mode) {
    case BG_KV_F32: return launch_d<BG_KV_F32>(a, st);
    case BG_KV_F16: return launch_d<BG_KV_F16>(a, st);
    case BG_KV_Q8: return launch_d<BG_KV_Q8>(a, st);
    case BG_KV_Q8R: return a.D % 128 ? BG_EUNSUPPORTED : launch_d<BG_KV_Q8R>(a, st);
    default: return BG_EINVAL;
  }
}

int launch_lse_merge(const float *partials, uint32_t nsplit, uint32_t rows, uint32_t D,
                     const float *gate, void *out, int out_f16, cudaStream_t st) {
  if (rows == 0) return BG_OK;
  if (D > 1024) return BG_EUNSUPPORTED;
  if (nsplit > 16 && D % kWideCols == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows, D / kWideCols);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, lse_merge_wide_kernel, partials, nsplit, rows, D, gate, out, out_f16) == cudaSuccess
               ? BG_OK
               : BG_ELAUNCH;
  }
  if (nsplit <= 8 * kMergeSpw && (D == 64 || D == 128 || D == 256)) {
    uint32_t wpr = 1;
    while (wpr * kMergeSpw < nsplit) wpr *= 2;
    const uint32_t rpb = 8 / wpr, blocks = (rows + rpb - 1) / rpb;
    if (D == 64) lse_merge_warp_kernel<2><<<blocks, 256, 0, st>>>(partials, nsplit, rows, wpr, gate, out, out_f16);
    else if (D == 128) lse_merge_warp_kernel<4><<<blocks, 256, 0, st>>>(partials, nsplit, rows, wpr, gate, out, out_f16);
    else lse_merge_warp_kernel<8><<<blocks, 256, 0, st>>>(partials, nsplit, rows, wpr, gate, out, out_f16);
    return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
  }
  // as many split groups as fit 1024 threads, but no more than there are splits
  uint32_t groups = 1024 / D;
  if (groups > nsplit) groups = nsplit;
  if (groups < 1) groups = 1;
  const uint32_t threads = ((groups * D + 31) / 32) * 32;
  const size_t smem = (size_t)(nsplit + groups * D) * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(lse_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return BG_EUNSUPPORTED;
  lse_merge_kernel<<<rows, threads, smem, st>>>(partials, nsplit, rows, D, gate, out, out_f16);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

}  // namespace bg
