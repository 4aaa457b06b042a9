// KV-cache writers: append (copy.wgsl / copy_kv16.wgsl / copy_kv8.wgsl), fused per-head RMSNorm
// + RoPE + cache write (rmsnorm_rope_sg{,_kv16,_kv8}.wgsl) and sink-eviction compaction
// (src/engine.ts:1188-1212).  One warp per cache row; a lane owns D/32 contiguous values, so a
// q8 block of 32 values is owned by 32/(D/32) adjacent lanes and its absmax is a short
// butterfly.  The q8 encode is bit-exact to the reference rule (see snorm8_encode).
#include "kv.h"

namespace bg {
namespace {

template <int DPL>
__device__ __forceinline__ void load_src(const void *src, int f16, uint64_t off, float (&x)[DPL]) {
  if (f16) load_f16<DPL>(static_cast<const __half *>(src) + off, x);
  else load_f32<DPL>(static_cast<const float *>(src) + off, x);
}

// Store one row (lane's DPL values) into the cache at `row` with the cache's codec.
template <int DPL>
__device__ __forceinline__ void store_row(void *data, float *scales, int mode, uint64_t row, int lane,
                                          const float (&x)[DPL]) {
  constexpr int D = DPL * 32;
  const uint64_t off = row * D + (uint64_t)lane * DPL;
  // a lane's DPL values are contiguous: one vector store per lane (DPL = 2, 4, 8)
  if (mode == BG_KV_F32) {
    float *d = static_cast<float *>(data) + off;
    if constexpr (DPL % 4 == 0) {
#pragma unroll
      for (int i = 0; i < DPL; i += 4) *reinterpret_cast<float4 *>(d + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < DPL; i += 2) *reinterpret_cast<float2 *>(d + i) = make_float2(x[i], x[i + 1]);
    }
  } else if (mode == BG_KV_F16) {
    __half *d = static_cast<__half *>(data) + off;
    uint32_t w[DPL / 2];
#pragma unroll
    for (int i = 0; i < DPL; i += 2) {
      __half2 hv = __floats2half2_rn(x[i], x[i + 1]);
      w[i / 2] = *reinterpret_cast<uint32_t *>(&hv);
    }
    if constexpr (DPL == 8) *reinterpret_cast<uint4 *>(d) = make_uint4(w[0], w[1], w[2], w[3]);
    else if constexpr (DPL == 4) *reinterpret_cast<uint2 *>(d) = make_uint2(w[0], w[1]);
    else *reinterpret_cast<uint32_t *>(d) = w[0];
  } else if (mode == BG_KV_Q8) {
    // per 32-element block: s = max(absmax, 1e-30) (copy_kv8.wgsl:30-35)
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) am = fmaxf(am, fabsf(x[i]));
    constexpr int LPB = 32 / DPL;  // lanes per 32-block
#pragma unroll
    for (int o = LPB / 2; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const float s = fmaxf(am, 1e-30f);
    int8_t *d = static_cast<int8_t *>(data) + off;
    uint32_t w[(DPL + 3) / 4] = {};
#pragma unroll
    for (int i = 0; i < DPL; ++i) w[i / 4] |= (uint32_t)(uint8_t)snorm8_encode(x[i], s) << (8 * (i % 4));
    if constexpr (DPL == 8) *reinterpret_cast<uint2 *>(d) = make_uint2(w[0], w[1]);
    else if constexpr (DPL == 4) *reinterpret_cast<uint32_t *>(d) = w[0];
    else *reinterpret_cast<uint16_t *>(d) = (uint16_t)w[0];
    if ((lane % LPB) == 0) scales[row * (D / 32) + (lane * DPL) / 32] = s;
  } else {  // BG_KV_Q8R: absmax/127 per 128 values, round-half-even
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) am = fmaxf(am, fabsf(x[i]));
    constexpr int LPB = 128 / DPL;
#pragma unroll
    for (int o = (LPB > 32 ? 16 : LPB / 2); o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const float s = am / 127.0f;
    const float sd = s > 0.f ? s : 1.0f;
    int8_t *d = static_cast<int8_t *>(data) + off;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      float c = rintf(__fdiv_rn(x[i], sd));
      c = fminf(fmaxf(c, -127.f), 127.f);
      d[i] = (int8_t)(int)c;
    }
    if ((lane * DPL) % 128 == 0) scales[row * (D / 128) + (lane * DPL) / 128] = s;
  }
}

// Rows [side][b][s][kv]: side 0 writes src0 into the cache's `first_v ? V : K`, side 1 (when
// nsides == 2) writes src1 into V.  With kv2.K != nullptr the same rows also go into a second cache
// (its own codec), read from the source once.
template <int DPL>
__global__ void kv_append_kernel(KVView kv, int mode, KVView kv2, int mode2, const void *src0, const void *src1,
                                 int src_f16, uint32_t B, uint32_t S, uint32_t pos0, int first_v, int nsides) {
  constexpr int D = DPL * 32;
  const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t total = B * S * kv.KV;
  if (gw >= total * nsides) return;
  const int side = gw >= total;
  const uint32_t r = gw - side * total;
  const uint32_t kvh = r % kv.KV, s = (r / kv.KV) % S, b = r / (kv.KV * S);
  const bool to_v = side || first_v;
  float x[DPL];
  load_src<DPL>(side ? src1 : src0, src_f16, (uint64_t)r * D + lane * DPL, x);
  const uint64_t row = cache_row(kv, b, pos0 + s, kvh);
  store_row<DPL>(const_cast<void *>(to_v ? kv.V : kv.K), const_cast<float *>(to_v ? kv.Vs : kv.Ks), mode, row, lane,
                 x);
  if (kv2.K) {
    const uint64_t row2 = cache_row(kv2, b, pos0 + s, kvh);
    store_row<DPL>(const_cast<void *>(to_v ? kv2.V : kv2.K), const_cast<float *>(to_v ? kv2.Vs : kv2.Ks), mode2, row2,
                   lane, x);
  }
}

// rmsnorm_rope_sg.wgsl:21-33 (+ the _kv8 write side): y = (x*inv*gamma) rotated by cos/sin.
template <int DPL>
__global__ void rmsnorm_rope_kernel(const float *x, uint32_t B, uint32_t R, const float *gamma, const float *cosv,
                                    const float *sinv, float eps, float *y, KVView kv, int mode, uint32_t pos,
                                    int to_cache) {
  constexpr int D = DPL * 32;
  const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= B * R) return;
  float v[DPL], g[DPL];
  load_f32<DPL>(x + (uint64_t)gw * D + lane * DPL, v);
  load_f32<DPL>(gamma + lane * DPL, g);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < DPL; ++i) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / (float)D + eps);
  float nd[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) nd[i] = v[i] * inv * g[i];
  float out[DPL];
  if (cosv) {
    float c[DPL], s[DPL];
    load_f32<DPL>(cosv + lane * DPL, c);
    load_f32<DPL>(sinv + lane * DPL, s);
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const float p = __shfl_xor_sync(0xffffffffu, nd[i], 16);
      const float rot = lane < 16 ? -p : p;
      out[i] = nd[i] * c[i] + rot * s[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < DPL; ++i) out[i] = nd[i];
  }
  if (y) {
#pragma unroll
    for (int i = 0; i < DPL; ++i) y[(uint64_t)gw * D + lane * DPL + i] = out[i];
  }
  if (to_cache) {
    const uint32_t r = gw % R, b = gw / R;
    store_row<DPL>(const_cast<void *>(kv.K), const_cast<float *>(kv.Ks), mode, cache_row(kv, b, pos, r), lane, out);
  }
}

__global__ void copy_rows_kernel(uint8_t *base, uint64_t seq_bytes, uint64_t dst_off, uint64_t src_off,
                                 uint64_t nbytes) {
  uint8_t *seq = base + blockIdx.y * seq_bytes;
  if ((nbytes & 15) == 0 && (dst_off & 15) == 0 && (src_off & 15) == 0 && (seq_bytes & 15) == 0) {
    const uint4 *s = reinterpret_cast<const uint4 *>(seq + src_off);
    uint4 *d = reinterpret_cast<uint4 *>(seq + dst_off);
    for (uint64_t i = blockIdx.x * blockDim.x + threadIdx.x; i < nbytes / 16; i += (uint64_t)gridDim.x * blockDim.x)
      d[i] = s[i];
  } else {
    for (uint64_t i = blockIdx.x * blockDim.x + threadIdx.x; i < nbytes; i += (uint64_t)gridDim.x * blockDim.x)
      seq[dst_off + i] = seq[src_off + i];
  }
}

// The gated-attention prologue of engine.ts:1471-1485 for one head row (b, s, h), one warp:
// split_head (the row is read at x + ((b*S + s)*heads + h)*x_stride + x_off), the plain RMSNorm
// with its baked scale (rms, y = x * rsqrt(mean(x^2) + eps) * gamma), rope_partial.wgsl:12-24
// (rotate_half inside the first `rot` dims, tables [pos][rot] at row pos0 + s, the rest passes
// through) and optionally the cache write of the result at logical position pos0 + s (appendKV).
template <int DPL>
__global__ void qk_norm_rope_kernel(const float *x, uint32_t B, uint32_t S, uint32_t heads, uint32_t x_stride,
                                    uint32_t x_off, const float *gamma, const float *cosT, const float *sinT,
                                    uint32_t rot, uint32_t pos0, float eps, float *y, KVView kv, int mode,
                                    int to_cache) {
  constexpr int D = DPL * 32;
  const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= B * S * heads) return;
  const float *src = x + (uint64_t)gw * x_stride + x_off;
  float v[DPL], g[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    v[i] = src[lane * DPL + i];
    g[i] = gamma[lane * DPL + i];
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < DPL; ++i) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / (float)D + eps);
  const uint32_t s = (gw / heads) % S;
  const uint32_t half = rot / 2;
  float out[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const uint32_t d = lane * DPL + i;
    const float nd = v[i] * inv * g[i];
    if (d < rot) {
      const uint32_t pd = d < half ? d + half : d - half;
      const float np = src[pd] * inv * gamma[pd];
      const float rv = d < half ? -np : np;
      const uint64_t t = (uint64_t)(pos0 + s) * rot + d;
      out[i] = nd * cosT[t] + rv * sinT[t];
    } else {
      out[i] = nd;
    }
  }
  if (y) {
#pragma unroll
    for (int i = 0; i < DPL; ++i) y[(uint64_t)gw * D + lane * DPL + i] = out[i];
  }
  if (to_cache) {
    const uint32_t h = gw % heads, b = gw / (heads * S);
    const uint64_t row = cache_row(kv, b, pos0 + s, h);
    store_row<DPL>(const_cast<void *>(kv.K), const_cast<float *>(kv.Ks), mode, row, lane, out);
  }
}

template <int DPL>
int launch_append_d(const KVView &kv, int mode, const KVView &kv2, int mode2, const void *src0, const void *src1,
                    int f16, uint32_t B, uint32_t S, uint32_t pos0, int first_v, int nsides, cudaStream_t st) {
  const uint64_t warps = (uint64_t)B * S * kv.KV * nsides;
  const uint32_t blocks = (uint32_t)((warps * 32 + 255) / 256);
  kv_append_kernel<DPL><<<blocks, 256, 0, st>>>(kv, mode, kv2, mode2, src0, src1, f16, B, S, pos0, first_v, nsides);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

}  // namespace

int launch_kv_append(const KVView &kv, int mode, uint32_t D, const void *src0, const void *src1, int src_f16,
                     uint32_t B, uint32_t S, uint32_t pos0, int first_v, int nsides, cudaStream_t st,
                     const KVView *kv2, int mode2) {
  KVView none = kv;
  none.K = none.V = nullptr;
  const KVView &k2 = kv2 ? *kv2 : none;
  switch (D) {
    case 64: return launch_append_d<2>(kv, mode, k2, mode2, src0, src1, src_f16, B, S, pos0, first_v, nsides, st);
    case 128: return launch_append_d<4>(kv, mode, k2, mode2, src0, src1, src_f16, B, S, pos0, first_v, nsides, st);
    case 256: return launch_append_d<8>(kv, mode, k2, mode2, src0, src1, src_f16, B, S, pos0, first_v, nsides, st);
    default: return BG_EUNSUPPORTED;
  }
}

int launch_rmsnorm_rope(const float *x, uint32_t B, uint32_t R, uint32_t D, const float *gamma, const float *cosv,
                        const float *sinv, float eps, float *y, const KVView &kv, int mode, uint32_t pos, int to_cache,
                        cudaStream_t st) {
  const uint64_t warps = (uint64_t)B * R;
  const uint32_t blocks = (uint32_t)((warps * 32 + 127) / 128);
  switch (D) {
    case 64: rmsnorm_rope_kernel<2><<<blocks, 128, 0, st>>>(x, B, R, gamma, cosv, sinv, eps, y, kv, mode, pos, to_cache); break;
    case 128: rmsnorm_rope_kernel<4><<<blocks, 128, 0, st>>>(x, B, R, gamma, cosv, sinv, eps, y, kv, mode, pos, to_cache); break;
    case 256: rmsnorm_rope_kernel<8><<<blocks, 128, 0, st>>>(x, B, R, gamma, cosv, sinv, eps, y, kv, mode, pos, to_cache); break;
    default: return BG_EUNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int launch_qk_norm_rope(const float *x, uint32_t B, uint32_t S, uint32_t heads, uint32_t D, uint32_t x_stride,
                        uint32_t x_off, const float *gamma, const float *cosT, const float *sinT, uint32_t rot,
                        uint32_t pos0, float eps, float *y, const KVView &kv, int mode, int to_cache,
                        cudaStream_t st) {
  const uint64_t warps = (uint64_t)B * S * heads;
  const uint32_t blocks = (uint32_t)((warps * 32 + 127) / 128);
#define BG_QKNR(DPL_)                                                                                        \
  qk_norm_rope_kernel<DPL_><<<blocks, 128, 0, st>>>(x, B, S, heads, x_stride, x_off, gamma, cosT, sinT, rot, \
                                                    pos0, eps, y, kv, mode, to_cache)
  switch (D) {
    case 64: BG_QKNR(2); break;
    case 128: BG_QKNR(4); break;
    case 256: BG_QKNR(8); break;
    default: return BG_EUNSUPPORTED;
  }
#undef BG_QKNR
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int launch_copy_rows(void *base, uint64_t seq_bytes, uint32_t B, uint64_t dst_off, uint64_t src_off, uint64_t nbytes,
                     cudaStream_t st) {
  if (nbytes == 0 || B == 0) return BG_OK;
  uint64_t units = (nbytes + 15) / 16;
  uint32_t gx = (uint32_t)((units + 255) / 256);
  if (gx > 1184) gx = 1184;
  copy_rows_kernel<<<dim3(gx, B), 256, 0, st>>>(static_cast<uint8_t *>(base), seq_bytes, dst_off, src_off, nbytes);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

}  // namespace bg
