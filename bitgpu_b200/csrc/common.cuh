// Shared device helpers for the bitgpu B200 attention library (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bgattn.h"

namespace bg {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kNegBig = -1e30f;  // the reference's running-max seed (attention_sg.wgsl:29)

// Device view of one layer's cache plus the geometry the kernels need.
struct KVView {
  const void *K, *V;
  const float *Ks, *Vs;
  uint64_t seq_stride;
  uint32_t sinks, window, ring_head;
  uint32_t KV;
  uint32_t row_offset;  // logical position of physical row 0 (split-KV slices)
};

// Logical cache slot -> physical row of the sequence slab (ring layout when window > 0).
__device__ __forceinline__ uint32_t phys_pos(const KVView &kv, uint32_t p) {
  p -= kv.row_offset;
  if (kv.window == 0 || p < kv.sinks) return p;
  return kv.sinks + (kv.ring_head + (p - kv.sinks)) % kv.window;
}

__device__ __forceinline__ uint64_t cache_row(const KVView &kv, uint32_t b, uint32_t p, uint32_t kvh) {
  return ((uint64_t)b * kv.seq_stride + phys_pos(kv, p)) * kv.KV + kvh;
}

template <int N>
__device__ __forceinline__ void load_f32(const float *src, float (&dst)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      float4 t = *reinterpret_cast<const float4 *>(src + i);
      dst[i] = t.x; dst[i + 1] = t.y; dst[i + 2] = t.z; dst[i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      float2 t = *reinterpret_cast<const float2 *>(src + i);
      dst[i] = t.x; dst[i + 1] = t.y;
    }
  }
}

template <int N>
__device__ __forceinline__ void load_f16(const __half *src, float (&dst)[N]) {
  if constexpr (N % 8 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 8) {
      uint4 t = *reinterpret_cast<const uint4 *>(src + i);
      const __half2 *h = reinterpret_cast<const __half2 *>(&t);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __half22float2(h[j]);
        dst[i + 2 * j] = f.x; dst[i + 2 * j + 1] = f.y;
      }
    }
  } else if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      uint2 t = *reinterpret_cast<const uint2 *>(src + i);
      const __half2 *h = reinterpret_cast<const __half2 *>(&t);
      float2 a = __half22float2(h[0]), b = __half22float2(h[1]);
      dst[i] = a.x; dst[i + 1] = a.y; dst[i + 2] = b.x; dst[i + 3] = b.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      float2 a = __half22float2(*reinterpret_cast<const __half2 *>(src + i));
      dst[i] = a.x; dst[i + 1] = a.y;
    }
  }
}

// snorm8 decode of the reference: unpack4x8snorm = max(code/127, -1) (attention_sg_kv8.wgsl:40).
__device__ __forceinline__ float snorm8(int8_t c) { return fmaxf((float)c * (1.0f / 127.0f), -1.0f); }

template <int N>
__device__ __forceinline__ void load_i8(const int8_t *src, int8_t (&dst)[N]) {
  if constexpr (N == 8) {
    uint2 t = *reinterpret_cast<const uint2 *>(src);
    const int8_t *c = reinterpret_cast<const int8_t *>(&t);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = c[i];
  } else if constexpr (N == 4) {
    uint32_t t = *reinterpret_cast<const uint32_t *>(src);
    const int8_t *c = reinterpret_cast<const int8_t *>(&t);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = c[i];
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) dst[i] = src[i];
  }
}

// q8 encode of one value with its block scale: pack4x8snorm(v/s) component
// = floor(0.5 + 127*clamp(v/s, -1, 1)) (shaders/copy_kv8.wgsl:39, WGSL pack4x8snorm).
__device__ __forceinline__ int8_t snorm8_encode(float v, float s) {
  float e = __fdiv_rn(v, s);
  e = fminf(fmaxf(e, -1.0f), 1.0f);
  return (int8_t)(int)floorf(0.5f + 127.0f * e);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace bg
