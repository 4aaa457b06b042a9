// Hybrid-layer glue around the DeltaNet scan and the gated attention (engine.ts:1418-1432,
// 1471-1474): the depthwise causal conv1d + SiLU with its carried left context
// (conv1d_causal.wgsl) and the column slice that splits q|k|v and query|gate (slice_cols.wgsl,
// split_head.wgsl).  Both are HBM-bound elementwise passes.
#include "kv.h"

namespace bg {
namespace {

constexpr int kConvT = 32;  // tokens per thread: a thread walks one channel down kConvT rows

// conv1d_causal.wgsl:18-35.  Thread = (channel c, run of kConvT tokens); the extended input
// ext = [state_in (K-1 rows, zero unless load_state); x] is read down the channel with the
// previous K-1 values kept in registers, so each input is loaded once per run.  Loads and stores
// of a warp are 32 consecutive channels of one row.
template <int K>
__global__ void conv1d_causal_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                     const float *__restrict__ state_in, int load_state, uint32_t S, uint32_t C,
                                     float *__restrict__ y, float *__restrict__ state_out) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t t0 = blockIdx.y * kConvT;
  if (c >= C) return;
  float wc[K];
#pragma unroll
  for (int j = 0; j < K; ++j) wc[j] = w[(uint64_t)c * K + j];
  // ext row m (m = t + j for output t): m < K-1 -> state_in[m], else x[m - (K-1)]
  auto ext = [&](uint32_t m) -> float {
    if (m + 1 < (uint32_t)K) return load_state ? state_in[(uint64_t)m * C + c] : 0.f;
    return x[(uint64_t)(m - (K - 1)) * C + c];
  };
  float win[K];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) win[j] = ext(t0 + j);
  const uint32_t t1 = min(S, t0 + kConvT);
  for (uint32_t t = t0; t < t1; ++t) {
    win[K - 1] = x[(uint64_t)t * C + c];  // ext row t + K - 1
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) acc += wc[j] * win[j];
    y[(uint64_t)t * C + c] = acc / (1.0f + expf(-acc));  // SiLU
#pragma unroll
    for (int j = 0; j < K - 1; ++j) win[j] = win[j + 1];
  }
  if (blockIdx.y == gridDim.y - 1) {
    // state_out[i] = ext[S + i], i < K-1 (the last K-1 rows of the extended input)
#pragma unroll
    for (int i = 0; i < K - 1; ++i) state_out[(uint64_t)i * C + c] = ext(S + i);
  }
}

__global__ void slice_cols_kernel(const float *__restrict__ src, uint32_t rows, uint32_t width, uint32_t stride,
                                  uint32_t off, float *__restrict__ dst) {
  const uint64_t n = (uint64_t)rows * width;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = i / width, c = i % width;
    dst[i] = src[r * stride + off + c];
  }
}

__global__ void slice_cols_vec4_kernel(const float4 *__restrict__ src, uint32_t rows, uint32_t w4, uint32_t stride4,
                                       uint32_t off4, float4 *__restrict__ dst) {
  const uint64_t n = (uint64_t)rows * w4;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = i / w4, c = i % w4;
    dst[i] = src[r * stride4 + off4 + c];
  }
}

}  // namespace

int launch_conv1d_causal(const float *x, const float *w, const float *state_in, int load_state, uint32_t S,
                         uint32_t C, uint32_t K, float *y, float *state_out, cudaStream_t st) {
  const dim3 grid((C + 127) / 128, S ? (S + kConvT - 1) / kConvT : 1);
  switch (K) {
#define BG_CONV(K_) \
  case K_: conv1d_causal_kernel<K_><<<grid, 128, 0, st>>>(x, w, state_in, load_state, S, C, y, state_out); break;
    BG_CONV(2)
    BG_CONV(3)
    BG_CONV(4)
    BG_CONV(5)
    BG_CONV(6)
    BG_CONV(7)
    BG_CONV(8)
#undef BG_CONV
    default: return BG_EUNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int launch_slice_cols(const float *src, uint32_t rows, uint32_t width, uint32_t stride, uint32_t off, float *dst,
                      cudaStream_t st) {
  const uint64_t n = (uint64_t)rows * width;
  if (n == 0) return BG_OK;
  const bool v4 = width % 4 == 0 && stride % 4 == 0 && off % 4 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(dst) % 16 == 0;
  const uint64_t items = v4 ? n / 4 : n;
  const uint64_t want = (items + 255) / 256, cap = 148ull * 16;
  const uint32_t blocks = (uint32_t)(want < cap ? want : cap);
  if (v4)
    slice_cols_vec4_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const float4 *>(src), rows, width / 4, stride / 4,
                                                   off / 4, reinterpret_cast<float4 *>(dst));
  else
    slice_cols_kernel<<<blocks, 256, 0, st>>>(src, rows, width, stride, off, dst);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

}  // namespace bg
