// Internal launch interface of the KV-cache writers and the DeltaNet kernels.
#pragma once
#include "common.cuh"

namespace bg {

// nsides 1: src0 -> K (first_v = 0) or V (first_v = 1); nsides 2: src0 -> K and src1 -> V.
int launch_kv_append(const KVView &kv, int mode, uint32_t D, const void *src0, const void *src1, int src_f16,
                     uint32_t B, uint32_t S, uint32_t pos0, int first_v, int nsides, cudaStream_t st,
                     const KVView *kv2 = nullptr, int mode2 = 0);
int launch_rmsnorm_rope(const float *x, uint32_t B, uint32_t R, uint32_t D, const float *gamma, const float *cosv,
                        const float *sinv, float eps, float *y, const KVView &kv, int mode, uint32_t pos, int to_cache,
                        cudaStream_t st);
// Copy nbytes within each of B sequence slabs (slab i at base + i*seq_bytes) from src_off to
// dst_off; the ranges must not overlap.
int launch_qk_norm_rope(const float *x, uint32_t B, uint32_t S, uint32_t heads, uint32_t D, uint32_t x_stride,
                        uint32_t x_off, const float *gamma, const float *cosT, const float *sinT, uint32_t rot,
                        uint32_t pos0, float eps, float *y, const KVView &kv, int mode, int to_cache,
                        cudaStream_t st);
int launch_conv1d_causal(const float *x, const float *w, const float *state_in, int load_state, uint32_t S,
                         uint32_t C, uint32_t K, float *y, float *state_out, cudaStream_t st);
int launch_slice_cols(const float *src, uint32_t rows, uint32_t width, uint32_t stride, uint32_t off, float *dst,
                      cudaStream_t st);
int launch_copy_rows(void *base, uint64_t seq_bytes, uint32_t B, uint64_t dst_off, uint64_t src_off, uint64_t nbytes,
                     cudaStream_t st);

struct DeltaArgs {
  uint32_t S, H, HK, DK, DV, tOff, betaOff, loadState;
  const float *q, *k, *v;
  const float *g, *beta;                   // unfused: precomputed g / beta
  const float *a, *b, *a_neg, *dt_bias;    // fused gbeta inputs (g/beta null)
  const float *z, *gamma;                  // fused norm-gate (null: write core only)
  float eps;
  const float *state_in;                   // null or loadState==0: zero state
  float *state_out, *core, *y;
};

int launch_deltanet(const DeltaArgs &a, cudaStream_t st);
int poll_device_error_deltanet();
int poll_device_error_dnchunk();
size_t deltanet_chunk_workspace(uint32_t S, uint32_t H);
int launch_deltanet_chunked(const DeltaArgs &a, void *ws, size_t ws_bytes, cudaStream_t st);
int launch_gbeta(const float *a, const float *b, const float *a_neg, const float *dt, uint32_t S, uint32_t H,
                 float *out, cudaStream_t st);
int launch_norm_gate(const float *core, const float *z, const float *gamma, uint32_t rows, uint32_t DV, float eps,
                     float *y, cudaStream_t st);
int launch_gate_sigmoid(const float *x, const float *gate, uint32_t n, float *y, cudaStream_t st);

}  // namespace bg
