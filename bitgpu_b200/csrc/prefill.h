// Internal launch interface of the tcgen05 causal prefill kernel.
#pragma once
#include "common.cuh"

namespace bg {

struct PrefillArgs {
  const void *q;          // [B][S][H][D] f32 (q_f32) or f16
  int q_f32;
  int mode;               // BG_KV_F16, BG_KV_Q8 or BG_KV_F32 (head_dim 128)
  uint32_t D;             // 128 or 256
  const void *K, *V;      // cache [B][seq_stride][KV][D]: f16 values or int8 codes
  const float *Ks, *Vs;   // q8 block scales [B][seq_stride][KV][D/32]
  uint64_t seq_stride;
  const float *gate;      // [B][S][H][D] sigmoid gate or nullptr
  void *out;              // [B][S][H][D] f16 or f32
  int out_f16;
  uint32_t B, S, H, KV, posBase, Ltot;
  float scale;
  void *ws;               // caller workspace (q8: room for an f16 copy of the cache lets the
  size_t ws_bytes;        //   kernel dequantise once up front instead of inside every CTA)
};

// Workspace bytes for the dequantised f16 copy of a q8 cache's positions [0, Ltot).
inline size_t prefill_q8_copy_bytes(uint32_t B, uint32_t Ltot, uint32_t KV, uint32_t D) {
  return (size_t)2 * B * Ltot * KV * D * 2;
}

bool prefill_tc_supported(int mode, uint32_t D, uint32_t S, bool roll, bool ring);
int launch_prefill_tc(const PrefillArgs &a, cudaStream_t st);
int launch_prefill_tf32(const PrefillArgs &a, cudaStream_t st);  // f32 cache, 3xTF32
int poll_device_error_prefill_tf32();
int poll_device_error_prefill();
int poll_device_error_selftest();

}  // namespace bg
