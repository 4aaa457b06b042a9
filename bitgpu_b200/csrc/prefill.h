// Internal launch interface of the tcgen05 causal prefill kernel.
#pragma once
#include "common.cuh"

namespace bg {

struct PrefillArgs {
  const void *q;          // [B][S][H][128] f16
  const void *K, *V;      // f16 cache [B][seq_stride][KV][128]
  uint64_t seq_stride;
  void *out;              // [B][S][H][128] f16 or f32
  int out_f16;
  uint32_t B, S, H, KV, posBase, Ltot;
  float scale;
};

bool prefill_tc_supported(int mode, uint32_t D, uint32_t S, int q_f16, bool roll, bool ring);
int launch_prefill_tc(const PrefillArgs &a, cudaStream_t st);
int poll_device_error_prefill();
int poll_device_error_selftest();

}  // namespace bg
