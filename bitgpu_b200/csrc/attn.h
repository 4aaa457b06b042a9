// Internal launch interface shared by the attention kernels and the C-ABI layer.
#pragma once
#include "common.cuh"

namespace bg {

struct AttnArgs {
  const void *q;
  int q_f16;
  KVView kv;
  int mode;  // BG_KV_*
  const float *cosT, *sinT;  // rope-at-read tables [positions][D/2] or null
  float scale;               // softmax scale (natural units)
  uint32_t B, S, H, KV, D, posBase;
  uint32_t pos_lo, pos_hi;   // attended logical positions are clipped to [pos_lo, pos_hi)
  float *partials;           // [nsplit][B*S*H][D+2]: o[D], m (natural log units), l
  uint32_t nsplit, chunk;    // split j covers [pos_lo + j*chunk, pos_lo + (j+1)*chunk)
};

// Number of KV splits used for a full attention call; the workspace holds
// nsplit * B*S*H * (D+2) floats.
uint32_t attn_num_splits(uint32_t B, uint32_t S, uint32_t H, uint32_t KV, uint32_t D, uint32_t L);

int launch_attn_generic(const AttnArgs &a, cudaStream_t st);
int launch_attn_tc(const AttnArgs &a, cudaStream_t st);  // returns BG_EUNSUPPORTED if not covered
int launch_lse_merge(const float *partials, uint32_t nsplit, uint32_t rows, uint32_t D,
                     const float *gate, void *out, int out_f16, cudaStream_t st);

}  // namespace bg
