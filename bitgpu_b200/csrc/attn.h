// Internal launch interface shared by the attention kernels and the C-ABI layer.
#pragma once
#include "common.cuh"
#include "merge.cuh"

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
  // direct mode (nsplit == 1 only): write the normalised (optionally gated) output instead of
  // partials, so single-split calls need no workspace and no merge launch
  void *out;
  int out_f16;
  const float *gate;
  // peer-exchange step (tensor-core kernel, nsplit >= 2): the last CTA of each (sequence, kv head)
  // group merges its splits, pushes the rows to every rank, waits for theirs and writes the final
  // (gated) rows to fout -- px.nranks == 0: off
  PeerArgs px;
  void *fout;
};

// Number of KV splits for one attention call over L positions with the given cache mode and
// kernel (tensor-core or not); the workspace holds nsplit * B*S*H * (D+2) floats.
// attn_max_splits is the maximum over every mode/kernel (what workspace sizing reserves).
uint32_t attn_num_splits(uint32_t B, uint32_t S, uint32_t H, uint32_t KV, uint32_t D, uint32_t L, int mode, bool tc,
                         bool roll = false);
uint32_t attn_max_splits(uint32_t B, uint32_t S, uint32_t H, uint32_t KV, uint32_t D, uint32_t L);
bool attn_tc_supported(int mode, uint32_t D, uint32_t S, uint32_t H, uint32_t KV, bool roll, bool ring);
int attn_tc_ctas_per_sm(int mode, uint32_t D, uint32_t M, bool roll);
int attn_generic_ctas_per_sm(int mode, uint32_t D, uint32_t rows, bool roll);

int launch_attn_generic(const AttnArgs &a, cudaStream_t st);
int launch_attn_tc(const AttnArgs &a, cudaStream_t st);  // returns BG_EUNSUPPORTED if not covered
int launch_lse_merge(const float *partials, uint32_t nsplit, uint32_t rows, uint32_t D,
                     const float *gate, void *out, int out_f16, cudaStream_t st);

// Rope-at-read decode with all kv heads of a group per CTA (stream-K schedule); its split count
// is fixed by the schedule, and launch_attn_roll returns BG_EUNSUPPORTED when a.nsplit differs.
bool attn_roll_supported(int mode, uint32_t D, uint32_t S, uint32_t H, uint32_t KV);
uint32_t attn_roll_num_splits(int mode, uint32_t B, uint32_t KV, uint32_t L);
int launch_attn_roll(const AttnArgs &a, cudaStream_t st);
bool roll_legacy();  // BGATTN_ROLL_LEGACY=1 selects the one-head-per-CTA kernel

// Read-and-clear the bounded-wait timeout flag of the TMA kernels (BG_ETIMEOUT or 0).
int poll_device_error_attn_tc();
// Split-KV partial scratch a bg_attention call may need (the part every kernel path shares).
size_t attention_split_workspace_bytes(const bg_attn_params *p, uint32_t batch);
// Peer-memory split-KV step after the decode kernel: merge this rank's splits of each row, push it
// to every rank, wait for theirs, merge, gate and write (splitkv_peer.cu).
int launch_lse_exchange(const float *partials, uint32_t nsplit, uint32_t rows, uint32_t D, const bg_peer_exchange *x,
                        const float *gate, void *out, int out_f16, cudaStream_t st);
int poll_device_error_peer();
PeerArgs peer_args(const bg_peer_exchange *x, uint32_t rows);
int poll_device_error_attn_roll();

}  // namespace bg
