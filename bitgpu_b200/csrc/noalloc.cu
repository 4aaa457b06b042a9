// bg_attention_noalloc: the decode / prefill attention of bg_attention for callers that cannot
// allocate device memory.
//
// bg_attention needs a caller-provided scratch buffer for its split-KV partial results.  Some
// hosts cannot produce one: an engine whose device memory is entirely owned by another allocator
// (a WebGPU-style host that hands the library only the buffers it already created, with no
// allocator exposed across the binding), or a caller on a latency-critical token loop that must
// not call cudaMalloc, which can synchronise the device.  For them this entry point keeps its
// scratch in a fixed array compiled into the library (kNoAllocScratchBytes per GPU, resident on
// every GPU that loads the library until the process exits) and allocates nothing at all.
#include "attn.h"

namespace {

constexpr size_t kNoAllocScratchBytes = BG_NOALLOC_SCRATCH_BYTES;  // 8 MiB per device

// The scratch itself.  In host code this name is only a host-side stand-in for the symbol:
// kernels must be given the device address from cudaGetSymbolAddress, never &g_noalloc_scratch.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch in the current context, looked up on every call (a cheap host-side
// table lookup).  Not caching it keeps the address right after cudaDeviceReset, which recreates
// the context and may place the module's symbols elsewhere.  Returns nullptr on failure.
void *scratch_for_current_device() {
  void *p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
  return p;
}

}  // namespace

extern "C" {

size_t bg_attention_noalloc_limit(void) { return kNoAllocScratchBytes; }

int bg_attention_noalloc(const bg_attn_params *p, uint32_t batch, const void *q, uint32_t q_dtype,
                         const bg_kv_cache *kv, const float *cosT, const float *sinT, float scale, const float *gate,
                         void *out, uint32_t out_dtype, bg_stream_t stream) {
  if (!p) return BG_EINVAL;
  // Shapes whose split partials do not fit the fixed scratch are rejected up front (BG_ENOMEM).  A
  // q8 prefill too large to dequantise into the scratch dequantises inside its kernel instead.
  if (bg::attention_split_workspace_bytes(p, batch) > kNoAllocScratchBytes) return BG_ENOMEM;
  void *ws = scratch_for_current_device();
  if (!ws) return BG_ELAUNCH;
  // Every partial row the merge reads is written earlier in the same call, so the scratch needs
  // no clearing between calls.
  return bg_attention(p, batch, q, q_dtype, kv, cosT, sinT, scale, gate, out, out_dtype, ws, kNoAllocScratchBytes,
                      stream);
}

}  // extern "C"
