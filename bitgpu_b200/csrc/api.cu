// extern "C" entry points of libbgattn.so: argument validation (mirroring the engine's
// validation throws) and dispatch to the sm_100a kernels.  See include/bgattn.h.
#include <math.h>
#include <stdlib.h>

#include "attn.h"
#include "kv.h"
#include "prefill.h"

using namespace bg;

namespace {

int g_force_generic = 0;  // bg_force_generic (the reference's forceNoSubgroups analogue)

bool kv_mode_ok(uint32_t m) { return m <= BG_KV_Q8R; }

bool d_ok(uint32_t D) { return D == 64 || D == 128 || D == 256; }

// engine.ts:232-235 (head_dim limits, H % KV), :372-373 (q8 needs D % 32).
int check_attn(const bg_attn_params *p, const bg_kv_cache *kv) {
  if (!p || !kv) return BG_EINVAL;
  if (p->H == 0 || p->KV == 0 || p->H % p->KV) return BG_EINVAL;
  if (!d_ok(p->D)) return BG_EUNSUPPORTED;
  if (!kv_mode_ok(kv->mode)) return BG_EINVAL;
  if (kv->mode == BG_KV_Q8R && p->D % 128) return BG_EINVAL;
  if ((kv->mode == BG_KV_Q8 || kv->mode == BG_KV_Q8R) && (!kv->Ks || !kv->Vs)) return BG_EINVAL;
  if (!kv->K || !kv->V) return BG_EINVAL;
  if (p->Ltot != p->posBase + p->S) return BG_EINVAL;
  if (kv->window) {
    if ((uint64_t)kv->sinks + kv->window > kv->seq_stride) return BG_EINVAL;
    if (p->Ltot > kv->sinks + kv->window) return BG_EINVAL;
  } else if (p->Ltot > kv->seq_stride) {
    return BG_EINVAL;
  }
  return BG_OK;
}

KVView make_view(const bg_kv_cache *kv, uint32_t KV, uint32_t row_offset) {
  KVView v;
  v.K = kv->K;
  v.V = kv->V;
  v.Ks = kv->Ks;
  v.Vs = kv->Vs;
  v.seq_stride = kv->seq_stride;
  v.sinks = kv->sinks;
  v.window = kv->window;
  v.ring_head = kv->window ? kv->ring_head % kv->window : 0;
  v.KV = KV;
  v.row_offset = row_offset;
  return v;
}

// BGATTN_PEER_FUSED=1 runs a peer-exchange step as one tensor-core kernel (the last CTA of each
// group merges, pushes, waits and writes); default: the split kernel, a push kernel and a merge kernel
bool peer_fused_enabled() {
  static const bool v = [] {
    const char *e = getenv("BGATTN_PEER_FUSED");
    return e && e[0] == '1';
  }();
  return v;
}

// BGATTN_NSPLIT: split-count override for tuning sweeps (0 / unset = the cost model's choice).
// bg_attention_workspace_size reserves for it, so an overridden call never under-allocates.
uint32_t env_nsplit() {
  const char *ov = getenv("BGATTN_NSPLIT");
  const int n = ov ? atoi(ov) : 0;
  return n > 0 ? (n < 512 ? (uint32_t)n : 512u) : 0u;
}

size_t part_bytes(uint32_t nsplit, uint64_t rows, uint32_t D) { return (size_t)nsplit * rows * (D + 2) * sizeof(float); }

int run_attention(const bg_attn_params *p, uint32_t batch, const void *q, uint32_t q_dtype, const bg_kv_cache *kv,
                  const float *cosT, const float *sinT, float scale, uint32_t pos_lo, uint32_t pos_hi,
                  uint32_t row_offset, float *partials_out, const float *gate, void *out, uint32_t out_dtype,
                  void *ws, size_t ws_bytes, cudaStream_t st, const bg_peer_exchange *peer = nullptr) {
  const float sc = scale > 0.f ? scale : 1.0f / sqrtf((float)p->D);
  // dense prefill on the tensor cores (f16 / f32 queries over an f16 or q8 cache, or an f32 cache
  // in 3xTF32; whole causal range, optional sigmoid gate)
  if (!partials_out && !peer && !g_force_generic &&
      prefill_tc_supported((int)kv->mode, p->D, p->S, cosT != nullptr, kv->window != 0)) {
    PrefillArgs pa;
    pa.q = q;
    pa.q_f32 = q_dtype == BG_DT_F32;
    pa.mode = (int)kv->mode;
    pa.D = p->D;
    pa.K = kv->K;
    pa.V = kv->V;
    pa.Ks = kv->Ks;
    pa.Vs = kv->Vs;
    pa.seq_stride = kv->seq_stride;
    pa.gate = gate;
    pa.out = out;
    pa.out_f16 = out_dtype == BG_DT_F16;
    pa.B = batch;
    pa.S = p->S;
    pa.H = p->H;
    pa.KV = p->KV;
    pa.posBase = p->posBase;
    pa.Ltot = p->Ltot;
    pa.scale = sc;
    pa.ws = ws;
    pa.ws_bytes = ws_bytes;
    return launch_prefill_tc(pa, st);
  }
  AttnArgs a;
  a.px.nranks = 0;
  a.fout = nullptr;
  a.q = q;
  a.q_f16 = q_dtype == BG_DT_F16;
  a.kv = make_view(kv, p->KV, row_offset);
  a.mode = (int)kv->mode;
  a.cosT = cosT;
  a.sinT = sinT;
  a.scale = sc;
  a.B = batch;
  a.S = p->S;
  a.H = p->H;
  a.KV = p->KV;
  a.D = p->D;
  a.posBase = p->posBase;
  a.pos_lo = pos_lo;
  a.pos_hi = pos_hi;
  a.out = nullptr;
  a.out_f16 = 0;
  a.gate = nullptr;
  const uint64_t rows = (uint64_t)batch * p->S * p->H;
  const uint32_t L = pos_hi > pos_lo ? pos_hi - pos_lo : 1;
  const bool tc = !g_force_generic && attn_tc_supported(a.mode, p->D, p->S, p->H, p->KV, cosT != nullptr,
                                                        kv->window != 0);
  a.nsplit = attn_num_splits(batch, p->S, p->H, p->KV, p->D, L, a.mode, tc, cosT != nullptr);
  if (const uint32_t ov = env_nsplit()) a.nsplit = ov;
  if (peer && a.nsplit < 2) a.nsplit = 2;  // the push kernel merges at least two local splits
  a.chunk = ((L + a.nsplit - 1) / a.nsplit + 63) / 64 * 64;  // whole 64-position tiles
  if (a.nsplit == 1) {
    // one split: the kernel writes the final rows (or the caller's partial rows) itself
    if (partials_out) {
      a.partials = partials_out;
    } else {
      a.partials = nullptr;
      a.out = out;
      a.out_f16 = out_dtype == BG_DT_F16;
      a.gate = gate;
    }
  } else {
    if (ws_bytes < part_bytes(a.nsplit, rows, p->D) || (!ws && rows)) return BG_ENOMEM;
    a.partials = static_cast<float *>(ws);
  }
  if (peer && tc && !cosT && peer_fused_enabled()) {
    a.px = peer_args(peer, (uint32_t)rows);
    a.fout = out;
    a.out_f16 = out_dtype == BG_DT_F16;
    a.gate = gate;
  }
  int rc = tc ? launch_attn_tc(a, st) : BG_EUNSUPPORTED;
  if (rc == BG_EUNSUPPORTED) a.px.nranks = 0;  // the CUDA-core kernel has no fused epilogue
  if (rc == BG_EUNSUPPORTED) rc = launch_attn_generic(a, st);
  if (rc || a.nsplit == 1) return rc;
  if (peer) {
    // the tensor-core kernel took the whole step (fused epilogue); the CUDA-core one left split
    // partials: push them, then the merge kernel waits for the other ranks and writes out
    if (a.px.nranks) return BG_OK;
    return launch_lse_exchange(a.partials, a.nsplit, (uint32_t)rows, p->D, peer, gate, out, out_dtype == BG_DT_F16, st);
  }
  if (partials_out) return launch_lse_merge(a.partials, a.nsplit, (uint32_t)rows, p->D, nullptr, partials_out, -1, st);
  return launch_lse_merge(a.partials, a.nsplit, (uint32_t)rows, p->D, gate, out, out_dtype == BG_DT_F16, st);
}

// Snapshot regions of one layer, in the reference order (engine.ts:2768-2776): K, V, then the q8
// block scales of K and V.  Bytes of one cache position of each region, or 0 if absent.
void snapshot_row_bytes(const bg_kv_cache *kv, uint32_t KV, uint32_t D, uint64_t rb[4]) {
  const uint64_t es = kv->mode == BG_KV_F32 ? 4 : kv->mode == BG_KV_F16 ? 2 : 1;
  rb[0] = rb[1] = (uint64_t)KV * D * es;
  const uint64_t blk = kv->mode == BG_KV_Q8 ? 32 : kv->mode == BG_KV_Q8R ? 128 : 0;
  rb[2] = rb[3] = blk ? (uint64_t)KV * (D / blk) * 4 : 0;
}

// Copy logical positions [base, base+count) of sequence `seq` between the cache and a packed
// snapshot region buffer (to_cache: restore).  A logical range is at most three physical runs of
// the ring (sinks, head..end of window, wrap), each one contiguous copy per region.
int snapshot_copy(const bg_kv_cache *kv, uint32_t seq, uint32_t KV, uint32_t D, uint32_t base, uint32_t count,
                  unsigned char *buf, bool to_cache, cudaStream_t st) {
  if (!kv || (!buf && count) || !kv_mode_ok(kv->mode) || KV == 0) return BG_EINVAL;
  if (!d_ok(D)) return BG_EUNSUPPORTED;
  if (kv->mode == BG_KV_Q8R && D % 128) return BG_EINVAL;
  const uint64_t cap = kv->window ? (uint64_t)kv->sinks + kv->window : kv->seq_stride;
  if ((uint64_t)base + count > cap) return BG_EINVAL;
  void *reg[4] = {kv->K, kv->V, const_cast<float *>(kv->Ks), const_cast<float *>(kv->Vs)};
  uint64_t rb[4];
  snapshot_row_bytes(kv, KV, D, rb);
  for (int r = 0; r < 4; ++r)
    if (rb[r] && !reg[r]) return BG_EINVAL;
  const uint32_t head = kv->window ? kv->ring_head % kv->window : 0;
  uint64_t boff = 0;
  for (int r = 0; r < 4; ++r) {
    if (!rb[r]) continue;
    unsigned char *slab = static_cast<unsigned char *>(reg[r]) + (uint64_t)seq * kv->seq_stride * rb[r];
    for (uint32_t p = base; p < base + count;) {
      uint32_t ph = p, run = base + count - p;
      if (kv->window) {
        if (p < kv->sinks) {
          run = min(run, kv->sinks - p);
        } else {
          uint32_t rel = head + (p - kv->sinks);
          if (rel >= kv->window) rel -= kv->window;
          ph = kv->sinks + rel;
          run = min(run, kv->window - rel);
        }
      }
      unsigned char *dev = slab + (uint64_t)ph * rb[r];
      unsigned char *pk = buf + boff + (uint64_t)(p - base) * rb[r];
      const uint64_t n = (uint64_t)run * rb[r];
      if (cudaMemcpyAsync(to_cache ? dev : pk, to_cache ? pk : dev, n, cudaMemcpyDefault, st) != cudaSuccess)
        return BG_ELAUNCH;
      p += run;
    }
    boff += (uint64_t)count * rb[r];
  }
  return BG_OK;
}

}  // namespace

namespace bg {
size_t attention_split_workspace_bytes(const bg_attn_params *p, uint32_t batch) {
  if (!p || !p->KV || !p->H) return 0;
  const uint32_t L = p->Ltot ? p->Ltot : 1;
  uint32_t ns = attn_max_splits(batch, p->S, p->H, p->KV, p->D, L);
  if (env_nsplit() > ns) ns = env_nsplit();
  return ns > 1 ? part_bytes(ns, (uint64_t)batch * p->S * p->H, p->D) : 0;  // one split needs no scratch
}
}  // namespace bg

extern "C" {

size_t bg_kv_snapshot_bytes(const bg_kv_cache *kv, uint32_t KV, uint32_t D, uint32_t count) {
  if (!kv || !kv_mode_ok(kv->mode)) return 0;
  uint64_t rb[4];
  snapshot_row_bytes(kv, KV, D, rb);
  return (size_t)count * (rb[0] + rb[1] + rb[2] + rb[3]);
}

int bg_kv_snapshot_save(const bg_kv_cache *kv, uint32_t seq, uint32_t KV, uint32_t D, uint32_t base, uint32_t count,
                        void *dst, bg_stream_t stream) {
  return snapshot_copy(kv, seq, KV, D, base, count, static_cast<unsigned char *>(dst), false, (cudaStream_t)stream);
}

int bg_kv_snapshot_restore(const bg_kv_cache *kv, uint32_t seq, uint32_t KV, uint32_t D, uint32_t base,
                           uint32_t count, const void *src, bg_stream_t stream) {
  return snapshot_copy(kv, seq, KV, D, base, count, static_cast<unsigned char *>(const_cast<void *>(src)), true,
                       (cudaStream_t)stream);
}

const char *bg_strerror(int code) {
  switch (code) {
    case BG_OK: return "ok";
    case BG_EINVAL: return "invalid argument";
    case BG_ENOMEM: return "workspace too small";
    case BG_ELAUNCH: return "CUDA launch failed";
    case BG_ETIMEOUT: return "device wait timed out";
    case BG_EUNSUPPORTED: return "unsupported shape or mode";
    default: return "unknown error";
  }
}

int bg_version(void) { return 1; }


int bg_force_generic(int on) {
  const int prev = g_force_generic;
  g_force_generic = on ? 1 : 0;
  return prev;
}

int bg_device_status(bg_stream_t stream) {
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return BG_ELAUNCH;
  int e = poll_device_error_attn_tc();
  if (!e) e = poll_device_error_attn_roll();
  if (!e) e = poll_device_error_prefill();
  if (!e) e = poll_device_error_selftest();
  if (!e) e = poll_device_error_prefill_tf32();
  if (!e) e = poll_device_error_deltanet();
  if (!e) e = poll_device_error_dnchunk();
  if (!e) e = poll_device_error_peer();
  return e ? (e < 0 ? e : BG_ELAUNCH) : BG_OK;
}

size_t bg_attention_workspace_size(const bg_attn_params *p, uint32_t batch) {
  if (!p || !p->KV || !p->H) return 0;
  size_t split = attention_split_workspace_bytes(p, batch);
  // a tensor-core prefill over a q8 cache dequantises it once into this workspace when it fits
  if (prefill_tc_supported(BG_KV_Q8, p->D, p->S, false, false)) {
    const size_t cp = prefill_q8_copy_bytes(batch, p->Ltot, p->KV, p->D);
    if (cp > split) split = cp;
  }
  return split;
}

int bg_attention(const bg_attn_params *p, uint32_t batch, const void *q, uint32_t q_dtype, const bg_kv_cache *kv,
                 const float *cosT, const float *sinT, float scale, const float *gate, void *out, uint32_t out_dtype,
                 void *workspace, size_t workspace_bytes, bg_stream_t stream) {
  int rc = check_attn(p, kv);
  if (rc) return rc;
  if (!q || !out || q_dtype > BG_DT_F16 || out_dtype > BG_DT_F16) return BG_EINVAL;
  if ((cosT == nullptr) != (sinT == nullptr)) return BG_EINVAL;
  if (batch == 0 || p->S == 0) return BG_OK;
  return run_attention(p, batch, q, q_dtype, kv, cosT, sinT, scale, 0, p->Ltot, 0, nullptr, gate, out, out_dtype,
                       workspace, workspace_bytes, (cudaStream_t)stream);
}

int bg_attention_partials(const bg_attn_params *p, uint32_t batch, const void *q, uint32_t q_dtype,
                          const bg_kv_cache *kv, const float *cosT, const float *sinT, float scale, uint32_t pos_lo,
                          uint32_t pos_hi, float *partials, void *workspace, size_t workspace_bytes,
                          bg_stream_t stream) {
  if (!p || !kv || !q || !partials) return BG_EINVAL;
  if (p->H == 0 || p->KV == 0 || p->H % p->KV || !kv_mode_ok(kv->mode)) return BG_EINVAL;
  if (!d_ok(p->D)) return BG_EUNSUPPORTED;
  if (p->Ltot != p->posBase + p->S || pos_lo > pos_hi || pos_hi > p->Ltot) return BG_EINVAL;
  if (kv->window) return BG_EUNSUPPORTED;
  if (pos_hi - pos_lo > kv->seq_stride) return BG_EINVAL;
  if ((cosT == nullptr) != (sinT == nullptr)) return BG_EINVAL;
  if (batch == 0 || p->S == 0) return BG_OK;
  if (pos_hi == pos_lo) {  // nothing attended here: an empty partial (l = 0)
    const uint64_t n = (uint64_t)batch * p->S * p->H * (p->D + 2);
    return cudaMemsetAsync(partials, 0, n * sizeof(float), (cudaStream_t)stream) == cudaSuccess ? BG_OK : BG_ELAUNCH;
  }
  return run_attention(p, batch, q, q_dtype, kv, cosT, sinT, scale, pos_lo, pos_hi, pos_lo, partials, nullptr,
                       nullptr, 0, workspace, workspace_bytes, (cudaStream_t)stream);
}

int bg_lse_merge(const float *partials, uint32_t nsplit, uint32_t rows, uint32_t D, const float *gate, void *out,
                 uint32_t out_dtype, bg_stream_t stream) {
  if (!partials || !out || nsplit == 0 || D == 0 || out_dtype > BG_DT_F16) return BG_EINVAL;
  return launch_lse_merge(partials, nsplit, rows, D, gate, out, out_dtype == BG_DT_F16, (cudaStream_t)stream);
}

static int check_peer(const bg_peer_exchange *x) {
  if (!x || x->nranks == 0 || x->nranks > BG_MAX_PEERS || x->rank >= x->nranks || !x->step || !x->done)
    return BG_EINVAL;
  for (uint32_t r = 0; r < x->nranks; ++r)
    if (!x->gather[r] || !x->flags[r]) return BG_EINVAL;
  return BG_OK;
}

size_t bg_peer_exchange_flags_offset(uint32_t nranks, uint32_t rows, uint32_t D) {
  const size_t g = (size_t)2 * nranks * rows * (D + 2) * sizeof(float);
  return (g + 255) / 256 * 256;
}

size_t bg_peer_exchange_bytes(uint32_t nranks, uint32_t rows, uint32_t D) {
  return bg_peer_exchange_flags_offset(nranks, rows, D) + ((size_t)nranks * rows * sizeof(uint32_t) + 255) / 256 * 256;
}

size_t bg_attention_peer_workspace_size(const bg_attn_params *p, uint32_t batch) {
  if (!p || !p->KV || !p->H) return 0;
  const size_t two = part_bytes(2, (uint64_t)batch * p->S * p->H, p->D);
  const size_t ws = attention_split_workspace_bytes(p, batch);
  return ws > two ? ws : two;
}

int bg_attention_peer(const bg_attn_params *p, uint32_t batch, const void *q, uint32_t q_dtype, const bg_kv_cache *kv,
                      float scale, uint32_t pos_lo, uint32_t pos_hi, const bg_peer_exchange *x, const float *gate,
                      void *out, uint32_t out_dtype, void *workspace, size_t workspace_bytes, bg_stream_t stream) {
  if (int rc = check_peer(x)) return rc;
  if (!p || !kv || !q || !out || q_dtype > BG_DT_F16 || out_dtype > BG_DT_F16) return BG_EINVAL;
  if (p->H == 0 || p->KV == 0 || p->H % p->KV || !kv_mode_ok(kv->mode)) return BG_EINVAL;
  if (!d_ok(p->D)) return BG_EUNSUPPORTED;
  if (p->Ltot != p->posBase + p->S || pos_lo > pos_hi || pos_hi > p->Ltot) return BG_EINVAL;
  if (kv->window) return BG_EUNSUPPORTED;
  if (pos_hi - pos_lo > kv->seq_stride) return BG_EINVAL;
  if (!x->tickets) return BG_EINVAL;
  if (batch == 0 || p->S == 0) return BG_OK;
  const uint32_t rows = batch * p->S * p->H;
  cudaStream_t st = (cudaStream_t)stream;
  if (pos_hi == pos_lo) {  // this slice attends nothing: push empty rows, then merge the others'
    return launch_lse_exchange(nullptr, 0, rows, p->D, x, gate, out, out_dtype == BG_DT_F16, st);
  }
  return run_attention(p, batch, q, q_dtype, kv, nullptr, nullptr, scale, pos_lo, pos_hi, pos_lo, nullptr, gate, out,
                       out_dtype, workspace, workspace_bytes, st, x);
}

int bg_kv_append(const bg_kv_cache *kv, uint32_t which, uint32_t batch, const void *src, uint32_t src_dtype,
                 uint32_t S, uint32_t KV, uint32_t D, uint32_t pos0, bg_stream_t stream) {
  if (!kv || !src || which > 1 || src_dtype > BG_DT_F16 || !kv_mode_ok(kv->mode) || KV == 0) return BG_EINVAL;
  if (!d_ok(D)) return BG_EUNSUPPORTED;
  if (kv->mode == BG_KV_Q8R && D % 128) return BG_EINVAL;
  if ((which ? kv->V : kv->K) == nullptr) return BG_EINVAL;
  if ((kv->mode == BG_KV_Q8 || kv->mode == BG_KV_Q8R) && (which ? kv->Vs : kv->Ks) == nullptr) return BG_EINVAL;
  const uint64_t cap = kv->window ? (uint64_t)kv->sinks + kv->window : kv->seq_stride;
  if ((uint64_t)pos0 + S > cap) return BG_EINVAL;  // the engine's ensureKvCapacity / evictFor precondition
  if (batch == 0 || S == 0) return BG_OK;
  return launch_kv_append(make_view(kv, KV, 0), (int)kv->mode, D, src, nullptr, src_dtype == BG_DT_F16, batch, S,
                          pos0, (int)which, 1, (cudaStream_t)stream);
}

// Validation shared by the K+V writers: the cache holds positions [pos0, pos0 + S) of this shape.
static int check_append_kv(const bg_kv_cache *kv, uint32_t S, uint32_t D, uint32_t pos0) {
  if (!kv || !kv_mode_ok(kv->mode)) return BG_EINVAL;
  if (kv->mode == BG_KV_Q8R && D % 128) return BG_EINVAL;
  if (!kv->K || !kv->V) return BG_EINVAL;
  if ((kv->mode == BG_KV_Q8 || kv->mode == BG_KV_Q8R) && (!kv->Ks || !kv->Vs)) return BG_EINVAL;
  const uint64_t cap = kv->window ? (uint64_t)kv->sinks + kv->window : kv->seq_stride;
  if ((uint64_t)pos0 + S > cap) return BG_EINVAL;
  return BG_OK;
}

int bg_kv_append_kv(const bg_kv_cache *kv, uint32_t batch, const void *k_src, const void *v_src, uint32_t src_dtype,
                    uint32_t S, uint32_t KV, uint32_t D, uint32_t pos0, bg_stream_t stream) {
  if (!kv || !k_src || !v_src || src_dtype > BG_DT_F16 || KV == 0) return BG_EINVAL;
  if (!d_ok(D)) return BG_EUNSUPPORTED;
  if (int rc = check_append_kv(kv, S, D, pos0)) return rc;
  if (batch == 0 || S == 0) return BG_OK;
  return launch_kv_append(make_view(kv, KV, 0), (int)kv->mode, D, k_src, v_src, src_dtype == BG_DT_F16, batch, S,
                          pos0, 0, 2, (cudaStream_t)stream);
}

int bg_kv_append_kv_pair(const bg_kv_cache *kv0, const bg_kv_cache *kv1, uint32_t batch, const void *k_src,
                         const void *v_src, uint32_t src_dtype, uint32_t S, uint32_t KV, uint32_t D, uint32_t pos0,
                         bg_stream_t stream) {
  if (!kv0 || !kv1 || !k_src || !v_src || src_dtype > BG_DT_F16 || KV == 0) return BG_EINVAL;
  if (!d_ok(D)) return BG_EUNSUPPORTED;
  if (int rc = check_append_kv(kv0, S, D, pos0)) return rc;
  if (int rc = check_append_kv(kv1, S, D, pos0)) return rc;
  if (batch == 0 || S == 0) return BG_OK;
  const KVView v1 = make_view(kv1, KV, 0);
  return launch_kv_append(make_view(kv0, KV, 0), (int)kv0->mode, D, k_src, v_src, src_dtype == BG_DT_F16, batch, S,
                          pos0, 0, 2, (cudaStream_t)stream, &v1, (int)kv1->mode);
}

int bg_qk_norm_rope(const float *x, uint32_t batch, uint32_t S, uint32_t heads, uint32_t D, uint32_t x_stride,
                    uint32_t x_off, const float *gamma, const float *cosT, const float *sinT, uint32_t rot,
                    uint32_t pos0, float eps, float *y, const bg_kv_cache *kv, bg_stream_t stream) {
  if (!x || !gamma || (!y && !kv) || rot > D || rot % 2 || (rot && (!cosT || !sinT))) return BG_EINVAL;
  if (!d_ok(D)) return BG_EUNSUPPORTED;
  if (x_stride < D || (uint64_t)x_off + D > x_stride || heads == 0) return BG_EINVAL;
  KVView v = {};
  int mode = 0;
  if (kv) {
    if (!kv_mode_ok(kv->mode) || !kv->K) return BG_EINVAL;
    if ((kv->mode == BG_KV_Q8 || kv->mode == BG_KV_Q8R) && !kv->Ks) return BG_EINVAL;
    if (kv->mode == BG_KV_Q8R && D % 128) return BG_EINVAL;
    const uint64_t cap = kv->window ? (uint64_t)kv->sinks + kv->window : kv->seq_stride;
    if ((uint64_t)pos0 + S > cap) return BG_EINVAL;
    v = make_view(kv, heads, 0);
    mode = (int)kv->mode;
  }
  if (batch == 0 || S == 0) return BG_OK;
  return launch_qk_norm_rope(x, batch, S, heads, D, x_stride, x_off, gamma, cosT, sinT, rot, pos0, eps, y, v, mode,
                             kv != nullptr, (cudaStream_t)stream);
}

int bg_conv1d_causal(const float *x, const float *w, const float *state_in, uint32_t load_state, uint32_t S,
                     uint32_t C, uint32_t K, float *y, float *state_out, bg_stream_t stream) {
  if ((!x && S) || !w || (!y && S) || !state_out || C == 0 || K < 2) return BG_EINVAL;
  if (load_state && (!state_in || state_in == state_out)) return BG_EINVAL;  // the engine ping-pongs them
  if (K > 8) return BG_EUNSUPPORTED;
  return launch_conv1d_causal(x, w, state_in, load_state != 0, S, C, K, y, state_out, (cudaStream_t)stream);
}

int bg_slice_cols(const float *src, uint32_t rows, uint32_t width, uint32_t stride, uint32_t off, float *dst,
                  bg_stream_t stream) {
  if (!src || !dst || (uint64_t)off + width > stride) return BG_EINVAL;
  return launch_slice_cols(src, rows, width, stride, off, dst, (cudaStream_t)stream);
}

int bg_rmsnorm_rope(const float *x, uint32_t batch, uint32_t R, uint32_t D, const float *gamma, const float *cos,
                    const float *sin, float eps, float *y, const bg_kv_cache *kv, uint32_t pos, bg_stream_t stream) {
  if (!x || !gamma || (!y && !kv) || ((cos == nullptr) != (sin == nullptr))) return BG_EINVAL;
  if (!d_ok(D)) return BG_EUNSUPPORTED;
  KVView v = {};
  int mode = 0;
  if (kv) {
    if (!kv_mode_ok(kv->mode) || !kv->K) return BG_EINVAL;
    if ((kv->mode == BG_KV_Q8 || kv->mode == BG_KV_Q8R) && !kv->Ks) return BG_EINVAL;
    if (kv->mode == BG_KV_Q8R && D % 128) return BG_EINVAL;
    const uint64_t cap = kv->window ? (uint64_t)kv->sinks + kv->window : kv->seq_stride;
    if (pos >= cap) return BG_EINVAL;
    v = make_view(kv, R, 0);
    mode = (int)kv->mode;
  }
  if (batch == 0 || R == 0) return BG_OK;
  return launch_rmsnorm_rope(x, batch, R, D, gamma, cos, sin, eps, y, v, mode, pos, kv != nullptr,
                             (cudaStream_t)stream);
}

int bg_kv_evict(const bg_kv_cache *kv, uint32_t batch, uint32_t KV, uint32_t D, uint32_t fill, uint32_t need,
                uint32_t max_seq_len, uint32_t *new_fill, bg_stream_t stream) {
  if (!kv || !new_fill || !kv_mode_ok(kv->mode) || kv->window || KV == 0) return BG_EINVAL;
  if (fill < kv->sinks || fill > kv->seq_stride || max_seq_len < kv->sinks) return BG_EINVAL;
  const uint32_t S0 = kv->sinks;
  const uint32_t recent = fill - S0;
  const uint32_t quarter = (max_seq_len - S0 + 3) / 4;  // ceil((maxSeqLen - SINKS) / 4)
  uint32_t batchn = need > quarter ? need : quarter;
  if (batchn > recent) batchn = recent;
  const int64_t keep = (int64_t)recent - batchn;
  if (keep <= 0) {
    *new_fill = S0;
    return BG_OK;
  }
  const uint64_t esz = kv->mode == BG_KV_F32 ? 4 : kv->mode == BG_KV_F16 ? 2 : 1;
  const uint64_t row_bytes = (uint64_t)KV * D * esz;
  const uint64_t srow_bytes =
      kv->mode == BG_KV_Q8 ? (uint64_t)KV * (D / 32) * 4 : kv->mode == BG_KV_Q8R ? (uint64_t)KV * (D / 128) * 4 : 0;
  struct Arr {
    void *p;
    uint64_t rb;
  } arrs[4] = {{kv->K, row_bytes}, {kv->V, row_bytes}, {kv->Ks, srow_bytes}, {kv->Vs, srow_bytes}};
  // Move [S0+batch, fill) down to S0 in ascending chunks of `batch` rows: within a chunk the
  // source and destination ranges are disjoint, and a chunk's source is only overwritten by a
  // later chunk (stream order), which is what the reference's scratch bounce guarantees.
  for (int ai = 0; ai < 4; ++ai) {
    if (!arrs[ai].p || !arrs[ai].rb) continue;
    const uint64_t rb = arrs[ai].rb;
    for (uint64_t c = 0; c < (uint64_t)keep; c += batchn) {
      const uint64_t n = ((uint64_t)keep - c) < batchn ? ((uint64_t)keep - c) : batchn;
      int rc = launch_copy_rows(arrs[ai].p, kv->seq_stride * rb, batch, (S0 + c) * rb, (S0 + batchn + c) * rb, n * rb,
                                (cudaStream_t)stream);
      if (rc) return rc;
    }
  }
  *new_fill = S0 + (uint32_t)keep;
  return BG_OK;
}

int bg_kv_ring_evict(bg_kv_cache *kv, uint32_t fill, uint32_t need, uint32_t max_seq_len, uint32_t *new_fill) {
  if (!kv || !new_fill || kv->window == 0 || fill < kv->sinks || max_seq_len < kv->sinks) return BG_EINVAL;
  const uint32_t S0 = kv->sinks;
  const uint32_t recent = fill - S0;
  const uint32_t quarter = (max_seq_len - S0 + 3) / 4;
  uint32_t batchn = need > quarter ? need : quarter;
  if (batchn > recent) batchn = recent;
  const int64_t keep = (int64_t)recent - batchn;
  if (keep <= 0) {
    *new_fill = S0;
    kv->ring_head = 0;
    return BG_OK;
  }
  kv->ring_head = (uint32_t)(((uint64_t)kv->ring_head + batchn) % kv->window);
  *new_fill = S0 + (uint32_t)keep;
  return BG_OK;
}

int bg_deltanet_gbeta(const float *a, const float *b, const float *a_neg, const float *dt_bias, uint32_t S, uint32_t H,
                      float *out, bg_stream_t stream) {
  if (!a || !b || !a_neg || !dt_bias || !out) return BG_EINVAL;
  return launch_gbeta(a, b, a_neg, dt_bias, S, H, out, (cudaStream_t)stream);
}

int bg_deltanet_recur(const uint32_t params[8], const float *q, const float *k, const float *v, const float *g,
                      const float *beta, const float *state_in, float *core, float *state_out, bg_stream_t stream) {
  if (!params || !q || !k || !v || !g || !beta || !core || !state_out) return BG_EINVAL;
  DeltaArgs a = {};
  a.S = params[0];
  a.H = params[1];
  a.DK = params[2];
  a.DV = params[3];
  a.HK = params[4];
  a.betaOff = params[5];
  a.loadState = params[6];
  a.tOff = params[7];
  if (!a.H || !a.HK || a.H % a.HK || !a.DV || a.DV > 256) return BG_EINVAL;
  if (a.loadState && !state_in) return BG_EINVAL;
  a.q = q;
  a.k = k;
  a.v = v;
  a.g = g;
  a.beta = beta;
  a.state_in = state_in;
  a.state_out = state_out;
  a.core = core;
  return launch_deltanet(a, (cudaStream_t)stream);
}

int bg_deltanet_norm_gate(const float *core, const float *z, const float *gamma, uint32_t rows, uint32_t DV, float eps,
                          float *y, bg_stream_t stream) {
  if (!core || !z || !gamma || !y || !DV) return BG_EINVAL;
  return launch_norm_gate(core, z, gamma, rows, DV, eps, y, (cudaStream_t)stream);
}

int bg_deltanet_fused(uint32_t S, uint32_t H, uint32_t HK, uint32_t DK, uint32_t DV, const float *q, const float *k,
                      const float *v, const float *a, const float *b, const float *a_neg, const float *dt_bias,
                      const float *z, const float *gamma, float eps, const float *state_in, float *state_out,
                      float *core, float *y, bg_stream_t stream) {
  if (!q || !k || !v || !a || !b || !a_neg || !dt_bias || !z || !gamma || !y || !state_out) return BG_EINVAL;
  if (!H || !HK || H % HK || !DV || DV > 256) return BG_EINVAL;
  DeltaArgs d = {};
  d.S = S;
  d.H = H;
  d.HK = HK;
  d.DK = DK;
  d.DV = DV;
  d.loadState = state_in != nullptr;
  d.q = q;
  d.k = k;
  d.v = v;
  d.a = a;
  d.b = b;
  d.a_neg = a_neg;
  d.dt_bias = dt_bias;
  d.z = z;
  d.gamma = gamma;
  d.eps = eps;
  d.state_in = state_in;
  d.state_out = state_out;
  d.core = core;
  d.y = y;
  return launch_deltanet(d, (cudaStream_t)stream);
}

size_t bg_deltanet_chunked_workspace_size(uint32_t S, uint32_t H, uint32_t DK, uint32_t DV) {
  if (DK != 128 || DV != 128) return 0;
  return deltanet_chunk_workspace(S, H);
}

int bg_deltanet_chunked(uint32_t S, uint32_t H, uint32_t HK, uint32_t DK, uint32_t DV, const float *q, const float *k,
                        const float *v, const float *a, const float *b, const float *a_neg, const float *dt_bias,
                        const float *z, const float *gamma, float eps, const float *state_in, float *state_out,
                        float *core, float *y, void *workspace, size_t workspace_bytes, bg_stream_t stream) {
  if (!q || !k || !v || !a || !b || !a_neg || !dt_bias || !z || !gamma || !y || !state_out || !core) return BG_EINVAL;
  if (!H || !HK || H % HK) return BG_EINVAL;
  if (DK != 128 || DV != 128) return BG_EUNSUPPORTED;
  DeltaArgs d = {};
  d.S = S;
  d.H = H;
  d.HK = HK;
  d.DK = DK;
  d.DV = DV;
  d.loadState = state_in != nullptr;
  d.q = q;
  d.k = k;
  d.v = v;
  d.a = a;
  d.b = b;
  d.a_neg = a_neg;
  d.dt_bias = dt_bias;
  d.state_in = state_in;
  d.state_out = state_out;
  d.core = core;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = launch_deltanet_chunked(d, workspace, workspace_bytes, st);
  if (rc || S == 0) return rc;
  return launch_norm_gate(core, z, gamma, S * H, DV, eps, y, st);  // deltanet_norm_gate.wgsl
}

int bg_gate_sigmoid(const float *x, const float *gate, uint32_t n, float *y, bg_stream_t stream) {
  if (!x || !gate || !y) return BG_EINVAL;
  return launch_gate_sigmoid(x, gate, n, y, (cudaStream_t)stream);
}

}  // extern "C"
