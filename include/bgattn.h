/* bgattn.h -- C ABI of the B200 (sm_100a) attention hot path for bitgpu.
 *
 * Every entry point replaces one WebGPU dispatch (or one engine helper) of bitgpu's attention
 * path; the reference interface is cited beside each declaration as file:line of the bitgpu
 * source tree.  Conventions shared by all entry points:
 *   - all pointers are DEVICE pointers owned by the caller; no entry point allocates device
 *     memory (scratch comes in through `workspace`);
 *   - work is enqueued asynchronously on `stream` (a cudaStream_t, NULL = legacy stream);
 *   - return 0 on success or a negative BG_E* code (never aborts); bg_strerror() names it;
 *   - float math is IEEE f32 (no fast-math); KV storage codecs follow the reference exactly.
 *
 * KV cache layout (reference: shaders/attention_sg.wgsl:11-12, src/engine.ts:1072-1079):
 *   element (seq b, position p, kv head h, dim d) lives at
 *     row = (b*seq_stride + phys(p))*KV + h,  offset = row*D + d
 *   f32/f16: one element per value; q8: int8 codes (== packed u32 snorm8 words, component 0 in
 *   the low byte, shaders/copy_kv8.wgsl:39) plus one f32 scale per 32-element block at
 *   Ks[row*(D/32) + d/32] (shaders/copy_kv8.wgsl:35); q8r (extra mode, not in the reference):
 *   one absmax/127 scale per row of 128 at Ks[row*(D/128) + d/128].
 *   phys(p) = p when window == 0; otherwise (rolling window with `sinks` pinned slots,
 *   overflow 'sinks', src/engine.ts:1180-1214) phys(p) = p < sinks ? p
 *   : sinks + (ring_head + p - sinks) % window, so eviction can advance ring_head instead of
 *   moving bytes (bg_kv_ring_evict) while logical slots keep the reference's order.
 */
#ifndef BGATTN_H
#define BGATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void *bg_stream_t; /* cudaStream_t */

enum {
  BG_OK = 0,
  BG_EINVAL = -1,       /* bad parameters (the engine's validation throws, engine.ts:232-235,372) */
  BG_ENOMEM = -2,       /* workspace too small */
  BG_ELAUNCH = -3,      /* CUDA launch / runtime error */
  BG_ETIMEOUT = -4,     /* a bounded device wait gave up */
  BG_EUNSUPPORTED = -5  /* shape / mode combination not built */
};

enum { BG_KV_F32 = 0, BG_KV_F16 = 1, BG_KV_Q8 = 2, BG_KV_Q8R = 3 };
enum { BG_DT_F32 = 0, BG_DT_F16 = 1 };

/* == struct Params of shaders/attention_sg.wgsl:7 (also _wg, _kv16, _kv8, _roll variants). */
typedef struct {
  uint32_t S, H, KV, D, posBase, Ltot;
} bg_attn_params;

/* One layer's K/V cache for `batch` sequences (src/engine.ts:1051-1079 Kc/Vc/Ksc/Vsc). */
typedef struct {
  void *K, *V;         /* f32 / f16 values or int8 codes */
  float *Ks, *Vs;      /* q8 / q8r scales, NULL otherwise */
  uint64_t seq_stride; /* positions per sequence slab (the cache capacity) */
  uint32_t mode;       /* BG_KV_* */
  uint32_t sinks, window, ring_head; /* rolling window; window == 0: linear */
} bg_kv_cache;

const char *bg_strerror(int code);
int bg_version(void);
/* Synchronise `stream`, then report (and clear) a bounded device wait that gave up in any kernel
 * of this library since the last call: BG_ETIMEOUT, else BG_OK.  Every spin on an mbarrier in
 * these kernels is bounded; on expiry the kernel records the timeout and returns instead of
 * hanging (the engine's device-lost path, engine.ts:400-409, is the reference counterpart). */
int bg_device_status(bg_stream_t stream);
/* Self-test of the bounded device waits (no reference counterpart: the reference's device-lost
 * path, engine.ts:400-409, is driven by the browser).  Launches one CTA that waits on an
 * mbarrier nothing ever arrives on, giving up after `polls` polls (1 .. 2^20) exactly as every
 * kernel of this library gives up after its own limit: the kernel records BG_ETIMEOUT and
 * returns, the context stays usable, and bg_device_status(stream) then reports BG_ETIMEOUT. */
int bg_selftest_wait_expiry(uint32_t polls, bg_stream_t stream);
/* Route every attention call through the CUDA-core kernel instead of the tensor-core one (the
 * reference's forceNoSubgroups option, src/types.ts / engine.ts:282, which forces the _wg
 * fallback kernels).  Process-wide; returns the previous setting.  For A/B checks only. */
int bg_force_generic(int on);

/* ---- attention (decode S small, prefill / PLD verify S > 1) -------------------------------
 * Replaces the ATT dispatch of src/engine.ts:1543 (fused decode) and :1580 (prefill), i.e.
 * shaders/attention_{sg,wg}{,_kv16,_kv8}.wgsl, and the head_dim-256 hybrid kernels
 * attention_online_cache{,_kv8}.wgsl via engine.ts:1487-1489, with gate_sigmoid.wgsl
 * (engine.ts:1491) fused when `gate` is non-NULL.
 * q [batch][S][H][D] (q_dtype), out [batch][S][H][D] (out_dtype); query row qi of every
 * sequence attends logical cache positions 0..posBase+qi (Ltot must be posBase+S).
 * scale == 0 selects 1/sqrt(D) (attention_sg.wgsl:24); the online kernels pass it explicitly.
 * cosT/sinT non-NULL selects rope-at-read of unroped keys by logical slot, tables
 * [positions][D/2] (the attention_*_roll.wgsl kernels, bindings engine.ts:1395-1399).
 * gate [batch][S][H][D] f32 or NULL: out = att / (1 + exp(-gate)).
 * Workspace: bg_attention_workspace_size bytes covers split-KV partials and, for a prefill
 * (S >= 64) over a q8 cache, an f16 copy of the cache positions [0, Ltot) that the tensor-core
 * prefill dequantises into once; with less, that prefill dequantises inside its kernel. */
size_t bg_attention_workspace_size(const bg_attn_params *p, uint32_t batch);
int bg_attention(const bg_attn_params *p, uint32_t batch, const void *q, uint32_t q_dtype,
                 const bg_kv_cache *kv, const float *cosT, const float *sinT, float scale,
                 const float *gate, void *out, uint32_t out_dtype, void *workspace,
                 size_t workspace_bytes, bg_stream_t stream);

/* bg_attention_noalloc: bg_attention for callers that cannot allocate device memory.
 * No counterpart in the reference (its kernels take every buffer from the engine).  Some hosts
 * cannot hand over a scratch buffer: the engine's device memory may all belong to another
 * allocator with none exposed across the binding, or the token loop may not call cudaMalloc
 * (which can synchronise the device).  This variant takes no workspace: it uses a fixed
 * BG_NOALLOC_SCRATCH_BYTES (8 MiB) scratch array compiled into the library, held on every GPU
 * that loads the library until the process exits.  Same arguments and results as bg_attention
 * minus the workspace; returns BG_ENOMEM when the call's split-KV partials exceed the limit
 * (bg_attention_noalloc_limit() reports it); a q8 prefill too large to dequantise into the array
 * dequantises inside its kernel instead.  Every call looks up the array's device
 * address in the current context (so it stays right after cudaDeviceReset); make the first call
 * on a device before any stream capture.  All calls share the one array: calls that overlap on
 * the GPU (different streams, or several host threads) race on it and must be serialised by the
 * caller. */
#define BG_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)
size_t bg_attention_noalloc_limit(void);
int bg_attention_noalloc(const bg_attn_params *p, uint32_t batch, const void *q, uint32_t q_dtype,
                         const bg_kv_cache *kv, const float *cosT, const float *sinT, float scale,
                         const float *gate, void *out, uint32_t out_dtype, bg_stream_t stream);

/* ---- split-KV across GPUs (no reference counterpart: the reference is single-device) ----
 * Partial attention over the cache positions [pos_lo, pos_hi) that THIS caller holds: the
 * local cache `kv` stores position pos_lo at physical row 0.  partials
 * [batch*S*H][D+2] = (unnormalised o[D], running max m, sum l), m = -inf / l = 0 for rows
 * that attend nothing in the slice.  bg_lse_merge combines nsplit such blocks laid out
 * [nsplit][rows][D+2] (e.g. an all-gather result) into out, applying the optional gate. */
int bg_attention_partials(const bg_attn_params *p, uint32_t batch, const void *q,
                          uint32_t q_dtype, const bg_kv_cache *kv, const float *cosT,
                          const float *sinT, float scale, uint32_t pos_lo, uint32_t pos_hi,
                          float *partials, void *workspace, size_t workspace_bytes,
                          bg_stream_t stream);
int bg_lse_merge(const float *partials, uint32_t nsplit, uint32_t rows, uint32_t D,
                 const float *gate, void *out, uint32_t out_dtype, bg_stream_t stream);

/* ---- split-KV exchange through peer memory (no reference counterpart) ----------------------
 * bg_attention_peer: one decode step of a stream whose cache positions are sharded over the ranks
 * of one node, with the partials' exchange done by NVLink peer stores instead of a collective.
 * Every rank allocates one buffer of bg_peer_exchange_bytes(nranks, rows, D) bytes that all ranks
 * can address (e.g. torch symmetric memory, or CUDA IPC / VMM mappings), zeroed before the first
 * step: gather slots [2][nranks][rows][D+2] f32 at offset 0, then per-row arrival counters
 * [nranks][rows] u32 at bg_peer_exchange_flags_offset(nranks, rows, D); rows = batch*S*H.  `step`,
 * `done` and `tickets` (batch*KV entries) are zeroed u32 in this rank's own device memory.
 * Each rank passes its local slice [pos_lo, pos_hi) as in bg_attention_partials; out receives the
 * merged, gated rows on every rank.  After the split-KV kernel a push kernel merges this rank's
 * splits and stores the rows into every rank; a merge kernel waits -- bounded by spin_limit polls,
 * 0 = default -- for the other ranks' rows, merges and gates.  (BGATTN_PEER_FUSED=1 lets the
 * tensor-core kernel do both in the last CTA of each (sequence, kv head) group instead.)  Every rank must run the same
 * sequence of steps with the same shapes; steps may be captured in a CUDA graph (the step number
 * lives in `step`).  A wait that runs out shows as BG_ETIMEOUT in bg_device_status. */
#define BG_MAX_PEERS 8
typedef struct {
  uint32_t nranks, rank;
  float *gather[BG_MAX_PEERS];    /* rank r's buffer, as addressed from this GPU */
  uint32_t *flags[BG_MAX_PEERS];  /* rank r's arrival counters, as addressed from this GPU */
  uint32_t *step, *done, *tickets;
  uint32_t spin_limit;
} bg_peer_exchange;
size_t bg_peer_exchange_bytes(uint32_t nranks, uint32_t rows, uint32_t D);
size_t bg_peer_exchange_flags_offset(uint32_t nranks, uint32_t rows, uint32_t D);
size_t bg_attention_peer_workspace_size(const bg_attn_params *p, uint32_t batch);
int bg_attention_peer(const bg_attn_params *p, uint32_t batch, const void *q, uint32_t q_dtype,
                      const bg_kv_cache *kv, float scale, uint32_t pos_lo, uint32_t pos_hi,
                      const bg_peer_exchange *x, const float *gate, void *out, uint32_t out_dtype,
                      void *workspace, size_t workspace_bytes, bg_stream_t stream);

/* ---- KV cache writers ---------------------------------------------------------------------
 * bg_kv_append: appendKV(pass, src, which, li, rows, dstRow0) of src/engine.ts:1385-1393
 * (copy.wgsl / copy_kv16.wgsl / copy_kv8.wgsl).  which: 0 = K, 1 = V.  src [batch][S][KV][D]
 * (src_dtype) is written at logical positions pos0..pos0+S-1 (dstRow0 = pos0*KV). */
int bg_kv_append(const bg_kv_cache *kv, uint32_t which, uint32_t batch, const void *src,
                 uint32_t src_dtype, uint32_t S, uint32_t KV, uint32_t D, uint32_t pos0,
                 bg_stream_t stream);

/* bg_kv_append_kv: both writes of one appendKV step (engine.ts:1385-1393 dispatches the K and
 * the V copy back to back) in a single launch; same layout, codec and errors as two
 * bg_kv_append calls with which = 0 and 1. */
int bg_kv_append_kv(const bg_kv_cache *kv, uint32_t batch, const void *k_src, const void *v_src,
                    uint32_t src_dtype, uint32_t S, uint32_t KV, uint32_t D, uint32_t pos0,
                    bg_stream_t stream);

/* bg_kv_append_kv_pair: the same K and V rows written into two caches of one shape in a single
 * pass that reads the source once (e.g. a prefill's rows into an f16 cache and a q8 cache, the
 * BASELINE config-3 write); each cache keeps its own codec.  Same layout and errors as
 * bg_kv_append_kv on each cache.  No single reference dispatch does this: it replaces two
 * appendKV steps (engine.ts:1385-1393) over different caches. */
int bg_kv_append_kv_pair(const bg_kv_cache *kv0, const bg_kv_cache *kv1, uint32_t batch,
                         const void *k_src, const void *v_src, uint32_t src_dtype, uint32_t S,
                         uint32_t KV, uint32_t D, uint32_t pos0, bg_stream_t stream);

/* bg_qk_norm_rope: the gated-attention prologue of engine.ts:1471-1485 in one launch, for
 * batch x S x heads head rows of width D:
 *   split_head.wgsl  row (b, s, h) is read at x + ((b*S + s)*heads + h)*x_stride + x_off
 *                    (x_stride = 2*D, x_off = 0 picks the query half of the doubled q_proj);
 *   rms              y = x * rsqrt(mean(x^2) + eps) * gamma (gamma = the baked (1 + w) scale);
 *   rope_partial.wgsl rotate_half inside the first `rot` dims with the tables cosT/sinT
 *                    [positions][rot] at row pos0 + s; dims >= rot pass through (rot = 0: none).
 * The result goes to y [batch][S][heads][D] when y != NULL and/or into the cache's K at logical
 * positions pos0 .. pos0+S-1 (heads == the cache's kv heads), with the cache's codec (the
 * appendKV that follows it in the engine). */
int bg_qk_norm_rope(const float *x, uint32_t batch, uint32_t S, uint32_t heads, uint32_t D,
                    uint32_t x_stride, uint32_t x_off, const float *gamma, const float *cosT,
                    const float *sinT, uint32_t rot, uint32_t pos0, float eps, float *y,
                    const bg_kv_cache *kv, bg_stream_t stream);

/* ---- KV snapshot wire format ---------------------------------------------------------------
 * saveCache / restoreCache of engine.ts:2719-2872 (KvSnapshot, src/types.ts:364-390): one
 * layer's share of `data` is, for cache positions [base, base+count) in LOGICAL order, the K rows,
 * then the V rows, then (q8) the K block-scale rows and the V block-scale rows, each row in the
 * cache's own bytes ([kv_head][D] of f32 / f16 / int8 codes; scales [kv_head][D/32] f32).  On a
 * ring cache (window > 0) the logical order is gathered from the physical ring (sinks, then the
 * window from ring_head), so the bytes equal those of the reference's compacted cache; restore
 * scatters through the same mapping (a restored snapshot is usually written with ring_head = 0).
 * dst / src may be host (pageable or pinned) or device memory; `seq` selects the sequence of a
 * batched cache.  The DeltaNet state [H][DK][DV] and the conv left context [K-1][C] that follow
 * the layers in `data` are plain copies of those buffers. */
size_t bg_kv_snapshot_bytes(const bg_kv_cache *kv, uint32_t KV, uint32_t D, uint32_t count);
int bg_kv_snapshot_save(const bg_kv_cache *kv, uint32_t seq, uint32_t KV, uint32_t D, uint32_t base,
                        uint32_t count, void *dst, bg_stream_t stream);
int bg_kv_snapshot_restore(const bg_kv_cache *kv, uint32_t seq, uint32_t KV, uint32_t D, uint32_t base,
                           uint32_t count, const void *src, bg_stream_t stream);

/* ---- hybrid-layer glue --------------------------------------------------------------------
 * bg_conv1d_causal: conv1d_causal.wgsl (engine.ts:1422-1427).  Depthwise causal conv + SiLU over
 * ext = [state_in (K-1 rows, zeros unless load_state); x (S rows)]:
 *   y[t][c] = silu(sum_{j<K} w[c][j] * ext[t+j][c]),  state_out[i][c] = ext[S+i][c] (i < K-1).
 * x, y [S][C]; w [C][K]; state_in, state_out [K-1][C] and distinct (the engine ping-pongs them).
 * K <= 8. */
int bg_conv1d_causal(const float *x, const float *w, const float *state_in, uint32_t load_state,
                     uint32_t S, uint32_t C, uint32_t K, float *y, float *state_out,
                     bg_stream_t stream);

/* bg_slice_cols: slice_cols.wgsl (engine.ts:1428-1430) and split_head.wgsl (engine.ts:1473-1474):
 * dst[r][c] = src[r*stride + off + c] for r < rows, c < width (off + width <= stride).
 * split_head(S, H, Dh, off) == bg_slice_cols(src, S*H, Dh, 2*Dh, off, dst). */
int bg_slice_cols(const float *src, uint32_t rows, uint32_t width, uint32_t stride, uint32_t off,
                  float *dst, bg_stream_t stream);

/* bg_rmsnorm_rope: rmsnorm_rope_sg{,_kv16,_kv8}.wgsl (engine.ts:1529-1540): per head row
 * y = rmsnorm(x)*gamma rotated by (cos, sin) ([D] tables of this position; NULL/NULL = no
 * rotation, the sink-mode cos=1/sin=0 binding of engine.ts:1533).  x [batch][R][D]; the result
 * goes to y [batch][R][D] when y != NULL and/or into the cache at logical position `pos`
 * (R == KV rows) when kv != NULL. */
int bg_rmsnorm_rope(const float *x, uint32_t batch, uint32_t R, uint32_t D, const float *gamma,
                    const float *cos, const float *sin, float eps, float *y,
                    const bg_kv_cache *kv, uint32_t pos, bg_stream_t stream);

/* bg_kv_evict: evict() of src/engine.ts:1188-1212 (batched sink compaction, bytes moved, no
 * re-rope / requantise) for a linear cache; *new_fill receives the engine's return value. */
int bg_kv_evict(const bg_kv_cache *kv, uint32_t batch, uint32_t KV, uint32_t D, uint32_t fill,
                uint32_t need, uint32_t max_seq_len, uint32_t *new_fill, bg_stream_t stream);
/* bg_kv_ring_evict: the same schedule on a ring cache (window > 0): advances kv->ring_head,
 * moves no bytes.  Host-only bookkeeping. */
int bg_kv_ring_evict(bg_kv_cache *kv, uint32_t fill, uint32_t need, uint32_t max_seq_len,
                     uint32_t *new_fill);

/* ---- gated DeltaNet ----------------------------------------------------------------------
 * bg_deltanet_gbeta: deltanet_gbeta.wgsl (engine.ts:1438); out [2*S*H] = [g ; beta]. */
int bg_deltanet_gbeta(const float *a, const float *b, const float *a_neg, const float *dt_bias,
                      uint32_t S, uint32_t H, float *out, bg_stream_t stream);
/* bg_deltanet_recur: deltanet_recur.wgsl (engine.ts:1446-1458); params == its Params
 * {S, H, DK, DV, HK, betaOff, loadState, tOff}.  q,k [*, HK, DK]; v [*, H, DV]; g and beta
 * [*, H] (beta read at beta[betaOff + ...], so it may point into the gbeta buffer);
 * state [H][DK][DV]; core [*, H, DV].  state_out may alias state_in. */
int bg_deltanet_recur(const uint32_t params[8], const float *q, const float *k, const float *v,
                      const float *g, const float *beta, const float *state_in, float *core,
                      float *state_out, bg_stream_t stream);
/* bg_deltanet_norm_gate: deltanet_norm_gate.wgsl (engine.ts:1462). */
int bg_deltanet_norm_gate(const float *core, const float *z, const float *gamma, uint32_t rows,
                          uint32_t DV, float eps, float *y, bg_stream_t stream);
/* bg_deltanet_fused: gbeta -> recurrence -> gated norm in one launch (engine.ts:1438-1462 for
 * one segment).  state_in NULL = zero state; y [S][H][DV] normed output; core may be NULL. */
int bg_deltanet_fused(uint32_t S, uint32_t H, uint32_t HK, uint32_t DK, uint32_t DV,
                      const float *q, const float *k, const float *v, const float *a,
                      const float *b, const float *a_neg, const float *dt_bias, const float *z,
                      const float *gamma, float eps, const float *state_in, float *state_out,
                      float *core, float *y, bg_stream_t stream);

/* bg_deltanet_chunked: the same segment computed in the chunk-parallel WY form of
 * tools/qwen35_numpy.py:144-187 (_delta_chunk; chunks of 64 tokens; equal to the recurrence up to
 * f32 accumulation order), for prefill.  Same arguments as bg_deltanet_fused plus a workspace of
 * bg_deltanet_chunked_workspace_size(S, H, DK, DV) bytes; DK = DV = 128 only. */
size_t bg_deltanet_chunked_workspace_size(uint32_t S, uint32_t H, uint32_t DK, uint32_t DV);
int bg_deltanet_chunked(uint32_t S, uint32_t H, uint32_t HK, uint32_t DK, uint32_t DV,
                        const float *q, const float *k, const float *v, const float *a,
                        const float *b, const float *a_neg, const float *dt_bias, const float *z,
                        const float *gamma, float eps, const float *state_in, float *state_out,
                        float *core, float *y, void *workspace, size_t workspace_bytes,
                        bg_stream_t stream);

/* bg_gate_sigmoid: gate_sigmoid.wgsl (engine.ts:1491), y = x / (1 + exp(-gate)). */
int bg_gate_sigmoid(const float *x, const float *gate, uint32_t n, float *y, bg_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* BGATTN_H */
