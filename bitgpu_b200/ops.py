"""Torch-facing host mirror of bitgpu's attention-path operators.

Each function launches the sm_100a kernels of ``libbgattn.so`` through its C ABI on the current
torch CUDA stream.  Names follow the reference engine (``src/engine.ts``): ``KVCache.append``
is ``appendKV`` (engine.ts:1385-1393), ``KVCache.evict`` is ``evict`` (:1188-1212),
``attention`` is the ATT dispatch (:1543 / :1580 / :1487-1491), ``deltanet_*`` are the
hybrid-layer dispatches (:1438-1462).  Errors surface as ``BgError`` (the engine throws);
nothing here falls back to a CPU or torch implementation.
"""
import ctypes as C

import torch

from . import _lib
from ._lib import AttnParams, KVCacheDesc, check, lib

MODES = {"f32": _lib.KV_F32, "f16": _lib.KV_F16, "q8": _lib.KV_Q8, "q8r": _lib.KV_Q8R}
_DT = {torch.float32: _lib.DT_F32, torch.float16: _lib.DT_F16}


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(t, dtype=None, name="tensor"):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    return t


class Workspace:
    """Per-device scratch for split-KV partials, grown on demand (owned by the caller,
    as every C entry point takes scratch from its caller)."""

    def __init__(self):
        self.buf = {}

    def get(self, nbytes, device):
        key = torch.device(device).index
        b = self.buf.get(key)
        if b is None or b.numel() < nbytes:
            b = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self.buf[key] = b
        return b


WORKSPACE = Workspace()


class KVCache:
    """One layer's K/V cache for ``batch`` sequences in the reference layout
    ``[pos][kv_head][head_dim]`` per sequence (engine.ts:1051-1079).

    mode: 'f32' | 'f16' | 'q8' (reference q8_0-style, 32-element blocks) | 'q8r' (one
    absmax/127 scale per 128).  ``window > 0`` makes a rolling-window ring of ``window`` slots
    after ``sinks`` pinned slots (overflow 'sinks'); eviction then advances the ring head."""

    def __init__(self, batch, capacity, kv_heads, head_dim, mode="f16", sinks=0, window=0, device="cuda"):
        if mode not in MODES:
            raise ValueError(mode)
        if mode in ("q8", "q8r") and head_dim % 32:
            raise ValueError("q8 KV needs head_dim % 32 == 0")   # engine.ts:372-373
        self.batch, self.KV, self.D, self.mode = batch, kv_heads, head_dim, mode
        self.sinks, self.window, self.ring_head = sinks, window, 0
        self.capacity = sinks + window if window else capacity
        shape = (batch, self.capacity, kv_heads, head_dim)
        dt = {"f32": torch.float32, "f16": torch.float16, "q8": torch.int8, "q8r": torch.int8}[mode]
        self.K = torch.zeros(shape, dtype=dt, device=device)
        self.V = torch.zeros(shape, dtype=dt, device=device)
        self.Ks = self.Vs = None
        if mode in ("q8", "q8r"):
            blk = 32 if mode == "q8" else 128
            sshape = (batch, self.capacity, kv_heads, head_dim // blk)
            self.Ks = torch.zeros(sshape, dtype=torch.float32, device=device)
            self.Vs = torch.zeros(sshape, dtype=torch.float32, device=device)

    def desc(self):
        return KVCacheDesc(self.K.data_ptr(), self.V.data_ptr(),
                           self.Ks.data_ptr() if self.Ks is not None else None,
                           self.Vs.data_ptr() if self.Vs is not None else None,
                           self.capacity, MODES[self.mode], self.sinks, self.window, self.ring_head)

    def append(self, which, src, pos0):
        """``appendKV``: write ``src[batch, S, KV, D]`` (f32 or f16) at logical positions
        ``pos0 ..``; which 0 = K, 1 = V."""
        _need(src, name="src")
        B, S, KV, D = src.shape
        d = self.desc()
        check("bg_kv_append", lib().bg_kv_append(C.byref(d), which, B, _p(src), _DT[src.dtype], S, KV, D, pos0,
                                                  _stream()))

    def append_kv(self, k, v, pos0):
        """Both writes of ``appendKV`` (K then V, same shapes and dtype) in one launch."""
        _need(k, name="k")
        _need(v, k.dtype, "v")
        if k.shape != v.shape:
            raise ValueError("k and v shapes differ")
        B, S, KV, D = k.shape
        d = self.desc()
        check("bg_kv_append_kv", lib().bg_kv_append_kv(C.byref(d), B, _p(k), _p(v), _DT[k.dtype], S, KV, D, pos0,
                                                        _stream()))

    def append_kv_pair(self, other, k, v, pos0):
        """``append_kv`` into this cache and ``other`` (same shape, any codec) in one pass."""
        _need(k, name="k")
        _need(v, k.dtype, "v")
        if k.shape != v.shape:
            raise ValueError("k and v shapes differ")
        B, S, KV, D = k.shape
        d0, d1 = self.desc(), other.desc()
        check("bg_kv_append_kv_pair", lib().bg_kv_append_kv_pair(C.byref(d0), C.byref(d1), B, _p(k), _p(v),
                                                                  _DT[k.dtype], S, KV, D, pos0, _stream()))

    def write_normed_k(self, x, gamma, eps, pos, cos=None, sin=None, y=None):
        """Fused K path of the decode step (``rmsnorm_rope_sg{,_kv16,_kv8}``, engine.ts:1533-1540):
        ``x[batch, KV, D]`` -> RMSNorm*gamma -> RoPE(cos, sin of this position; None = unroped)
        -> cache at ``pos``."""
        _need(x, torch.float32, "x")
        B, R, D = x.shape
        d = self.desc()
        check("bg_rmsnorm_rope", lib().bg_rmsnorm_rope(_p(x), B, R, D, _p(gamma), _p(cos), _p(sin), eps, _p(y),
                                                        C.byref(d), pos, _stream()))

    def evict(self, fill, need, max_seq_len):
        """``evict(fill, need)`` of engine.ts:1188-1212; returns the new fill."""
        nf = C.c_uint32(0)
        d = self.desc()
        if self.window:
            check("bg_kv_ring_evict", lib().bg_kv_ring_evict(C.byref(d), fill, need, max_seq_len, C.byref(nf)))
            self.ring_head = d.ring_head
        else:
            check("bg_kv_evict", lib().bg_kv_evict(C.byref(d), self.batch, self.KV, self.D, fill, need, max_seq_len,
                                                    C.byref(nf), _stream()))
        return nf.value

    def evict_for(self, fill, n, max_seq_len):
        """``evictFor`` (engine.ts:1214): make room for ``n`` more rows."""
        return self.evict(fill, fill + n - max_seq_len, max_seq_len) if fill + n > max_seq_len else fill

    def logical_rows(self, fill):
        """Physical row index of each logical slot ``0..fill-1`` (ring mapping)."""
        idx = torch.arange(fill)
        if not self.window:
            return idx
        r = idx.clone()
        m = idx >= self.sinks
        r[m] = self.sinks + (self.ring_head + idx[m] - self.sinks) % self.window
        return r


def attention(q, cache, pos_base, scale=0.0, gate=None, cos_t=None, sin_t=None, out_dtype=torch.float32,
              out=None):
    """Causal GQA attention of ``q[batch, S, H, D]`` (f32 or f16) over ``cache``; query row
    ``qi`` attends logical positions ``0 .. pos_base+qi``.  ``cos_t/sin_t[positions, D/2]``
    select rope-at-read (sink mode); ``gate[batch, S, H, D]`` applies the sigmoid output gate."""
    _need(q, name="q")
    B, S, H, D = q.shape
    p = AttnParams(S, H, cache.KV, D, pos_base, pos_base + S)
    if out is None:
        out = torch.empty((B, S, H, D), dtype=out_dtype, device=q.device)
    nbytes = lib().bg_attention_workspace_size(C.byref(p), B)
    ws = WORKSPACE.get(nbytes, q.device)
    d = cache.desc()
    if gate is not None:
        _need(gate, torch.float32, "gate")
    check("bg_attention", lib().bg_attention(C.byref(p), B, _p(q), _DT[q.dtype], C.byref(d), _p(cos_t), _p(sin_t),
                                              float(scale), _p(gate), _p(out), _DT[out.dtype], _p(ws), ws.numel(),
                                              _stream()))
    return out


def attention_partials(q, cache, pos_base, pos_lo, pos_hi, scale=0.0, cos_t=None, sin_t=None):
    """Split-KV partial ``[B*S*H, D+2]`` over logical positions ``[pos_lo, pos_hi)`` held in
    ``cache`` starting at physical row 0."""
    B, S, H, D = q.shape
    p = AttnParams(S, H, cache.KV, D, pos_base, pos_base + S)
    part = torch.empty((B * S * H, D + 2), dtype=torch.float32, device=q.device)
    nbytes = lib().bg_attention_workspace_size(C.byref(p), B)
    ws = WORKSPACE.get(nbytes, q.device)
    d = cache.desc()
    check("bg_attention_partials", lib().bg_attention_partials(C.byref(p), B, _p(q), _DT[q.dtype], C.byref(d),
                                                                _p(cos_t), _p(sin_t), float(scale), pos_lo, pos_hi,
                                                                _p(part), _p(ws), ws.numel(), _stream()))
    return part


def attention_peer(q, cache, pos_base, pos_lo, pos_hi, exchange, scale=0.0, gate=None, out_dtype=torch.float32,
                   out=None):
    """One split-KV decode step over ranks that each hold positions ``[pos_lo, pos_hi)`` of the
    stream in ``cache``: this rank's partials go straight into every rank's gather buffer
    (``exchange``: a ``bitgpu_b200.splitkv.PeerExchange``) and the merged, gated rows come back in
    ``out`` on every rank -- one kernel for f16 / q8 caches."""
    _need(q, name="q")
    B, S, H, D = q.shape
    p = AttnParams(S, H, cache.KV, D, pos_base, pos_base + S)
    if out is None:
        out = torch.empty((B, S, H, D), dtype=out_dtype, device=q.device)
    if gate is not None:
        _need(gate, torch.float32, "gate")
    nbytes = lib().bg_attention_peer_workspace_size(C.byref(p), B)
    ws = WORKSPACE.get(nbytes, q.device)
    d = cache.desc()
    check("bg_attention_peer", lib().bg_attention_peer(C.byref(p), B, _p(q), _DT[q.dtype], C.byref(d), float(scale),
                                                        pos_lo, pos_hi, C.byref(exchange.desc), _p(gate), _p(out),
                                                        _DT[out.dtype], _p(ws), ws.numel(), _stream()))
    return out


def lse_merge(partials, out_shape, gate=None, out_dtype=torch.float32):
    """Merge ``partials[nsplit, rows, D+2]`` into the normalised (optionally gated) output."""
    _need(partials, torch.float32, "partials")
    ns, rows, D2 = partials.shape
    out = torch.empty(out_shape, dtype=out_dtype, device=partials.device)
    check("bg_lse_merge", lib().bg_lse_merge(_p(partials), ns, rows, D2 - 2, _p(gate), _p(out), _DT[out_dtype],
                                              _stream()))
    return out


def deltanet_gbeta(a, b, a_neg, dt_bias):
    S, H = a.shape
    out = torch.empty(2 * S * H, dtype=torch.float32, device=a.device)
    check("bg_deltanet_gbeta", lib().bg_deltanet_gbeta(_p(a), _p(b), _p(a_neg), _p(dt_bias), S, H, _p(out),
                                                        _stream()))
    return out


def deltanet_recur(params, q, k, v, g, beta, state_in, core, state_out):
    """``deltanet_recur`` with its WGSL Params ``[S, H, DK, DV, HK, betaOff, loadState, tOff]``."""
    arr = (C.c_uint32 * 8)(*[int(x) for x in params])
    check("bg_deltanet_recur", lib().bg_deltanet_recur(C.byref(arr), _p(q), _p(k), _p(v), _p(g), _p(beta),
                                                        _p(state_in), _p(core), _p(state_out), _stream()))


def deltanet_norm_gate(core, z, gamma, eps):
    rows, DV = core.shape
    y = torch.empty_like(core)
    check("bg_deltanet_norm_gate", lib().bg_deltanet_norm_gate(_p(core), _p(z), _p(gamma), rows, DV, float(eps),
                                                                _p(y), _stream()))
    return y


def deltanet_fused(q, k, v, a, b, a_neg, dt_bias, z, gamma, eps, state_in=None, state_out=None, want_core=False):
    """One segment of the linear-attention mixer: g/beta -> recurrence -> gated RMSNorm.
    q, k ``[S, HK, DK]``; v, z ``[S, H, DV]``; a, b ``[S, H]``.  Returns ``(y, state_out, core)``."""
    S, HK, DK = q.shape
    H, DV = v.shape[1], v.shape[2]
    if state_out is None:
        state_out = torch.empty((H, DK, DV), dtype=torch.float32, device=q.device)
    y = torch.empty((S, H, DV), dtype=torch.float32, device=q.device)
    core = torch.empty_like(y) if want_core else None
    check("bg_deltanet_fused", lib().bg_deltanet_fused(S, H, HK, DK, DV, _p(q), _p(k), _p(v), _p(a), _p(b),
                                                        _p(a_neg), _p(dt_bias), _p(z), _p(gamma), float(eps),
                                                        _p(state_in), _p(state_out), _p(core), _p(y), _stream()))
    return y, state_out, core


def deltanet_chunked(q, k, v, a, b, a_neg, dt_bias, z, gamma, eps, state_in=None, state_out=None):
    """Prefill form of ``deltanet_fused``: the chunk-parallel (WY, 64-token chunks) delta rule,
    then the gated RMSNorm.  Returns ``(y, state_out, core)``."""
    S, HK, DK = q.shape
    H, DV = v.shape[1], v.shape[2]
    if state_out is None:
        state_out = torch.empty((H, DK, DV), dtype=torch.float32, device=q.device)
    y = torch.empty((S, H, DV), dtype=torch.float32, device=q.device)
    core = torch.empty_like(y)
    nbytes = lib().bg_deltanet_chunked_workspace_size(S, H, DK, DV)
    ws = WORKSPACE.get(nbytes, q.device)
    check("bg_deltanet_chunked", lib().bg_deltanet_chunked(S, H, HK, DK, DV, _p(q), _p(k), _p(v), _p(a), _p(b),
                                                            _p(a_neg), _p(dt_bias), _p(z), _p(gamma), float(eps),
                                                            _p(state_in), _p(state_out), _p(core), _p(y), _p(ws),
                                                            ws.numel(), _stream()))
    return y, state_out, core


def conv1d_causal(x, w, state_in=None, state_out=None):
    """``conv1d_causal`` (engine.ts:1422-1427): depthwise causal conv + SiLU of ``x[S, C]`` with
    ``w[C, K]`` after the carried ``state_in[K-1, C]`` (None: zero left pad).
    Returns ``(y[S, C], state_out[K-1, C])``."""
    _need(x, torch.float32, "x")
    _need(w, torch.float32, "w")
    S, Cc = x.shape
    K = w.shape[1]
    y = torch.empty_like(x)
    if state_out is None:
        state_out = torch.empty((K - 1, Cc), dtype=torch.float32, device=x.device)
    check("bg_conv1d_causal", lib().bg_conv1d_causal(_p(x), _p(w), _p(state_in), int(state_in is not None), S, Cc,
                                                      K, _p(y), _p(state_out), _stream()))
    return y, state_out


def slice_cols(src, rows, width, stride, off):
    """``slice_cols`` / ``split_head``: ``dst[r, c] = src.flat[r*stride + off + c]`` -> ``[rows, width]``."""
    _need(src, torch.float32, "src")
    dst = torch.empty((rows, width), dtype=torch.float32, device=src.device)
    check("bg_slice_cols", lib().bg_slice_cols(_p(src), rows, width, stride, off, _p(dst), _stream()))
    return dst


def qk_norm_rope(x, batch, S, heads, D, x_stride, x_off, gamma, cos, sin, rot, pos0, eps, cache=None, want_y=True):
    """The gated-attention prologue (engine.ts:1471-1485): split_head row read, RMSNorm with the
    baked scale ``gamma``, partial RoPE over the first ``rot`` dims (tables ``[pos][rot]`` at row
    ``pos0 + s``); returns ``y[batch, S, heads, D]`` (when ``want_y``) and/or writes the cache."""
    _need(x, torch.float32, "x")
    y = torch.empty((batch, S, heads, D), dtype=torch.float32, device=x.device) if want_y else None
    d = cache.desc() if cache is not None else None
    check("bg_qk_norm_rope", lib().bg_qk_norm_rope(_p(x), batch, S, heads, D, x_stride, x_off, _p(gamma), _p(cos),
                                                    _p(sin), rot, pos0, float(eps), _p(y),
                                                    C.byref(d) if d is not None else None, _stream()))
    return y


def gate_sigmoid(x, gate):
    y = torch.empty_like(x)
    check("bg_gate_sigmoid", lib().bg_gate_sigmoid(_p(x), _p(gate), x.numel(), _p(y), _stream()))
    return y


class Graphed:
    """Capture a sequence of these ops once as a CUDA graph and replay it.

    Decode steps of the small layers (one DeltaNet token, a short-context attention) are a few
    microseconds of GPU work behind tens of microseconds of host launch overhead; replaying a
    captured graph removes the host from the per-step path.  Inputs and outputs must live in
    fixed buffers (copy new inputs into them before ``replay``)."""

    def __init__(self, fn, warmup=2):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = fn()

    def replay(self):
        self.graph.replay()
        return self.out

    __call__ = replay
