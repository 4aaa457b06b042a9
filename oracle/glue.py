"""Hybrid-layer glue -- CPU restatement (TEST INFRASTRUCTURE ONLY; see ``oracle/__init__``).

* ``conv1d_causal``: depthwise causal conv + SiLU over ``ext = [state_in (K-1 rows); x]``,
  ``y[t,c] = silu(sum_j w[c,j] ext[t+j,c])``, ``state_out = ext[S:S+K-1]``
  (``shaders/conv1d_causal.wgsl:1-36``; with a zero state it is ``tools/qwen35_numpy.py``
  ``_conv1d_causal``, ``:118-125``).
* ``slice_cols``: ``dst[r, c] = src[r*stride + off + c]`` (``shaders/slice_cols.wgsl:9-15``);
  ``split_head`` is the same with ``stride = 2*Dh`` (``shaders/split_head.wgsl:9-16``).
* ``rmsnorm``: ``x * rsqrt(mean(x^2) + eps) * gamma`` with the baked scale
  (``tools/qwen35_numpy.py:71-74`` stores ``1 + weight``).
* ``rope_partial``: rotate_half inside the first ``rot`` dims, tables ``[S, rot]``, the rest
  passes through (``shaders/rope_partial.wgsl:12-24``; ``tools/qwen35_numpy.py:84-89``).
* ``qk_norm_rope``: split_head -> rmsnorm -> rope_partial, the prologue of
  ``src/engine.ts:1471-1485``.
"""
import numpy as np

F32 = np.float32


def conv1d_causal(x, w, state_in=None):
    """x [S, C], w [C, K], state_in [K-1, C] or None (zeros) -> (y [S, C], state_out [K-1, C])."""
    x = np.asarray(x, F32)
    w = np.asarray(w, F32)
    S, C = x.shape
    K = w.shape[1]
    st = np.zeros((K - 1, C), F32) if state_in is None else np.asarray(state_in, F32).reshape(K - 1, C)
    ext = np.concatenate([st, x], 0)
    acc = np.zeros((S, C), F32)
    for j in range(K):
        acc = (acc + w[:, j][None, :] * ext[j:j + S]).astype(F32)
    y = (acc / (F32(1.0) + np.exp(-acc))).astype(F32)
    return y, ext[S:S + K - 1].copy()


def slice_cols(src, rows, width, stride, off):
    s = np.asarray(src, F32).reshape(-1)[: rows * stride].reshape(rows, stride)
    return s[:, off:off + width].copy()


def rmsnorm(x, gamma, eps):
    x = np.asarray(x, F32)
    inv = (F32(1.0) / np.sqrt((x * x).mean(-1, keepdims=True) + F32(eps))).astype(F32)
    return (x * inv * np.asarray(gamma, F32)).astype(F32)


def rope_partial(x, cos, sin, rot):
    """x [S, H, D]; cos, sin [S, rot]."""
    x = np.asarray(x, F32)
    if rot == 0:
        return x.copy()
    half = rot // 2
    xr, xp = x[..., :rot], x[..., rot:]
    rotated = np.concatenate([-xr[..., half:], xr[..., :half]], -1)
    out = xr * np.asarray(cos, F32)[:, None, :] + rotated * np.asarray(sin, F32)[:, None, :]
    return np.concatenate([out.astype(F32), xp], -1)


def qk_norm_rope(x, heads, D, x_stride, x_off, gamma, cos, sin, rot, eps):
    """x [S, heads*x_stride] (rows read at h*x_stride + x_off) -> [S, heads, D]."""
    x = np.asarray(x, F32)
    S = x.shape[0]
    rows = slice_cols(x.reshape(S * heads, x_stride), S * heads, D, x_stride, x_off).reshape(S, heads, D)
    return rope_partial(rmsnorm(rows, gamma, eps), cos, sin, rot)


def rope_tables(S, rot, theta):
    """[S, rot] cos/sin with f64 angles rounded once to f32 (tools/qwen35_numpy.py:77-81)."""
    inv = 1.0 / (theta ** (np.arange(0, rot, 2, dtype=np.float64) / rot))
    frq = np.outer(np.arange(S, dtype=np.float64), inv)
    emb = np.concatenate([frq, frq], -1)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)
