"""Causal GQA attention over a KV cache -- CPU restatement of the reference math.

Semantics (``shaders/attention_sg.wgsl:15-45``, identical in every ``attention_*`` variant):
query row ``qi`` of head ``h`` sits at cache position ``posBase + qi`` and attends to cache
positions ``0 .. posBase+qi`` inclusive of kv head ``kvh = h / (H/KV)``; score =
``(q . K[j]) * scale`` with ``scale = 1/sqrt(D)`` (``attention_sg.wgsl:24``) or the explicit
``scale`` parameter of the head_dim-256 kernels (``attention_online_cache.wgsl:7,38``);
softmax over the attended positions; output ``sum_j p_j V[j]``.  The softmax is written the
way ``tools/reference.py:158-175`` / ``tools/gen-kernel-cases.py:108-115`` write it (masked
positions ``-1e30``, max-subtract, exp, normalise), all float32.

Cache layout: ``K[pos, KV, D]`` float32 values *after* the storage codec's read
(``oracle.kvcodec.decode``), so f16/q8 caches are checked through the exact values the
reference kernels reconstruct at read.

Rolling window (``overflow: 'sinks'``): keys are cached unroped and rotated at read by their
cache slot ``j``: ``k' = k*cos[j, d%half] + rotate_half(k)*sin[j, d%half]``
(``shaders/attention_sg_roll.wgsl:40-51``; q8: ``attention_sg_kv8_roll.wgsl:44-54`` rotates the
dequantised values identically).  Queries arrive already roped at their slot.

Sigmoid output gate (27B hybrid): ``y = att / (1 + exp(-gate))`` (``shaders/gate_sigmoid.wgsl:13``).
"""
import numpy as np

F32 = np.float32


def default_scale(D):
    return F32(1.0) / np.sqrt(F32(D))


def rotate_keys_at_read(K, cosT, sinT, slot0=0):
    """Rotate cached keys ``K[L, KV, D]`` by their slot index ``slot0 + j`` with tables
    ``cosT/sinT[positions, D/2]`` (``attention_sg_roll.wgsl:42-50``)."""
    K = np.asarray(K, F32)
    L, KV, D = K.shape
    half = D // 2
    c = np.asarray(cosT, F32)[slot0:slot0 + L]
    s = np.asarray(sinT, F32)[slot0:slot0 + L]
    cf = np.concatenate([c, c], -1)[:, None, :]
    sf = np.concatenate([s, s], -1)[:, None, :]
    rot = np.concatenate([-K[..., half:], K[..., :half]], -1)
    return (K * cf + rot * sf).astype(F32)


def attend(q, K, V, posBase, scale=None, gate=None):
    """``q[S,H,D]``, ``K,V[L,KV,D]`` (float32 values) -> ``out[S,H,D]`` float32.

    Only cache rows ``0 .. posBase+S-1`` are read (``Ltot = posBase + S``)."""
    q = np.asarray(q, F32)
    S, H, D = q.shape
    KV = K.shape[1]
    G = H // KV
    Ltot = posBase + S
    K = np.asarray(K[:Ltot], F32)
    V = np.asarray(V[:Ltot], F32)
    sc_ = default_scale(D) if scale is None else F32(scale)
    pos = posBase + np.arange(S)
    mask = np.where(np.arange(Ltot)[None, :] <= pos[:, None], F32(0.0), F32(-1e30)).astype(F32)
    out = np.empty((S, H, D), F32)
    for h in range(H):
        kvh = h // G
        sc = (q[:, h] @ K[:, kvh].T) * sc_ + mask          # [S, Ltot]
        sc = sc - sc.max(-1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(-1, keepdims=True)
        out[:, h] = p @ V[:, kvh]
    if gate is not None:
        out = (out / (F32(1.0) + np.exp(-np.asarray(gate, F32)))).astype(F32)
    return out


def attend_partials(q, K, V, posBase, lo, hi, scale=None):
    """Split-KV partial over cache positions ``[lo, hi)``: returns ``(m, l, o)`` per row with
    ``m[S,H]`` the running max of the (scaled) scores, ``l`` the sum of ``exp(score-m)`` and
    ``o[S,H,D]`` the unnormalised ``sum exp(score-m) V``.  Rows with no attended position in
    the range get ``m=-inf, l=0, o=0``."""
    q = np.asarray(q, F32)
    S, H, D = q.shape
    KV = K.shape[1]
    G = H // KV
    sc_ = default_scale(D) if scale is None else F32(scale)
    m = np.full((S, H), -np.inf, F32)
    l = np.zeros((S, H), F32)
    o = np.zeros((S, H, D), F32)
    for qi in range(S):
        last = min(hi, posBase + qi + 1)
        if last <= lo:
            continue
        for h in range(H):
            kvh = h // G
            sc = (np.asarray(K[lo:last, kvh], F32) @ q[qi, h]) * sc_
            mm = sc.max()
            p = np.exp(sc - mm)
            m[qi, h], l[qi, h] = mm, p.sum()
            o[qi, h] = p @ np.asarray(V[lo:last, kvh], F32)
    return m, l, o


def lse_merge(ms, ls, os_, gate=None):
    """Merge split-KV partials (lists over splits) into the normalised output."""
    ms = np.stack(ms)
    ls = np.stack(ls)
    os_ = np.stack(os_)
    M = ms.max(0)
    w = np.where(np.isfinite(ms), np.exp(ms - M[None]), 0.0).astype(F32)
    L = (w * ls).sum(0)
    O = (w[..., None] * os_).sum(0) / L[..., None]
    O = O.astype(F32)
    if gate is not None:
        O = (O / (F32(1.0) + np.exp(-np.asarray(gate, F32)))).astype(F32)
    return O


def attend_rows(q_rows, positions, K, V, scale=None, gate=None):
    """Selected query rows only: ``q_rows[n, D]`` (one head) at absolute positions
    ``positions[n]``, over one kv head's ``K, V[L, D]`` (float32 values).  Row ``i`` attends
    cache positions ``0 .. positions[i]`` -- the same causal rule and softmax as ``attend``
    (``shaders/attention_sg.wgsl:21-44``), restricted to the rows asked for so that parity at
    full prefill sizes (8192 rows x 8192 positions) stays a few matrix products."""
    q = np.asarray(q_rows, F32)
    D = q.shape[-1]
    pos = np.asarray(positions)
    Lmax = int(pos.max()) + 1
    Kf = np.asarray(K[:Lmax], F32)
    Vf = np.asarray(V[:Lmax], F32)
    sc_ = default_scale(D) if scale is None else F32(scale)
    sc = (q @ Kf.T) * sc_
    sc = np.where(np.arange(Lmax)[None, :] <= pos[:, None], sc, F32(-1e30)).astype(F32)
    sc = sc - sc.max(-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(-1, keepdims=True)
    out = (p @ Vf).astype(F32)
    if gate is not None:
        out = (out / (F32(1.0) + np.exp(-np.asarray(gate, F32)))).astype(F32)
    return out
