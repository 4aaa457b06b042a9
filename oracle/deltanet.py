"""Gated DeltaNet (Qwen3.5 linear attention) -- CPU restatement of the reference numpy.

* ``gbeta``: ``g = a_neg[h] * softplus(a + dt_bias[h])`` with the stable softplus
  ``max(x,0) + log(1+exp(-|x|))``, ``beta = sigmoid(b)``; output ``[g (S*H); beta (S*H)]``
  (``shaders/deltanet_gbeta.wgsl:15-25``; ``tools/qwen35_numpy.py:198-199``).
* ``recurrent``: per value head ``h`` with shared key head ``hk = h % HK`` ("tile" GQA,
  ``shaders/deltanet_recur.wgsl:27``), per token ``S *= exp(g); kv = Kn.S;
  delta = (v - kv)*beta; S += Kn (x) delta; o = Qn.S`` with ``Kn = l2norm(k)``,
  ``Qn = l2norm(q)/sqrt(DK)``, ``l2norm(x) = x / sqrt(sum x^2 + 1e-6)``
  (``tools/qwen35_numpy.py:66-68,128-141``; ``deltanet_recur.wgsl:35-58``).  State layout
  ``[H, DK, DV]`` (``deltanet_recur.wgsl:30``); ``state_in`` continues a previous segment.
* ``chunk``: the chunk-parallel WY form (``tools/qwen35_numpy.py:144-187``), equal to the
  recurrence up to float32 accumulation order.
* ``norm_gate``: ``y = gamma * core / sqrt(mean(core^2) + eps) * silu(z)`` with the raw
  weight (``shaders/deltanet_norm_gate.wgsl:19-31``; ``tools/qwen35_numpy.py:212``).
"""
import numpy as np

F32 = np.float32


def sigmoid(x):
    return (F32(1.0) / (F32(1.0) + np.exp(-np.asarray(x, F32)))).astype(F32)


def silu(x):
    x = np.asarray(x, F32)
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def softplus(x):
    x = np.asarray(x, F32)
    return (np.maximum(x, F32(0.0)) + np.log(F32(1.0) + np.exp(-np.abs(x)))).astype(F32)


def l2norm(x, eps=1e-6):
    x = np.asarray(x, F32)
    return (x * (F32(1.0) / np.sqrt((x * x).sum(-1, keepdims=True) + F32(eps)))).astype(F32)


def gbeta(a, b, a_neg, dt_bias):
    """a, b ``[S, H]``; a_neg, dt_bias ``[H]`` -> ``(g, beta)`` each ``[S, H]``."""
    a = np.asarray(a, F32)
    g = (np.asarray(a_neg, F32)[None, :] * softplus(a + np.asarray(dt_bias, F32)[None, :])).astype(F32)
    return g, sigmoid(b)


def expand_tile(x, H):
    """Key/query heads ``[S, HK, DK]`` -> per value head ``[S, H, DK]`` with ``h -> h % HK``."""
    HK = x.shape[1]
    return np.tile(np.asarray(x, F32), (1, H // HK, 1))


def recurrent(q, k, v, g, beta, state_in=None):
    """q, k ``[S, HK, DK]``; v ``[S, H, DV]``; g, beta ``[S, H]``.
    Returns ``(core [S, H, DV], state_out [H, DK, DV])``."""
    v = np.asarray(v, F32)
    S, H, DV = v.shape
    DK = q.shape[-1]
    qn = expand_tile(l2norm(q), H) * F32(1.0 / np.sqrt(DK))
    kn = expand_tile(l2norm(k), H)
    st = np.zeros((H, DK, DV), F32) if state_in is None else np.asarray(state_in, F32).reshape(H, DK, DV).copy()
    o = np.empty((S, H, DV), F32)
    g = np.asarray(g, F32)
    beta = np.asarray(beta, F32)
    for t in range(S):
        st = st * np.exp(g[t])[:, None, None]
        kv = (st * kn[t][:, :, None]).sum(1)
        delta = (v[t] - kv) * beta[t][:, None]
        st = st + kn[t][:, :, None] * delta[:, None, :]
        o[t] = (st * qn[t][:, :, None]).sum(1)
    return o.astype(F32), st.astype(F32)


def chunk(q, k, v, g, beta, chunk_size=64, state_in=None):
    """Chunk-parallel WY gated delta rule (``tools/qwen35_numpy.py:144-187``), extended with
    an optional initial state (the reference starts from zero).  Returns ``(core, state)``."""
    v = np.asarray(v, F32)
    S, H, DV = v.shape
    DK = q.shape[-1]
    C = chunk_size
    qh = np.transpose(expand_tile(l2norm(q), H), (1, 0, 2)).astype(F32)
    kh = np.transpose(expand_tile(l2norm(k), H), (1, 0, 2)).astype(F32)
    vh = np.transpose(v, (1, 0, 2)).astype(F32)
    bh = np.transpose(np.asarray(beta, F32), (1, 0))
    gh = np.transpose(np.asarray(g, F32), (1, 0))
    pad = (C - S % C) % C
    padv = lambda x: np.pad(x, [(0, 0), (0, pad)] + [(0, 0)] * (x.ndim - 2))
    qh = padv(qh) * F32(1.0 / np.sqrt(DK))
    kh, vh = padv(kh), padv(vh)
    bh, gh = np.pad(bh, [(0, 0), (0, pad)]), np.pad(gh, [(0, 0), (0, pad)])
    vb, kb = vh * bh[..., None], kh * bh[..., None]
    nc = (S + pad) // C
    rs = lambda x: x.reshape(H, nc, C, x.shape[-1])
    qh, kh, vh, kb, vb = rs(qh), rs(kh), rs(vh), rs(kb), rs(vb)
    gh = np.cumsum(gh.reshape(H, nc, C), -1)
    tri0 = np.triu(np.ones((C, C), bool), 0)
    diff = gh[..., :, None] - gh[..., None, :]
    dmask = np.tril(np.exp(np.tril(diff)))
    attn = np.where(tri0, 0.0, -((kb @ np.swapaxes(kh, -1, -2)) * dmask))
    for i in range(1, C):
        row = attn[..., i, :i].copy()
        sub = attn[..., :i, :i].copy()
        attn[..., i, :i] = row + (row[..., None] * sub).sum(-2)
    attn = attn + np.eye(C, dtype=attn.dtype)
    u = attn @ vb
    k_cumdecay = attn @ (kb * np.exp(gh)[..., None])
    st = np.zeros((H, DK, DV), F32) if state_in is None else np.asarray(state_in, F32).reshape(H, DK, DV).copy()
    o = np.zeros((H, nc, C, DV), F32)
    for i in range(nc):
        qi, ki, ui = qh[:, i], kh[:, i], u[:, i]
        a_intra = (qi @ np.swapaxes(ki, -1, -2)) * dmask[:, i]
        v_new = ui - k_cumdecay[:, i] @ st
        a_inter = (qi * np.exp(gh[:, i])[..., None]) @ st
        o[:, i] = a_inter + a_intra @ v_new
        glast = gh[:, i, -1]
        st = st * np.exp(glast)[:, None, None] + \
            np.swapaxes(ki * np.exp(glast[:, None] - gh[:, i])[..., None], -1, -2) @ v_new
    o = o.reshape(H, nc * C, DV)[:, :S]
    return np.transpose(o, (1, 0, 2)).astype(F32), st.astype(F32)


def norm_gate(core, z, gamma, eps):
    """core, z ``[rows, DV]``; gamma ``[DV]``."""
    c = np.asarray(core, F32)
    inv = F32(1.0) / np.sqrt((c * c).mean(-1, keepdims=True) + F32(eps))
    return (np.asarray(gamma, F32) * (c * inv) * silu(z)).astype(F32)
