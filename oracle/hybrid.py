"""Qwen3.5 hybrid text forward -- CPU restatement (TEST INFRASTRUCTURE ONLY).

Restates ``tools/qwen35_numpy.py:216-237`` (``forward``) with its token mixers: the gated
DeltaNet layer (``:190-213``: in_qkv projection, causal conv1d + SiLU, q|k|v split, g/beta,
chunked delta rule with "tile" GQA pairing, gated RMSNorm, out projection) and the gated
full-attention layer (``:92-115``: doubled q_proj into query | gate, q/k RMSNorm with the
(1 + weight) scale, partial RoPE, causal GQA softmax attention, sigmoid gate, o_proj); each layer
adds the SwiGLU MLP.  The projections are dense f32 matrices here: the reference's 1-bit GEMVs
are outside the attention hot path, so an end-to-end check feeds identical dense weights to this
restatement, to the reference's numpy forward (fixtures) and to the CUDA mixer kernels.

``synth_weights`` draws a seeded random model with the dimensions of the reference's synthetic
hybrid model (``tools/gen-synth-qwen35.py:27-43``: hidden 256, 4 layers with full attention at
layer 3, 4 query / 2 kv heads of dim 256 with rotary dims 64, 16 key / 48 value heads of dim 128,
conv width 4, vocabulary 256).
"""
from dataclasses import dataclass

import numpy as np

from . import deltanet as DN
from . import glue as GL

F32 = np.float32


@dataclass
class Cfg:
    hidden: int = 256
    n_layers: int = 4
    full_every: int = 4         # layer i is full attention when (i + 1) % full_every == 0
    inter: int = 512
    n_heads: int = 4
    n_kv_heads: int = 2
    head_dim: int = 256
    rot_dim: int = 64
    n_k_heads: int = 16
    n_v_heads: int = 48
    k_dim: int = 128
    v_dim: int = 128
    conv_k: int = 4
    vocab: int = 256
    eps: float = 1e-6
    theta: float = 1e6

    @property
    def key_dim(self):
        return self.n_k_heads * self.k_dim

    @property
    def value_dim(self):
        return self.n_v_heads * self.v_dim

    @property
    def conv_dim(self):
        return 2 * self.key_dim + self.value_dim

    def layer_type(self, i):
        return "full_attention" if (i + 1) % self.full_every == 0 else "linear_attention"


def synth_weights(cfg: Cfg, seed: int):
    """Seeded dense weights; matrices are [out, in] with N(0, 1/in) entries, norms 0-centred."""
    rng = np.random.default_rng(seed)

    def mat(o, i):
        return (rng.standard_normal((o, i)) / np.sqrt(i)).astype(F32)

    def vec(n, s=0.1):
        return (s * rng.standard_normal(n)).astype(F32)

    W = {"embed": rng.standard_normal((cfg.vocab, cfg.hidden)).astype(F32),
         "final_norm": vec(cfg.hidden), "lm_head": mat(cfg.vocab, cfg.hidden), "layers": []}
    H = cfg.hidden
    for i in range(cfg.n_layers):
        d = {"type": cfg.layer_type(i), "in_ln": vec(H), "post_ln": vec(H),
             "gate": mat(cfg.inter, H), "up": mat(cfg.inter, H), "down": mat(H, cfg.inter)}
        if d["type"] == "full_attention":
            hd = cfg.head_dim
            d.update(q=mat(cfg.n_heads * hd * 2, H), k=mat(cfg.n_kv_heads * hd, H), v=mat(cfg.n_kv_heads * hd, H),
                     o=mat(H, cfg.n_heads * hd), qn=vec(hd), kn=vec(hd))
        else:
            nv = cfg.n_v_heads
            d.update(qkv=mat(cfg.conv_dim, H),
                     conv=(0.5 * rng.standard_normal((cfg.conv_dim, 1, cfg.conv_k))).astype(F32),
                     z=mat(cfg.value_dim, H), pb=mat(nv, H), pa=mat(nv, H),
                     Alog=(-np.exp(rng.uniform(-1.0, 1.0, nv))).astype(F32), dt=vec(nv, 0.5),
                     gn=(1.0 + vec(cfg.v_dim)).astype(F32), out=mat(H, cfg.value_dim))
        W["layers"].append(d)
    return W


def _rms(x, g, eps):
    return GL.rmsnorm(x, F32(1.0) + g, eps)


def linear_mixer(x, d, cfg: Cfg):
    S = x.shape[0]
    mixed, _ = GL.conv1d_causal(x @ d["qkv"].T, d["conv"][:, 0, :])
    KD = cfg.key_dim
    q = mixed[:, :KD].reshape(S, cfg.n_k_heads, cfg.k_dim)
    k = mixed[:, KD:2 * KD].reshape(S, cfg.n_k_heads, cfg.k_dim)
    v = mixed[:, 2 * KD:].reshape(S, cfg.n_v_heads, cfg.v_dim)
    a = x @ d["pa"].T
    b = x @ d["pb"].T
    g, beta = DN.gbeta(a, b, d["Alog"], d["dt"])
    core, _ = DN.chunk(q, k, v, g, beta)
    z = (x @ d["z"].T).reshape(S * cfg.n_v_heads, cfg.v_dim)
    normed = DN.norm_gate(core.reshape(S * cfg.n_v_heads, cfg.v_dim), z, d["gn"], cfg.eps)
    return normed.reshape(S, cfg.value_dim) @ d["out"].T


def full_mixer(x, d, cfg: Cfg, cos, sin):
    S, H, KV, hd = x.shape[0], cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    qg = x @ d["q"].T
    q = GL.qk_norm_rope(qg, H, hd, 2 * hd, 0, F32(1.0) + d["qn"], cos, sin, cfg.rot_dim, cfg.eps)
    gate = GL.slice_cols(qg, S * H, hd, 2 * hd, hd).reshape(S, H, hd)
    k = GL.qk_norm_rope(x @ d["k"].T, KV, hd, hd, 0, F32(1.0) + d["kn"], cos, sin, cfg.rot_dim, cfg.eps)
    v = (x @ d["v"].T).reshape(S, KV, hd)
    rep = H // KV
    o = np.empty((S, H, hd), F32)
    causal = np.triu(np.full((S, S), -np.inf, F32), 1)
    for h in range(H):
        sc = (q[:, h] @ k[:, h // rep].T) * F32(1.0 / np.sqrt(hd)) + causal
        w = np.exp(sc - sc.max(-1, keepdims=True))
        o[:, h] = (w / w.sum(-1, keepdims=True)) @ v[:, h // rep]
    o = o * DN.sigmoid(gate)
    return o.reshape(S, H * hd) @ d["o"].T


def forward(W, cfg: Cfg, ids):
    """Returns {'layers': [hidden after each layer], 'logits': [S, vocab]}."""
    ids = np.asarray(ids)
    S = len(ids)
    cos, sin = GL.rope_tables(S, cfg.rot_dim, cfg.theta)
    h = W["embed"][ids].astype(F32)
    out = {"layers": []}
    for d in W["layers"]:
        x = _rms(h, d["in_ln"], cfg.eps)
        mix = full_mixer(x, d, cfg, cos, sin) if d["type"] == "full_attention" else linear_mixer(x, d, cfg)
        h = (h + mix).astype(F32)
        x = _rms(h, d["post_ln"], cfg.eps)
        h = (h + (DN.silu(x @ d["gate"].T) * (x @ d["up"].T)) @ d["down"].T).astype(F32)
        out["layers"].append(h.copy())
    out["logits"] = _rms(h, W["final_norm"], cfg.eps) @ W["lm_head"].T
    return out

