"""The reference's synthetic Qwen3.5 hybrid model, regenerated (TEST INFRASTRUCTURE ONLY).

``tools/gen-synth-qwen35.py`` seeds ``np.random.seed(1)`` and draws a tiny 1-bit model with the
27B's layer structure (hidden 256, 4 layers with full attention at layer 3, 4 query / 2 kv heads of
dim 256 with 64 rotary dims, 16 key / 48 value linear heads of dim 128, conv width 4, vocabulary
256).  Its golden fixture ``test-fixtures/forward-synth-qwen35/{ids,embed,layer0,finalnorm,
logits}.bin`` is the reference's numpy forward (``tools/qwen35_numpy.py:216-237``, recurrent delta
rule, "tile" head pairing) on the dequantised weights.

``synth_weights`` makes the same draws in the same order and dequantises them the same way, so the
fixture's bytes can be checked against this library's kernels without the reference tree:

* a Q1_0 tensor ``[N, K]`` (``add_q1``, ``:60-75``) draws ``randint(0, 256, (N, K/128*16))`` sign
  bytes, then ``randn(N, K/128) * 0.1`` rounded to f16 block scales; element ``8*i + j`` of a row is
  ``+scale`` when bit ``j`` of sign byte ``i`` is set, else ``-scale`` (the ``tgt2`` table's codes
  3 / 1 minus 2, ``:40-57``), with one scale per 128 elements;
* norms (``add_norm``, ``:87-93``) draw ``randn(n) * 0.1`` and the numpy forward takes them raw
  (it applies ``1 + w`` itself);
* the linear layer's conv ``randn(C, K) * 0.3`` (f32), ``Alog = -exp(randn(H) * 0.5)``,
  ``dt = randn(H) * 0.5``, gated-norm weight ``randn(DV) * 0.1`` (raw, ``:118-126``);
* draw order (``:96-130``): embed, then per layer in_ln, post_ln, gate, up, down, then
  q, k, v, o, q_norm, k_norm (full) or in_qkv, z, b, a, conv, A_log, dt_bias, norm, out_proj
  (linear); then the final norm and lm_head.
* ids: ``RandomState(1234).randint(0, 256, 300)`` (``:150``).

The returned dict uses the key names of ``oracle.hybrid`` / ``qwen35_numpy.forward``.
"""
import numpy as np

from .hybrid import Cfg

F32 = np.float32


def _q1(rs, N, K):
    nb = K // 128
    signs = rs.randint(0, 256, (N, nb * 16), np.uint8)
    scales = (rs.randn(N, nb) * 0.1).astype(np.float16).astype(F32)
    bits = np.unpackbits(signs, axis=1, bitorder="little").astype(F32)      # element 8*i + j <- bit j
    return ((2.0 * bits - 1.0) * scales[:, np.arange(K) // 128]).astype(F32)


def synth_weights():
    cfg = Cfg()
    rs = np.random.RandomState(1)
    H, I = cfg.hidden, cfg.inter
    W = {"embed": _q1(rs, cfg.vocab, H), "layers": []}
    for li in range(cfg.n_layers):
        d = {"type": cfg.layer_type(li)}
        d["in_ln"] = (rs.randn(H) * 0.1).astype(F32)
        d["post_ln"] = (rs.randn(H) * 0.1).astype(F32)
        d["gate"], d["up"], d["down"] = _q1(rs, I, H), _q1(rs, I, H), _q1(rs, H, I)
        if d["type"] == "full_attention":
            hd = cfg.head_dim
            d["q"] = _q1(rs, cfg.n_heads * hd * 2, H)
            d["k"] = _q1(rs, cfg.n_kv_heads * hd, H)
            d["v"] = _q1(rs, cfg.n_kv_heads * hd, H)
            d["o"] = _q1(rs, H, cfg.n_heads * hd)
            d["qn"] = (rs.randn(hd) * 0.1).astype(F32)
            d["kn"] = (rs.randn(hd) * 0.1).astype(F32)
        else:
            nv = cfg.n_v_heads
            d["qkv"] = _q1(rs, cfg.conv_dim, H)
            d["z"] = _q1(rs, cfg.value_dim, H)
            d["pb"] = _q1(rs, nv, H)
            d["pa"] = _q1(rs, nv, H)
            d["conv"] = (rs.randn(cfg.conv_dim, cfg.conv_k).astype(F32) * F32(0.3))[:, None, :]
            d["Alog"] = (-np.exp(rs.randn(nv) * 0.5)).astype(F32)
            d["dt"] = (rs.randn(nv) * 0.5).astype(F32)
            d["gn"] = (rs.randn(cfg.v_dim) * 0.1).astype(F32)
            d["out"] = _q1(rs, H, cfg.value_dim)
        W["layers"].append(d)
    W["final_norm"] = (rs.randn(H) * 0.1).astype(F32)
    W["lm_head"] = _q1(rs, cfg.vocab, H)
    return cfg, W


def synth_ids():
    return np.random.RandomState(1234).randint(0, 256, 300).astype(np.int32)
