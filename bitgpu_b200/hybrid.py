"""Token mixers of the Qwen3.5 hybrid layer, wired through the C ABI the way the reference
engine dispatches them (``src/engine.ts:1404-1491``, ``hybridLayer``).

The hot-path steps run on this library's kernels: causal conv1d with its carried state, the
q|k|v column split, the chunked (prefill) or recurrent (decode) gated delta rule with fused
g/beta and gated RMSNorm, the fused split_head + q/k RMSNorm + partial RoPE (+ K cache write),
the V append and the gated attention.  The dense projections (the reference's 1-bit GEMVs) are
outside this library's scope and run as plain torch matmuls here.

State carried between calls, as in the engine: the conv left context ``[K-1, conv_dim]``
(``hyCS``), the DeltaNet state ``[H, DK, DV]`` (``hyRS``) and the layer's KV cache.
"""
import torch

from . import ops


def rope_tables(positions, rot, theta, device="cuda"):
    """[positions, rot] cos/sin of the partial rotary (angles in float64, rounded once to
    float32, duplicated halves), the layout rope_partial.wgsl reads (engine.ts:117-147)."""
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.float64) / rot))
    frq = torch.outer(torch.arange(positions, dtype=torch.float64), inv)
    emb = torch.cat([frq, frq], -1)
    return emb.cos().float().to(device), emb.sin().float().to(device)


class LinearMixer:
    """Gated-DeltaNet token mixer (engine.ts:1411-1458).  ``w``: dict of float32 CUDA tensors
    qkv [conv_dim, hidden], conv [conv_dim, K], z [value_dim, hidden], pa/pb [H, hidden],
    a_neg/dt_bias [H], gamma [DV], out [hidden, value_dim]."""

    CHUNKED_MIN = 64  # segments at least one chunk long use the chunked kernels

    def __init__(self, w, n_k_heads, n_v_heads, k_dim, v_dim, eps):
        self.w, self.HK, self.H, self.DK, self.DV, self.eps = w, n_k_heads, n_v_heads, k_dim, v_dim, eps
        self.conv_state = None  # [K-1, conv_dim]
        self.state = None       # [H, DK, DV]

    def __call__(self, x):
        w, S = self.w, x.shape[0]
        KD, VD = self.HK * self.DK, self.H * self.DV
        cd = 2 * KD + VD
        mixed = x @ w["qkv"].T
        conv, self.conv_state = ops.conv1d_causal(mixed, w["conv"], self.conv_state)
        q = ops.slice_cols(conv, S, KD, cd, 0).view(S, self.HK, self.DK)
        k = ops.slice_cols(conv, S, KD, cd, KD).view(S, self.HK, self.DK)
        v = ops.slice_cols(conv, S, VD, cd, 2 * KD).view(S, self.H, self.DV)
        a = (x @ w["pa"].T).contiguous()
        b = (x @ w["pb"].T).contiguous()
        z = (x @ w["z"].T).contiguous().view(S, self.H, self.DV)
        if S >= self.CHUNKED_MIN:
            y, self.state, _ = ops.deltanet_chunked(q, k, v, a, b, w["a_neg"], w["dt_bias"], z, w["gamma"], self.eps,
                                                    state_in=self.state)
        else:
            y, self.state = ops.deltanet_fused(q, k, v, a, b, w["a_neg"], w["dt_bias"], z, w["gamma"], self.eps,
                                               state_in=self.state)[:2]
        return y.view(S, VD) @ w["out"].T


class FullMixer:
    """Gated full-attention token mixer (engine.ts:1459-1491).  ``w``: q [2*H*hd, hidden],
    k/v [KV*hd, hidden], o [hidden, H*hd], q_gamma/k_gamma [hd] (the baked 1 + weight)."""

    def __init__(self, w, n_heads, n_kv_heads, head_dim, rot_dim, eps, capacity, mode="f32"):
        self.w, self.H, self.KV, self.hd, self.rot, self.eps = w, n_heads, n_kv_heads, head_dim, rot_dim, eps
        self.cache = ops.KVCache(1, capacity, n_kv_heads, head_dim, mode=mode, device=w["q"].device)

    def __call__(self, x, pos0, cos, sin):
        """x [S, hidden] at positions pos0 .. pos0+S-1; cos/sin [positions, rot] (row = position)."""
        w, S, H, KV, hd = self.w, x.shape[0], self.H, self.KV, self.hd
        qg = x @ w["q"].T                                                  # [S, H, 2*hd]
        q = ops.qk_norm_rope(qg, 1, S, H, hd, 2 * hd, 0, w["q_gamma"], cos, sin, self.rot, pos0, self.eps)
        gate = ops.slice_cols(qg, S * H, hd, 2 * hd, hd).view(1, S, H, hd)
        kk = x @ w["k"].T
        ops.qk_norm_rope(kk, 1, S, KV, hd, hd, 0, w["k_gamma"], cos, sin, self.rot, pos0, self.eps,
                         cache=self.cache, want_y=False)
        self.cache.append(1, (x @ w["v"].T).view(1, S, KV, hd).contiguous(), pos0)
        att = ops.attention(q, self.cache, pos0, scale=1.0 / hd ** 0.5, gate=gate)
        return att.view(S, H * hd) @ w["o"].T
