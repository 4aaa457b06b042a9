"""End-to-end: the Qwen3.5 hybrid forward with this library's token-mixer kernels against the
reference's numpy forward on the same seeded dense weights (fixture ``hy_forward_s300.npz``,
made by ``tests/golden/make_golden.py`` from ``tools/qwen35_numpy.py``).  Embedding, RMSNorms,
MLP and lm_head are plain torch here (outside the hot path); every token-mixer step runs on
the CUDA kernels through the C ABI."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import hybrid as HY

pytestmark = pytest.mark.gpu


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


class Model:
    def __init__(self, W, cfg, mode="f32", capacity=512):
        from bitgpu_b200 import hybrid
        self.cfg, self.W = cfg, W
        self.cos, self.sin = hybrid.rope_tables(capacity, cfg.rot_dim, cfg.theta)
        self.embed, self.fn, self.lm = t(W["embed"]), t(W["final_norm"]), t(W["lm_head"])
        self.layers = []
        for d in W["layers"]:
            mlp = {k: t(d[k]) for k in ("gate", "up", "down")}
            lns = (t(d["in_ln"]), t(d["post_ln"]))
            if d["type"] == "full_attention":
                mix = hybrid.FullMixer({"q": t(d["q"]), "k": t(d["k"]), "v": t(d["v"]), "o": t(d["o"]),
                                        "q_gamma": t(1.0 + d["qn"]), "k_gamma": t(1.0 + d["kn"])},
                                       cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.rot_dim, cfg.eps, capacity, mode)
            else:
                mix = hybrid.LinearMixer({"qkv": t(d["qkv"]), "conv": t(d["conv"][:, 0, :]), "z": t(d["z"]),
                                          "pa": t(d["pa"]), "pb": t(d["pb"]), "a_neg": t(d["Alog"]),
                                          "dt_bias": t(d["dt"]), "gamma": t(d["gn"]), "out": t(d["out"])},
                                         cfg.n_k_heads, cfg.n_v_heads, cfg.k_dim, cfg.v_dim, cfg.eps)
            self.layers.append((d["type"], mix, lns, mlp))
        self.pos = 0

    def rms(self, x, g):
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + self.cfg.eps) * (1.0 + g)

    def __call__(self, ids):
        h = self.embed[torch.as_tensor(np.asarray(ids, np.int64), device="cuda")]
        last = []
        for typ, mix, (ln1, ln2), mlp in self.layers:
            x = self.rms(h, ln1).contiguous()
            h = h + (mix(x, self.pos, self.cos, self.sin) if typ == "full_attention" else mix(x))
            x = self.rms(h, ln2)
            h = h + (torch.nn.functional.silu(x @ mlp["gate"].T) * (x @ mlp["up"].T)) @ mlp["down"].T
            last.append(h[-1].clone())
        self.pos += len(ids)
        return self.rms(h, self.fn) @ self.lm.T, torch.stack(last)


@pytest.fixture(scope="module")
def case():
    z = np.load(os.path.join(GOLDEN, "hy_forward_s300.npz"))
    cfg = HY.Cfg()
    return z, cfg, HY.synth_weights(cfg, int(z["seed"]))


def test_hybrid_prefill_matches_reference(case):
    z, cfg, W = case
    logits, last = Model(W, cfg)(z["ids"])
    lg = logits.cpu().numpy()
    err = np.abs(lg[-16:] - z["logits_tail"]).max()
    assert err < 2e-3 * max(1.0, np.abs(z["logits_tail"]).max()), err
    agree = (lg.argmax(-1) == z["argmax"]).mean()
    assert agree >= 0.99 and lg[-1].argmax() == z["argmax"][-1], agree
    assert np.abs(last.cpu().numpy() - z["last_hidden"]).max() < 2e-3


@pytest.mark.parametrize("cuts", [[200, 100], [150, 146, 1, 1, 1, 1]])
def test_hybrid_segmented_and_decode(case, cuts):
    """Segmented prefill (chunked scan, carried conv / DeltaNet state, growing KV cache) and
    token-by-token decode (recurrent scan) give the full-prefill logits of the last token."""
    z, cfg, W = case
    ids = z["ids"]
    m = Model(W, cfg)
    off = 0
    for n in cuts:
        logits, last = m(ids[off:off + n])
        off += n
    err = np.abs(logits[-1].cpu().numpy() - z["logits_tail"][-1]).max()
    assert err < 2e-3 * max(1.0, np.abs(z["logits_tail"]).max()), err
    assert np.abs(last.cpu().numpy() - z["last_hidden"]).max() < 2e-3


def test_hybrid_q8_cache(case):
    """The full-attention layer on a q8 KV cache (the 27B's 8-bit cache): same argmax."""
    z, cfg, W = case
    logits, _ = Model(W, cfg, mode="q8")(z["ids"])
    lg = logits.cpu().numpy()
    assert (lg.argmax(-1) == z["argmax"]).mean() >= 0.97
    assert np.abs(lg[-16:] - z["logits_tail"]).max() < 0.05 * max(1.0, np.abs(z["logits_tail"]).max())


def test_synth_qwen35_reference_fixture():
    """The reference's own end-to-end fixture (test-fixtures/forward-synth-qwen35: its synthetic
    1-bit hybrid model, seed 1, through its numpy forward): the 4-layer forward with this
    library's token-mixer kernels on the same dequantised weights gives the fixture's logits
    (max|d| < 5e-3, cos > 0.9999) and its greedy token argmax_last = 201
    (scripts/verify-hybrid.mjs:146-161)."""
    from oracle import synth_qwen35 as SQ
    z = np.load(os.path.join(GOLDEN, "synth_qwen35_fixture.npz"))
    cfg, W = SQ.synth_weights()
    logits, _ = Model(W, cfg)(z["ids"])
    lg = logits.cpu().numpy()
    ref = z["logits"]
    err = float(np.abs(lg - ref).max())
    cos = float((lg * ref).sum() / (np.linalg.norm(lg) * np.linalg.norm(ref)))
    assert err < 5e-3 and cos > 0.9999, (err, cos)
    assert int(lg[-1].argmax()) == int(z["argmax_last"]) == 201
    assert (lg.argmax(-1) == ref.argmax(-1)).all()
