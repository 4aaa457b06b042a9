#!/usr/bin/env python3
"""Regenerate the golden fixtures in this folder from the reference's own numpy code.

Run only where the reference checkout exists (it is read-only and never needed at test time):

    python tests/golden/make_golden.py /path/to/bitgpu

It (1) runs the reference's ``tools/gen-kernel-cases.py`` (seeded ``np.random.seed(0)``) into a
temporary folder and stores each case's inputs / expected outputs as float32 ``.npz``;
(2) calls ``tools/qwen35_numpy.py`` directly for larger delta-rule cases (recurrent and
chunked) and for gated / plain causal attention at head_dim 256 and 128 (through
``_full_attention`` with an identity hidden state and identity output projection, so the
expected array is exactly the gated attention output the kernels must produce); (3) runs the
reference's q/k prologue functions and its whole hybrid ``forward`` on seeded dense weights
(``oracle.hybrid.synth_weights``) for the end-to-end check; (4) copies the reference's own
fixture of its synthetic 1-bit hybrid model (``test-fixtures/forward-synth-qwen35``).
"""
import glob
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref):
    tools = os.path.join(ref, "tools")
    sys.path.insert(0, tools)
    import qwen35_numpy as qn  # the reference's own oracle

    # (1) the reference's per-kernel cases, bit-identical to its generator
    with tempfile.TemporaryDirectory() as td:
        subprocess.check_call([sys.executable, os.path.join(tools, "gen-kernel-cases.py"), td])
        for fn in sorted(glob.glob(os.path.join(td, "*.json"))):
            c = json.load(open(fn))
            arrs = {f"in{i}": np.asarray(a, np.float32) for i, a in enumerate(c["inputs"])}
            arrs["expected"] = np.asarray(c["expected"], np.float32)
            arrs["params"] = np.asarray([p[1] for p in c["params"]], np.float64)
            np.savez_compressed(os.path.join(HERE, f"kc_{c['name']}.npz"), **arrs)
            print("wrote", f"kc_{c['name']}.npz")

    rng = np.random.default_rng(20260701)

    # (2a) delta rule, recurrent and chunked, GQA tile pairing, non-multiple-of-64 length
    S, HK, H, DK, DV = 70, 2, 4, 128, 128
    q = rng.standard_normal((S, HK, DK)).astype(np.float32)
    k = rng.standard_normal((S, HK, DK)).astype(np.float32)
    v = rng.standard_normal((S, H, DV)).astype(np.float32)
    g = (-np.logaddexp(0.0, rng.standard_normal((S, H)))).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((S, H))))).astype(np.float32)
    C = qn.Qwen35Cfg(hidden=0, n_layers=0, eps=1e-6, n_heads=0, n_kv_heads=0, head_dim=0, rot_dim=0,
                     rope_theta=1e7, n_k_heads=HK, n_v_heads=H, k_dim=DK, v_dim=DV, conv_kernel=4)
    rep = H // HK
    qt, kt = np.tile(q, (1, rep, 1)), np.tile(k, (1, rep, 1))
    rec = qn._delta_recurrent(qt, kt, v, g, beta, C)
    chk = qn._delta_chunk(qt, kt, v, g, beta, C)
    np.savez_compressed(os.path.join(HERE, "dn_delta_s70.npz"), q=q, k=k, v=v, g=g, beta=beta,
                        recurrent=rec, chunk=chk)
    print("wrote dn_delta_s70.npz")

    # (2b) gated causal attention through the reference _full_attention
    def gated_case(name, S, H, KV, HD, rot, theta, gate_bias):
        Cg = qn.Qwen35Cfg(hidden=S, n_layers=0, eps=1e-6, n_heads=H, n_kv_heads=KV, head_dim=HD, rot_dim=rot,
                          rope_theta=theta, n_k_heads=1, n_v_heads=1, k_dim=1, v_dim=1, conv_kernel=4)
        qg = rng.standard_normal((S, H, 2 * HD)).astype(np.float32)
        qg[..., HD:] += gate_bias
        kraw = rng.standard_normal((S, KV, HD)).astype(np.float32)
        vraw = rng.standard_normal((S, KV, HD)).astype(np.float32)
        d = {"q": qg.reshape(S, -1).T.copy(), "k": kraw.reshape(S, -1).T.copy(), "v": vraw.reshape(S, -1).T.copy(),
             "qn": (0.1 * rng.standard_normal(HD)).astype(np.float32),
             "kn": (0.1 * rng.standard_normal(HD)).astype(np.float32),
             "o": np.eye(H * HD, dtype=np.float32)}
        x = np.eye(S, dtype=np.float32)
        cos, sin = qn._rope_tables(Cg, S)
        out = qn._full_attention(x, d, Cg, cos, sin).reshape(S, H, HD)
        # the kernels' inputs: roped/normed q and k exactly as _full_attention forms them
        qin = qn._rope_partial(qn.rmsnorm(qg[..., :HD], d["qn"], Cg.eps), cos, sin, rot)
        kin = qn._rope_partial(qn.rmsnorm(kraw, d["kn"], Cg.eps), cos, sin, rot)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), q=qin, k=kin, v=vraw,
                            gate=qg[..., HD:].copy(), expected=out.astype(np.float32))
        print("wrote", f"{name}.npz")

    gated_case("ga_d256_gated", S=13, H=6, KV=2, HD=256, rot=64, theta=1e7, gate_bias=0.0)
    # gate bias +100 makes sigmoid(gate) == 1.0 exactly in f32: plain causal GQA attention, D=128
    gated_case("ga_d128_plain", S=11, H=8, KV=4, HD=128, rot=128, theta=1e6, gate_bias=100.0)


    # (2c) the fused q/k prologue: split_head -> rmsnorm (1 + w) -> rope_partial, through the
    # reference's own rmsnorm / _rope_partial (engine.ts:1471-1485 dispatches them separately)
    S, H, HD, ROT = 7, 3, 256, 64
    Cp = qn.Qwen35Cfg(hidden=0, n_layers=0, eps=1e-6, n_heads=H, n_kv_heads=H, head_dim=HD, rot_dim=ROT,
                      rope_theta=1e7, n_k_heads=1, n_v_heads=1, k_dim=1, v_dim=1, conv_kernel=4)
    qg = rng.standard_normal((S, H, 2 * HD)).astype(np.float32)
    wq = (0.1 * rng.standard_normal(HD)).astype(np.float32)
    cos, sin = qn._rope_tables(Cp, S)
    exp_q = qn._rope_partial(qn.rmsnorm(qg[..., :HD], wq, Cp.eps), cos, sin, ROT)
    np.savez_compressed(os.path.join(HERE, "kc_qk_prologue.npz"), qg=qg, w=wq, cos=cos, sin=sin,
                        expected=exp_q.astype(np.float32), gate=qg[..., HD:].copy())
    print("wrote kc_qk_prologue.npz")

    # (2d) end to end: the reference's numpy hybrid forward (tools/qwen35_numpy.py:216-237,
    # "tile" value-head pairing as in the engine) on seeded dense weights with the synthetic
    # model's dimensions (oracle.hybrid.synth_weights draws them; the test redraws the same).
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle import hybrid as HY
    cfg = HY.Cfg()
    seed, S = 7, 300
    W = HY.synth_weights(cfg, seed)
    ids = np.random.default_rng(11).integers(0, cfg.vocab, S).astype(np.int32)
    Cf = qn.Qwen35Cfg(hidden=cfg.hidden, n_layers=cfg.n_layers, eps=cfg.eps, n_heads=cfg.n_heads,
                      n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, rot_dim=cfg.rot_dim, rope_theta=cfg.theta,
                      n_k_heads=cfg.n_k_heads, n_v_heads=cfg.n_v_heads, k_dim=cfg.k_dim, v_dim=cfg.v_dim,
                      conv_kernel=cfg.conv_k)
    ref = qn.forward(W, Cf, ids, delta="chunk", repeat="tile")
    np.savez_compressed(os.path.join(HERE, "hy_forward_s300.npz"), seed=np.int64(seed), ids=ids,
                        logits_tail=ref["logits"][-16:].astype(np.float32),
                        argmax=ref["logits"].argmax(-1).astype(np.int32),
                        last_hidden=np.stack([h[-1] for h in ref["layers"]]).astype(np.float32))
    print("wrote hy_forward_s300.npz")

    # (2e) the reference's own end-to-end fixture for its synthetic 1-bit hybrid model
    # (test-fixtures/forward-synth-qwen35, written by tools/gen-synth-qwen35.py with the reference's
    # numpy forward): copied byte for byte.  oracle.synth_qwen35 regenerates the weights.
    fx = os.path.join(os.path.dirname(tools), "test-fixtures", "forward-synth-qwen35")
    prm = json.load(open(os.path.join(fx, "params.json")))
    S, Hd, V = prm["S"], prm["hidden"], prm["vocab"]
    rd = lambda n, *shape: np.fromfile(os.path.join(fx, n), np.float32).reshape(shape)
    np.savez_compressed(os.path.join(HERE, "synth_qwen35_fixture.npz"),
                        ids=np.fromfile(os.path.join(fx, "ids.i32.bin"), np.int32),
                        logits=rd("logits.bin", S, V), layer0=rd("layer0.bin", S, Hd),
                        embed_tail=rd("embed.bin", S, Hd)[-32:], argmax_last=np.int64(prm["argmax_last"]))
    print("wrote synth_qwen35_fixture.npz")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path of the bitgpu source tree>")
    main(sys.argv[1])
