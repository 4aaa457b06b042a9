"""Pin the CPU oracle against golden vectors made by the reference's own numpy code."""
import os

import numpy as np

from conftest import GOLDEN, close
from oracle import attention, deltanet, evict, kvcodec, rope


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_kc_attention_d256():
    z = load("kc_attention.npz")
    S, H, KV, D = [int(x) for x in z["params"][:4]]
    scale = float(z["params"][4])
    q = z["in0"].reshape(S, H, D)
    k = z["in1"].reshape(S, KV, D)
    v = z["in2"].reshape(S, KV, D)
    out = attention.attend(q, k, v, posBase=0, scale=scale)
    ok, mad, cos = close(out, z["expected"], tol=1e-5)
    assert ok, (mad, cos)


def test_gated_attention_d256():
    z = load("ga_d256_gated.npz")
    out = attention.attend(z["q"], z["k"], z["v"], posBase=0, gate=z["gate"])
    ok, mad, cos = close(out, z["expected"], tol=1e-5)
    assert ok, (mad, cos)


def test_plain_attention_d128():
    z = load("ga_d128_plain.npz")
    out = attention.attend(z["q"], z["k"], z["v"], posBase=0)
    ok, mad, cos = close(out, z["expected"], tol=1e-5)
    assert ok, (mad, cos)


def test_kc_deltanet_recur():
    z = load("kc_deltanet_recur.npz")
    S, H, DK, DV, HK = [int(x) for x in z["params"][:5]]
    q = z["in0"].reshape(S, HK, DK)
    k = z["in1"].reshape(S, HK, DK)
    v = z["in2"].reshape(S, H, DV)
    g = z["in3"].reshape(S, H)
    b = z["in4"].reshape(S, H)
    core, _ = deltanet.recurrent(q, k, v, g, b)
    ok, mad, cos = close(core, z["expected"], tol=1e-5)
    assert ok, (mad, cos)


def test_delta_s70_recurrent_and_chunk():
    z = load("dn_delta_s70.npz")
    core, st = deltanet.recurrent(z["q"], z["k"], z["v"], z["g"], z["beta"])
    assert close(core, z["recurrent"], tol=1e-5)[0]
    core2, st2 = deltanet.chunk(z["q"], z["k"], z["v"], z["g"], z["beta"])
    assert close(core2, z["chunk"], tol=1e-5)[0]
    assert np.abs(st - st2).max() < 1e-4
    # chunk continuation from a carried state == one long recurrence
    a, sa = deltanet.chunk(z["q"][:40], z["k"][:40], z["v"][:40], z["g"][:40], z["beta"][:40])
    b, sb = deltanet.chunk(z["q"][40:], z["k"][40:], z["v"][40:], z["g"][40:], z["beta"][40:], state_in=sa)
    assert close(np.concatenate([a, b]), z["recurrent"], tol=1e-4)[0]


def test_kc_gbeta():
    z = load("kc_gbeta.npz")
    S, H = [int(x) for x in z["params"][:2]]
    g, b = deltanet.gbeta(z["in0"].reshape(S, H), z["in1"].reshape(S, H), z["in2"], z["in3"])
    ok, mad, cos = close(np.concatenate([g.ravel(), b.ravel()]), z["expected"], tol=1e-6)
    assert ok, (mad, cos)


def test_kc_norm_gate():
    z = load("kc_norm_gate.npz")
    rows, DV = int(z["params"][0]), int(z["params"][1])
    eps = float(z["params"][2])
    y = deltanet.norm_gate(z["in0"].reshape(rows, DV), z["in1"].reshape(rows, DV), z["in2"], eps)
    ok, mad, cos = close(y, z["expected"], tol=1e-5)
    assert ok, (mad, cos)


def test_q8_codec_roundtrip_and_rules():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((17, 8, 128)).astype(np.float32)
    x[3, 2, :32] = 0.0                     # all-zero block: scale clamps to 1e-30, codes 0
    c, s = kvcodec.q8_encode(x)
    assert c.dtype == np.int8 and s.shape == (17, 8, 4)
    assert np.all(c[3, 2, :32] == 0) and s[3, 2, 0] == np.float32(1e-30)
    assert np.abs(c).max() <= 127
    # the block absmax element encodes to +-127 exactly
    xb = x.reshape(17, 8, 4, 32)
    amax = np.abs(xb).argmax(-1)
    cb = c.reshape(17, 8, 4, 32)
    got = np.take_along_axis(np.abs(cb.astype(np.int32)), amax[..., None], -1)[..., 0]
    assert np.all(got[s > 1e-20] == 127)
    y = kvcodec.q8_decode(c, s)
    assert np.abs(y - x).max() <= (np.abs(x).max() / 127.0) * 0.5 + 1e-6
    # ties round up (floor(0.5 + 127 e)): e = 0.5/127 -> code 1, e = -0.5/127 -> code 0
    t = np.zeros((1, 32), np.float32)
    t[0, 0] = 1.0
    t[0, 1] = np.float32(0.5 / 127)
    t[0, 2] = np.float32(-0.5 / 127)
    ct, _ = kvcodec.q8_encode(t)
    ref = np.floor(np.float32(0.5) + np.float32(127) * (t[0, :3] / np.float32(1.0)))
    assert list(ct[0, :3]) == list(ref.astype(np.int8))


def test_roll_identity_before_eviction():
    """rope-at-read by slot j == keys roped at write with position j (f32 path)."""
    rng = np.random.default_rng(1)
    L, KV, D, H, S = 40, 2, 128, 4, 1
    cosT, sinT = rope.synth_rope(D, 64, 1e6, "yarn", 4.0, 8192)
    k = rng.standard_normal((L, KV, D)).astype(np.float32)
    v = rng.standard_normal((L, KV, D)).astype(np.float32)
    q = rng.standard_normal((S, H, D)).astype(np.float32)
    kr = attention.rotate_keys_at_read(k, cosT, sinT)
    cf = np.concatenate([cosT, cosT], -1)[:L, None, :]
    sf = np.concatenate([sinT, sinT], -1)[:L, None, :]
    kw = rope.rope_rotate_half(k, cf, sf)
    assert np.array_equal(kr, kw)
    a = attention.attend(q, kr, v, posBase=L - 1)
    assert np.all(np.isfinite(a))


def test_eviction_schedule():
    # engine.ts:1188-1214 with 4 sinks, maxSeqLen 4100: first eviction at fill 4100 + 1 row
    b, nf = evict.evict_for(4100, 1, 4, 4100)
    assert (b, nf) == (1024, 3076)
    assert evict.evict_for(4099, 1, 4, 4100) == (0, 4099)
    # giant need: sinks only
    assert evict.evict_plan(100, 500, 4, 100) == (96, 4)
    w = evict.LogicalWindow(4, 100)
    w.append(range(100))
    w.append([100])
    assert w.fill == 4 + (96 - 24) + 1
    assert w.slots[:4] == [0, 1, 2, 3] and w.slots[4] == 28 and w.slots[-1] == 100


def test_partials_merge_equals_attend():
    rng = np.random.default_rng(2)
    L, KV, D, H, S = 300, 2, 128, 6, 3
    k = rng.standard_normal((L, KV, D)).astype(np.float32)
    v = rng.standard_normal((L, KV, D)).astype(np.float32)
    q = rng.standard_normal((S, H, D)).astype(np.float32)
    pb = L - S
    ref = attention.attend(q, k, v, pb)
    parts = [attention.attend_partials(q, k, v, pb, lo, min(lo + 128, L)) for lo in range(0, L, 128)]
    out = attention.lse_merge(*zip(*parts))
    assert np.abs(out - ref).max() < 1e-5


# ---- hybrid-layer glue and the end-to-end forward ----

def test_kc_conv1d():
    from oracle import glue
    z = load("kc_conv1d.npz")
    S, C, K, _ = [int(x) for x in z["params"]]
    y, st = glue.conv1d_causal(z["in0"].reshape(S, C), z["in1"].reshape(C, K))
    assert np.array_equal(y.reshape(-1), z["expected"])
    assert np.array_equal(st, z["in0"].reshape(S, C)[S - (K - 1):])


def test_conv1d_segments_carry_state():
    """Two segments chained through the carried state == one segment (conv1d_causal.wgsl:4-6)."""
    from oracle import glue
    z = load("kc_conv1d.npz")
    S, C, K, _ = [int(x) for x in z["params"]]
    x, w = z["in0"].reshape(S, C), z["in1"].reshape(C, K)
    y1, s1 = glue.conv1d_causal(x[:5], w)
    y2, s2 = glue.conv1d_causal(x[5:], w, s1)
    assert np.array_equal(np.concatenate([y1, y2]).reshape(-1), z["expected"])
    y3, s3 = glue.conv1d_causal(x[:1], w)          # shorter than K-1: state keeps zeros
    assert np.array_equal(s3[:K - 2], np.zeros((K - 2, C), np.float32)) and np.array_equal(s3[-1], x[0])


def test_kc_rope_partial():
    from oracle import glue
    z = load("kc_rope_partial.npz")
    S, H, D, R = [int(x) for x in z["params"]]
    y = glue.rope_partial(z["in0"].reshape(S, H, D), z["in1"].reshape(S, R), z["in2"].reshape(S, R), R)
    assert np.array_equal(y.reshape(-1), z["expected"])


def test_qk_prologue():
    from oracle import glue
    z = load("kc_qk_prologue.npz")
    S, H, D2 = z["qg"].shape
    D, R = D2 // 2, z["cos"].shape[1]
    y = glue.qk_norm_rope(z["qg"].reshape(S, -1), H, D, 2 * D, 0, 1.0 + z["w"], z["cos"], z["sin"], R, 1e-6)
    ok, mad, cos = close(y, z["expected"], tol=1e-6)
    assert ok, (mad, cos)
    gate = glue.slice_cols(z["qg"], S * H, D, 2 * D, D).reshape(S, H, D)
    assert np.array_equal(gate, z["gate"])


def test_hybrid_forward_vs_reference():
    """Restated hybrid forward == the reference's numpy forward on the same seeded weights."""
    from oracle import hybrid
    z = load("hy_forward_s300.npz")
    cfg = hybrid.Cfg()
    out = hybrid.forward(hybrid.synth_weights(cfg, int(z["seed"])), cfg, z["ids"])
    assert np.abs(out["logits"][-16:] - z["logits_tail"]).max() < 1e-4
    assert np.array_equal(out["logits"].argmax(-1), z["argmax"])
    assert np.abs(np.stack([h[-1] for h in out["layers"]]) - z["last_hidden"]).max() < 1e-4


def test_synth_qwen35_weights_and_forward_match_reference_fixture():
    """oracle.synth_qwen35 redraws the reference's synthetic 1-bit hybrid model
    (tools/gen-synth-qwen35.py, seed 1): its embedding rows equal the fixture's bytes, and the
    oracle forward over them reproduces the reference's own logits and layer-0 output."""
    from oracle import hybrid as HY
    from oracle import synth_qwen35 as SQ
    z = np.load(os.path.join(GOLDEN, "synth_qwen35_fixture.npz"))
    cfg, W = SQ.synth_weights()
    ids = SQ.synth_ids()
    assert np.array_equal(ids, z["ids"])
    assert np.array_equal(W["embed"][ids][-32:], z["embed_tail"])
    out = HY.forward(W, cfg, ids)
    assert np.abs(out["layers"][0] - z["layer0"]).max() < 1e-3
    assert np.abs(out["logits"] - z["logits"]).max() < 1e-3
    assert int(out["logits"][-1].argmax()) == int(z["argmax_last"]) == 201
