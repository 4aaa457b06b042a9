"""GPU parity: hybrid-layer glue (conv1d + state, column slices, fused q/k prologue) vs the oracle."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from gpu_util import gate_ok
from oracle import glue, kvcodec

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from bitgpu_b200 import ops
    return ops


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def test_conv1d_golden(ops):
    """conv1d_causal.wgsl case of the reference's kernel-case generator (zero state)."""
    z = load("kc_conv1d.npz")
    S, C, K, _ = [int(x) for x in z["params"]]
    y, st = ops.conv1d_causal(cu(z["in0"].reshape(S, C)), cu(z["in1"].reshape(C, K)))
    ok, mad, cs = gate_ok(y.cpu().numpy().reshape(-1), z["expected"], tol=1e-5)
    assert ok, (mad, cs)
    assert torch.equal(st.cpu(), torch.from_numpy(z["in0"].reshape(S, C)[S - K + 1:]))


@pytest.mark.parametrize("K,C,cuts", [(4, 10240, [300]), (4, 1000, [1, 2, 70, 200]), (2, 96, [33, 5]),
                                      (8, 257, [3, 100])])
def test_conv1d_segments(ops, K, C, cuts):
    """Segmented calls chained through the carried state (engine ping-pong) == the oracle over
    the whole stream; includes segments shorter than K-1."""
    rng = np.random.default_rng(K * 1000 + C)
    S = sum(cuts)
    x = rng.standard_normal((S, C)).astype(np.float32)
    w = (0.5 * rng.standard_normal((C, K))).astype(np.float32)
    exp, exp_st = glue.conv1d_causal(x, w)
    wd, st, outs, t = cu(w), None, [], 0
    for n in cuts:
        y, st = ops.conv1d_causal(cu(x[t:t + n]), wd, st)
        outs.append(y.cpu().numpy())
        t += n
    got = np.concatenate(outs)
    assert np.abs(got - exp).max() < 2e-5
    assert np.abs(st.cpu().numpy() - exp_st).max() == 0


def test_slice_cols(ops):
    rng = np.random.default_rng(5)
    src = rng.standard_normal((37, 100)).astype(np.float32)
    for width, off in ((40, 0), (40, 40), (20, 80), (13, 7)):
        got = ops.slice_cols(cu(src), 37, width, 100, off).cpu().numpy()
        assert np.array_equal(got, glue.slice_cols(src, 37, width, 100, off))


def test_qk_prologue_golden(ops):
    """split_head + rmsnorm + rope_partial of the reference's own functions, one launch."""
    z = load("kc_qk_prologue.npz")
    S, H, D2 = z["qg"].shape
    D, R = D2 // 2, z["cos"].shape[1]
    y = ops.qk_norm_rope(cu(z["qg"]), 1, S, H, D, 2 * D, 0, cu(1.0 + z["w"]), cu(z["cos"]), cu(z["sin"]), R, 0, 1e-6)
    ok, mad, cs = gate_ok(y[0].cpu().numpy(), z["expected"], tol=1e-5)
    assert ok, (mad, cs)
    gate = ops.slice_cols(cu(z["qg"]), S * H, D, 2 * D, D).cpu().numpy().reshape(S, H, D)
    assert np.array_equal(gate, z["gate"])


@pytest.mark.parametrize("mode", ["f32", "f16", "q8", "q8r"])
@pytest.mark.parametrize("D,rot", [(256, 64), (128, 128), (128, 0), (64, 32)])
def test_qk_prologue_to_cache(ops, mode, D, rot):
    """K path: norm + partial rope written straight into the cache (positions pos0..) with the
    cache codec; the stored bytes are the codec of the kernel's own y, and y matches the oracle."""
    if mode == "q8r" and D % 128:
        pytest.skip()
    rng = np.random.default_rng(D + rot)
    B, S, KV, pos0, P = 2, 5, 2, 9, 40
    x = rng.standard_normal((B, S, KV, D)).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    cos, sin = glue.rope_tables(P, max(rot, 2), 1e7)
    cache = ops.KVCache(B, P, KV, D, mode=mode)
    y = ops.qk_norm_rope(cu(x), B, S, KV, D, D, 0, cu(gamma), cu(cos), cu(sin), rot, pos0, 1e-6, cache=cache)
    yn = y.cpu().numpy()
    for b in range(B):
        exp = glue.qk_norm_rope(x[b].reshape(S, -1), KV, D, D, 0, gamma, cos[pos0:pos0 + S], sin[pos0:pos0 + S],
                                rot, 1e-6)
        ok, mad, cs = gate_ok(yn[b], exp, tol=1e-5)
        assert ok, (mad, cs)
    enc, sc = kvcodec.encode(mode, yn)
    got = cache.K[:, pos0:pos0 + S].cpu().numpy()
    if mode in ("q8", "q8r"):
        assert np.array_equal(got.view(np.uint8), enc.view(np.uint8))
        assert np.array_equal(cache.Ks[:, pos0:pos0 + S].cpu().numpy(), sc)
    else:
        assert np.array_equal(got, enc)


def test_glue_errors(ops):
    from bitgpu_b200._lib import lib
    L = lib()
    assert L.bg_slice_cols(None, 1, 1, 1, 0, None, None) < 0
    x = torch.zeros(8, 4, device="cuda")
    assert L.bg_slice_cols(ops._p(x), 8, 3, 4, 2, ops._p(x), None) < 0        # off + width > stride
    w = torch.zeros(4, 9, device="cuda")
    st = torch.zeros(8, 4, device="cuda")
    assert L.bg_conv1d_causal(ops._p(x), ops._p(w), None, 0, 8, 4, 9, ops._p(x), ops._p(st), None) < 0  # K > 8
    assert L.bg_conv1d_causal(ops._p(x), ops._p(w), ops._p(st), 1, 8, 4, 4, ops._p(x), ops._p(st), None) < 0
