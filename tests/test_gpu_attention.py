"""GPU parity: attention kernels (through the C ABI) vs the CPU oracle."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from gpu_util import TOL, fill_cache, gate_ok, rand
from oracle import attention as OA
from oracle import rope as OR

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from bitgpu_b200 import ops
    return ops


def run_case(ops, mode, B, S, H, KV, D, pos_base, seed, q_dtype=torch.float32, gate=False, scale=0.0,
             out_dtype=torch.float32, roll=False, window=0, ring_head=0, sinks=0, cap_extra=5):
    rng = np.random.default_rng(seed)
    L = pos_base + S
    cache = ops.KVCache(B, L + cap_extra, KV, D, mode=mode, sinks=sinks, window=window, device="cuda")
    cache.ring_head = ring_head
    Kraw, Vraw = rand(rng, B, L, KV, D), rand(rng, B, L, KV, D)
    Kd, Vd = fill_cache(cache, Kraw, Vraw)
    q = rand(rng, B, S, H, D)
    if q_dtype == torch.float16:
        q = q.astype(np.float16).astype(np.float32)
    g = rand(rng, B, S, H, D) if gate else None
    cos_t = sin_t = None
    if roll:
        c, s = OR.synth_rope(D, L + 8, 1e6, "yarn", 4.0, 8192)
        cos_t, sin_t = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
    out = ops.attention(torch.from_numpy(q).to("cuda", q_dtype), cache, pos_base, scale=scale,
                        gate=None if g is None else torch.from_numpy(g).cuda(), cos_t=cos_t, sin_t=sin_t,
                        out_dtype=out_dtype)
    out = out.float().cpu().numpy()
    for b in range(B):
        Kb = OA.rotate_keys_at_read(Kd[b], c, s) if roll else Kd[b]
        exp = OA.attend(q[b], Kb, Vd[b], pos_base, scale=scale if scale else None,
                        gate=None if g is None else g[b])
        ok, mad, cos = gate_ok(out[b], exp, tol=TOL)
        assert ok, (mode, b, mad, cos)
    return out


@pytest.mark.parametrize("mode", ["f32", "f16", "q8", "q8r"])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_decode_modes(ops, mode, D):
    if mode == "q8r" and D % 128:
        pytest.skip("q8r needs D % 128 == 0")
    run_case(ops, mode, B=2, S=1, H=8, KV=2, D=D, pos_base=777, seed=D)


@pytest.mark.parametrize("mode", ["f32", "f16", "q8"])
@pytest.mark.parametrize("S,H,KV,pos_base", [(3, 16, 8, 100), (9, 32, 8, 1500), (17, 24, 4, 0), (5, 6, 6, 63)])
def test_multi_row_causal(ops, mode, S, H, KV, pos_base):
    """PLD verify / prefill rows: row qi attends 0..posBase+qi (attention_sg.wgsl:21,31)."""
    run_case(ops, mode, B=1, S=S, H=H, KV=KV, D=128, pos_base=pos_base, seed=S * 7 + H)


def test_cfg1_shape(ops):
    """Config 1: Qwen3-1.7B shape, 2048-position f32 cache, one query token."""
    run_case(ops, "f32", B=1, S=1, H=16, KV=8, D=128, pos_base=2047, seed=1)


def test_long_context_f16_q8(ops):
    for mode in ("f16", "q8"):
        run_case(ops, mode, B=2, S=1, H=32, KV=8, D=128, pos_base=32767, seed=2)


def test_gated_d256(ops):
    """27B gated attention shape (H24/KV4/D256) with the sigmoid gate fused in the merge."""
    for mode in ("f32", "f16", "q8"):
        run_case(ops, mode, B=1, S=2, H=24, KV=4, D=256, pos_base=4000, seed=3, gate=True,
                 scale=float(1 / np.sqrt(256)))


def test_f16_q_and_f16_out(ops):
    run_case(ops, "f16", B=2, S=4, H=32, KV=8, D=128, pos_base=300, seed=4, q_dtype=torch.float16,
             out_dtype=torch.float16)


@pytest.mark.parametrize("mode", ["f32", "f16", "q8"])
def test_roll_rope_at_read(ops, mode):
    run_case(ops, mode, B=2, S=1, H=16, KV=8, D=128, pos_base=500, seed=5, roll=True)


@pytest.mark.parametrize("mode", ["f16", "q8"])
def test_roll_ring_wrapped(ops, mode):
    """Ring layout with the head mid-window: logical slot order must not depend on it."""
    run_case(ops, mode, B=2, S=1, H=16, KV=8, D=128, pos_base=299, seed=6, roll=True, sinks=4, window=296,
             ring_head=123, cap_extra=0)


def test_golden_gated_d256(ops):
    z = np.load(os.path.join(GOLDEN, "ga_d256_gated.npz"))
    S, H, D = z["q"].shape
    KV = z["k"].shape[1]
    cache = ops.KVCache(1, S, KV, D, mode="f32")
    cache.K[0] = torch.from_numpy(z["k"]).cuda()
    cache.V[0] = torch.from_numpy(z["v"]).cuda()
    out = ops.attention(torch.from_numpy(z["q"])[None].cuda(), cache, 0, scale=float(1 / np.sqrt(D)),
                        gate=torch.from_numpy(z["gate"])[None].cuda().contiguous())
    ok, mad, cos = gate_ok(out[0].cpu().numpy(), z["expected"])
    assert ok, (mad, cos)


def test_golden_kernel_case_attention(ops):
    """tools/gen-kernel-cases.py 'attention' case (head_dim 256) through the cache path."""
    z = np.load(os.path.join(GOLDEN, "kc_attention.npz"))
    S, H, KV, D = [int(x) for x in z["params"][:4]]
    cache = ops.KVCache(1, S, KV, D, mode="f32")
    cache.K[0] = torch.from_numpy(z["in1"].reshape(S, KV, D)).cuda()
    cache.V[0] = torch.from_numpy(z["in2"].reshape(S, KV, D)).cuda()
    out = ops.attention(torch.from_numpy(z["in0"].reshape(1, S, H, D)).cuda(), cache, 0, scale=float(z["params"][4]))
    ok, mad, cos = gate_ok(out.cpu().numpy(), z["expected"])
    assert ok, (mad, cos)


def test_golden_plain_d128(ops):
    z = np.load(os.path.join(GOLDEN, "ga_d128_plain.npz"))
    S, H, D = z["q"].shape
    KV = z["k"].shape[1]
    for mode in ("f32", "f16"):
        cache = ops.KVCache(1, S + 3, KV, D, mode=mode)
        fill_cache(cache, z["k"][None], z["v"][None])
        out = ops.attention(torch.from_numpy(z["q"])[None].cuda(), cache, 0)
        ok, mad, cos = gate_ok(out[0].cpu().numpy(), z["expected"], tol=2e-3 if mode == "f16" else 1e-5)
        assert ok, (mode, mad, cos)


def test_split_partials_merge(ops):
    """bg_attention_partials over disjoint slices + bg_lse_merge == full attention."""
    rng = np.random.default_rng(9)
    B, S, H, KV, D, pb = 1, 2, 24, 4, 256, 3000
    L = pb + S
    Kraw, Vraw = rand(rng, B, L, KV, D), rand(rng, B, L, KV, D)
    q = torch.from_numpy(rand(rng, B, S, H, D)).cuda()
    gate = torch.from_numpy(rand(rng, B, S, H, D)).cuda()
    full = ops.KVCache(B, L, KV, D, mode="f16")
    fill_cache(full, Kraw, Vraw)
    ref = ops.attention(q, full, pb, gate=gate).cpu().numpy()
    bounds = [0, 700, 1800, 1801, L]
    parts = []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        c = ops.KVCache(B, max(hi - lo, 1), KV, D, mode="f16")
        fill_cache(c, Kraw[:, lo:hi], Vraw[:, lo:hi])
        parts.append(ops.attention_partials(q, c, pb, lo, hi))
    out = ops.lse_merge(torch.stack(parts), (B, S, H, D), gate=gate).cpu().numpy()
    assert np.abs(out - ref).max() < 1e-4


def test_abi_errors(ops):
    """Validation mirrors the engine's throws: H % KV, q8 head_dim, Ltot, capacity."""
    from bitgpu_b200._lib import BgError
    cache = ops.KVCache(1, 16, 3, 128, mode="f16")
    q = torch.zeros(1, 1, 8, 128, device="cuda")
    with pytest.raises(BgError):
        ops.attention(q, cache, 0)          # 8 % 3 != 0
    cache = ops.KVCache(1, 16, 2, 128, mode="f16")
    with pytest.raises(BgError):
        ops.attention(q, cache, 16)         # posBase + S > capacity


@pytest.mark.parametrize("mode", ["f16", "q8"])
@pytest.mark.parametrize("shape", [(64, 1, 32, 8, 128, 32767), (3, 2, 32, 8, 128, 5000), (2, 4, 32, 8, 128, 700),
                                   (1, 1, 24, 4, 256, 131071 // 4), (2, 1, 16, 8, 128, 2047), (1, 3, 6, 6, 128, 90)])
def test_tensor_core_vs_generic(ops, mode, shape):
    """The tensor-core decode kernel and the CUDA-core kernel agree (both also match the oracle
    in the tests above); shapes cover G = 1..6, 1..16 rows per group and long contexts."""
    from bitgpu_b200._lib import lib
    B, S, H, KV, D, pb = shape
    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    cache = ops.KVCache(B, pb + S, KV, D, mode=mode)
    cache.append(0, torch.randn((B, pb + S, KV, D), generator=g, device="cuda"), 0)
    cache.append(1, torch.randn((B, pb + S, KV, D), generator=g, device="cuda"), 0)
    q = torch.randn((B, S, H, D), generator=g, device="cuda")
    a = ops.attention(q, cache, pb)
    prev = lib().bg_force_generic(1)
    try:
        b = ops.attention(q, cache, pb)
    finally:
        lib().bg_force_generic(prev)
    err = (a - b).abs().max().item()
    assert err < 1e-3, err
    assert lib().bg_device_status(None) == 0


def test_tc_oracle_spot(ops):
    """Tensor-core path vs oracle at the config-2 shape (2 sequences sampled)."""
    for mode in ("f16", "q8"):
        run_case(ops, mode, B=2, S=1, H=32, KV=8, D=128, pos_base=32767, seed=31)


@pytest.mark.parametrize("mode", ["f16", "q8"])
@pytest.mark.parametrize("S,ring_head", [(1, 0), (1, 1500), (2, 4090), (3, 77)])
def test_roll_tensor_core_vs_generic(ops, mode, S, ring_head):
    """Rope-at-read on the tensor cores (cp.async ring producer, rotation in registers) vs the
    CUDA-core kernel, on a ring whose wrap point falls inside tiles."""
    from bitgpu_b200._lib import lib
    B, H, KV, D, SINKS, W = 3, 16, 8, 128, 4, 4096
    g = torch.Generator(device="cuda").manual_seed(S + ring_head)
    cache = ops.KVCache(B, 0, KV, D, mode=mode, sinks=SINKS, window=W)
    cache.ring_head = ring_head
    L = SINKS + W - 5
    cache.append(0, torch.randn((B, L, KV, D), generator=g, device="cuda"), 0)
    cache.append(1, torch.randn((B, L, KV, D), generator=g, device="cuda"), 0)
    c, s_ = OR.synth_rope(D, SINKS + W, 1e6, "yarn", 4.0, 8192)
    cos_t, sin_t = torch.from_numpy(c).cuda(), torch.from_numpy(s_).cuda()
    q = torch.randn((B, S, H, D), generator=g, device="cuda")
    a = ops.attention(q, cache, L - S, cos_t=cos_t, sin_t=sin_t)
    prev = lib().bg_force_generic(1)
    try:
        b = ops.attention(q, cache, L - S, cos_t=cos_t, sin_t=sin_t)
    finally:
        lib().bg_force_generic(prev)
    err = (a - b).abs().max().item()
    assert err < 1e-3, err
    assert lib().bg_device_status(None) == 0


@pytest.mark.parametrize("mode", ["f16", "q8"])
@pytest.mark.parametrize("H,KV,S", [(16, 4, 1), (12, 2, 1), (12, 6, 1), (9, 3, 1), (32, 8, 3)])
def test_roll_head_groups(ops, mode, H, KV, S):
    """Rope-at-read kernels across kv-head grouping: 4 and 2 heads per CTA (KV = 4, 2, 6), no
    grouping (KV = 3: the one-head-per-CTA kernel) and a GQA group wider than 8 rows (H32 KV8,
    S = 3: the two-column-tile kernel), on a wrapped ring, vs the CUDA-core kernel and the oracle."""
    from bitgpu_b200._lib import lib
    B, D, SINKS, W = 2, 128, 4, 1000
    rng = np.random.default_rng(H * 100 + KV * 10 + S)
    cache = ops.KVCache(B, 0, KV, D, mode=mode, sinks=SINKS, window=W)
    cache.ring_head = 321
    L = SINKS + W - 7
    Kraw, Vraw = rand(rng, B, L, KV, D), rand(rng, B, L, KV, D)
    Kd, Vd = fill_cache(cache, Kraw, Vraw)
    c, s_ = OR.synth_rope(D, SINKS + W, 1e6, "yarn", 4.0, 8192)
    cos_t, sin_t = torch.from_numpy(c).cuda(), torch.from_numpy(s_).cuda()
    q = rand(rng, B, S, H, D)
    a = ops.attention(torch.from_numpy(q).cuda(), cache, L - S, cos_t=cos_t, sin_t=sin_t)
    prev = lib().bg_force_generic(1)
    try:
        g = ops.attention(torch.from_numpy(q).cuda(), cache, L - S, cos_t=cos_t, sin_t=sin_t)
    finally:
        lib().bg_force_generic(prev)
    assert (a - g).abs().max().item() < 1e-3
    an = a.cpu().numpy()
    for b in range(B):
        exp = OA.attend(q[b], OA.rotate_keys_at_read(Kd[b], c, s_), Vd[b], L - S)
        ok, mad, cs = gate_ok(an[b], exp, tol=TOL)
        assert ok, (mode, H, KV, S, b, mad, cs)
    assert lib().bg_device_status(None) == 0



@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("nsplit", [17, 40, 130])
def test_lse_merge_many_splits(ops, D, nsplit):
    """bg_lse_merge beyond 16 splits (the column-sliced merge kernel) against a numpy log-sum-exp
    merge, gated output; empty splits (l = 0 with arbitrary m / o bits) are skipped."""
    rng = np.random.default_rng(nsplit + D)
    rows = 24
    o = rng.standard_normal((nsplit, rows, D)).astype(np.float32)
    m = (3.0 * rng.standard_normal((nsplit, rows))).astype(np.float32)
    l = rng.uniform(0.5, 4.0, (nsplit, rows)).astype(np.float32)
    empty = rng.random((nsplit, rows)) < 0.2
    empty[0] = False
    l[empty] = 0.0
    o[empty] = np.nan
    m[empty] = np.nan
    part = np.concatenate([o, m[..., None], l[..., None]], axis=-1)
    gate = rng.standard_normal((1, 1, rows, D)).astype(np.float32)
    w = np.where(empty, 0.0, np.exp(np.where(empty, 0.0, m) - np.nanmax(np.where(empty, -np.inf, m), axis=0)))
    num = np.einsum("sr,srd->rd", w, np.where(empty[..., None], 0.0, o))
    den = (w * l).sum(0)
    exp = (num / den[:, None]) / (1.0 + np.exp(-gate[0, 0]))
    out = ops.lse_merge(torch.from_numpy(part).cuda(), (1, 1, rows, D), gate=torch.from_numpy(gate).cuda())
    got = out.cpu().numpy()[0, 0]
    assert np.isfinite(got).all()
    assert np.abs(got - exp).max() < 1e-5 * max(1.0, np.abs(exp).max())
