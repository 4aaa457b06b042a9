"""GPU parity: tcgen05 causal prefill (f16 Q over an f16 cache) vs the oracle and vs the CUDA-core
path.  The reference computes in f32 on the f16-rounded inputs (its kv16 convention,
shaders/attention_sg_kv16.wgsl:1-4); the f16 output adds at most half an f16 ulp of rounding, so
the bound is 2e-3 + 0.5 ulp_f16(expected) for f16 outputs and 2e-3 for f32 outputs."""
import numpy as np
import pytest
import torch

from gpu_util import fill_cache, rand
from oracle import attention as OA

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from bitgpu_b200 import ops
    return ops


def half_ulp(x):
    x = np.abs(np.asarray(x, np.float32)).astype(np.float16)
    return (np.spacing(x).astype(np.float32)) * 0.5


@pytest.mark.parametrize("mode", ["f16", "q8", "f32"])
@pytest.mark.parametrize("q32", [False, True])
@pytest.mark.parametrize("B,S,H,KV,D,pos_base,out16,gated", [
    (2, 300, 32, 8, 128, 0, True, False),     # ragged S (not a multiple of 256), GQA 4
    (1, 256, 16, 8, 128, 0, False, False),    # exactly one block, GQA 2, f32 output
    (1, 200, 32, 8, 128, 77, True, False),    # continuing segment: posBase > 0 (engine prefill segments)
    (1, 64, 8, 8, 128, 1000, True, False),    # smallest S on this path, MHA, long prefix
    (1, 256, 24, 4, 256, 0, False, True),     # the 27B hybrid's gated head_dim-256 prefill segment
    (1, 200, 24, 4, 256, 3000, False, True),  # ... continuing after a long context
    (2, 130, 8, 2, 256, 5, True, False),      # head_dim 256, ragged, f16 output, no gate
])
def test_prefill_vs_oracle(ops, mode, q32, B, S, H, KV, D, pos_base, out16, gated):
    """tcgen05 prefill over f16 and q8 caches with f16 and f32 queries (the engine's call passes
    f32 queries, engine.ts:1580), head_dim 128 and the gated head_dim 256, and over an f32 cache
    in 3xTF32 (head_dim 128; head_dim 256 f32 runs on the CUDA-core kernel), vs the oracle."""
    rng = np.random.default_rng(S + H + pos_base + D)
    L = pos_base + S
    cache = ops.KVCache(B, L + 7, KV, D, mode=mode)
    Kd, Vd = fill_cache(cache, rand(rng, B, L, KV, D), rand(rng, B, L, KV, D))
    q = rand(rng, B, S, H, D)
    if not q32:
        q = q.astype(np.float16)
    gate = rand(rng, B, S, H, D) if gated else None
    scale = 1.0 / np.sqrt(D)
    out = ops.attention(torch.from_numpy(q).cuda(), cache, pos_base, scale=scale,
                        gate=torch.from_numpy(gate).cuda() if gated else None,
                        out_dtype=torch.float16 if out16 else torch.float32).float().cpu().numpy()
    for b in range(B):
        exp = OA.attend(q[b].astype(np.float32), Kd[b], Vd[b], pos_base, scale=scale,
                        gate=gate[b] if gated else None)
        bound = 2e-3 + (half_ulp(exp) if out16 else 0.0)
        err = np.abs(out[b] - exp)
        assert np.all(err <= bound), (b, float(err.max()), float((err - bound).max()))
        cos = float((out[b] * exp).sum() / (np.linalg.norm(out[b]) * np.linalg.norm(exp)))
        assert cos > 0.99999
    from bitgpu_b200._lib import lib
    assert lib().bg_device_status(None) == 0


def test_prefill_vs_generic_long(ops):
    """2048-token prefill: tcgen05 kernel vs the CUDA-core kernel (forced), same inputs."""
    from bitgpu_b200._lib import lib
    B, S, H, KV, D = 1, 2048, 32, 8, 128
    g = torch.Generator(device="cuda").manual_seed(5)
    cache = ops.KVCache(B, S, KV, D, mode="f16")
    cache.append(0, torch.randn((B, S, KV, D), generator=g, device="cuda"), 0)
    cache.append(1, torch.randn((B, S, KV, D), generator=g, device="cuda"), 0)
    q = torch.randn((B, S, H, D), generator=g, device="cuda").half()
    a = ops.attention(q, cache, 0)
    prev = lib().bg_force_generic(1)
    try:
        b = ops.attention(q, cache, 0)
    finally:
        lib().bg_force_generic(prev)
    assert (a - b).abs().max().item() < 2e-3
    assert lib().bg_device_status(None) == 0


@pytest.mark.parametrize("D,H,KV", [(128, 32, 8), (256, 24, 4)])
def test_prefill_q8_fused_equals_prepass(ops, D, H, KV):
    """A q8 prefill dequantises the cache once into the workspace when it has room (the path
    ops.attention takes), else inside every CTA (no workspace): both vs the oracle."""
    import ctypes as C
    from bitgpu_b200._lib import AttnParams, DT_F32, lib
    rng = np.random.default_rng(D)
    B, S = 1, 512
    cache = ops.KVCache(B, S, KV, D, mode="q8")
    Kd, Vd = fill_cache(cache, rand(rng, B, S, KV, D), rand(rng, B, S, KV, D))
    q = torch.from_numpy(rand(rng, B, S, H, D)).cuda()
    a = ops.attention(q, cache, 0)
    p = AttnParams(S, H, KV, D, 0, S)
    d = cache.desc()
    b = torch.empty_like(q)
    rc = lib().bg_attention(C.byref(p), B, C.c_void_p(q.data_ptr()), DT_F32, C.byref(d), None, None, 0.0, None,
                            C.c_void_p(b.data_ptr()), DT_F32, None, 0,
                            C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    exp = OA.attend(q[0].cpu().numpy(), Kd[0], Vd[0], 0)
    for out in (a, b):
        err = np.abs(out[0].cpu().numpy() - exp).max()
        assert err < 2e-3, err
    assert lib().bg_device_status(None) == 0


def test_prefill_f32_3xtf32_precision(ops):
    """The 3xTF32 split (hi/lo operands, three products each for Q K^T and P V) keeps the f32
    cache's prefill at f32-class accuracy: errors near 1e-6 against the oracle, where one TF32
    product per matrix would sit near 1e-3."""
    rng = np.random.default_rng(123)
    B, S, H, KV, D = 1, 512, 16, 4, 128
    cache = ops.KVCache(B, S, KV, D, mode="f32")
    Kd, Vd = fill_cache(cache, rand(rng, B, S, KV, D), rand(rng, B, S, KV, D))
    q = rand(rng, B, S, H, D)
    out = ops.attention(torch.from_numpy(q).cuda(), cache, 0).cpu().numpy()
    exp = OA.attend(q[0], Kd[0], Vd[0], 0)
    err = float(np.abs(out[0] - exp).max())
    assert err < 5e-5, err
