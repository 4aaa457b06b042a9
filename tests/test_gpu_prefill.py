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


@pytest.mark.parametrize("B,S,H,KV,pos_base,out16", [
    (2, 300, 32, 8, 0, True),      # ragged S (not a multiple of 256), GQA 4
    (1, 256, 16, 8, 0, False),     # exactly one block, GQA 2, f32 output
    (1, 200, 32, 8, 77, True),     # continuing segment: posBase > 0 (engine prefill segments)
    (1, 64, 8, 8, 1000, True),     # smallest S on this path, MHA, long prefix
])
def test_prefill_vs_oracle(ops, B, S, H, KV, pos_base, out16):
    rng = np.random.default_rng(S + H + pos_base)
    D = 128
    L = pos_base + S
    cache = ops.KVCache(B, L + 7, KV, D, mode="f16")
    Kd, Vd = fill_cache(cache, rand(rng, B, L, KV, D), rand(rng, B, L, KV, D))
    q = rand(rng, B, S, H, D).astype(np.float16)
    out = ops.attention(torch.from_numpy(q).cuda(), cache, pos_base,
                        out_dtype=torch.float16 if out16 else torch.float32).float().cpu().numpy()
    for b in range(B):
        exp = OA.attend(q[b].astype(np.float32), Kd[b], Vd[b], pos_base)
        bound = 2e-3 + (half_ulp(exp) if out16 else 0.0)
        err = np.abs(out[b] - exp)
        assert np.all(err <= bound), (b, float(err.max()), float((err - bound).max()))
        cos = float((out[b] * exp).sum() / (np.linalg.norm(out[b]) * np.linalg.norm(exp)))
        assert cos > 0.99999


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
