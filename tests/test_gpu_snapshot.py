"""KV snapshot wire format on the GPU: byte layout, ring == compacted, round trips, delta,
hybrid mixer state (engine.ts:2719-2872)."""
import numpy as np
import pytest
import torch

from gpu_util import rand
from oracle import rope as OR

pytestmark = pytest.mark.gpu

MODEL = {"layers": 2, "kvHeads": 8, "headDim": 128, "hidden": 2048, "vocab": 1000}


@pytest.fixture(scope="module")
def ops():
    from bitgpu_b200 import ops
    return ops


def packed_reference_bytes(cache, seq, lo, hi):
    """The layout restated in numpy from the engine's piece list: K rows, V rows, K scale rows,
    V scale rows of positions [lo, hi) of a linear (compacted) cache."""
    parts = [cache.K[seq, lo:hi], cache.V[seq, lo:hi]]
    if cache.Ks is not None:
        parts += [cache.Ks[seq, lo:hi], cache.Vs[seq, lo:hi]]
    return b"".join(p.contiguous().cpu().numpy().tobytes() for p in parts)


@pytest.mark.parametrize("mode", ["f32", "f16", "q8"])
def test_layout_and_round_trip(ops, mode):
    from bitgpu_b200.snapshot import restore_cache, save_cache
    rng = np.random.default_rng(3)
    B, L, KV, D = 2, 50, 8, 128
    layers = [ops.KVCache(B, 64, KV, D, mode=mode) for _ in range(2)]
    for c in layers:
        c.append_kv(torch.from_numpy(rand(rng, B, L, KV, D)).cuda(), torch.from_numpy(rand(rng, B, L, KV, D)).cuda(), 0)
    ids = list(range(L + 1))
    snap = save_cache(layers, ids, mode, MODEL, seq=1)
    assert snap["version"] == 1 and "base" not in snap and "roll" not in snap
    assert snap["data"] == b"".join(packed_reference_bytes(c, 1, 0, L) for c in layers)
    fresh = [ops.KVCache(1, 64, KV, D, mode=mode) for _ in range(2)]
    got_ids, n = restore_cache(snap, fresh, mode, MODEL, max_seq_len=64)
    assert got_ids == ids and n == L
    for a, b in zip(layers, fresh):
        assert torch.equal(a.K[1, :L], b.K[0, :L]) and torch.equal(a.V[1, :L], b.V[0, :L])
        if a.Ks is not None:
            assert torch.equal(a.Ks[1, :L], b.Ks[0, :L]) and torch.equal(a.Vs[1, :L], b.Vs[0, :L])


def test_delta_snapshot(ops):
    from bitgpu_b200.snapshot import restore_cache, save_cache
    rng = np.random.default_rng(4)
    L, base, KV, D = 40, 16, 8, 128
    src = ops.KVCache(1, 64, KV, D, mode="q8")
    src.append_kv(torch.from_numpy(rand(rng, 1, L, KV, D)).cuda(), torch.from_numpy(rand(rng, 1, L, KV, D)).cuda(), 0)
    ids = list(range(100, 100 + L + 1))
    snap = save_cache([src], ids, "q8", dict(MODEL, layers=1), base=base)
    assert snap["base"] == base and snap["data"] == packed_reference_bytes(src, 0, base, L)
    dst = ops.KVCache(1, 64, KV, D, mode="q8")
    dst.K[:, :base] = src.K[:, :base]        # the prewarmed shared prefix
    dst.V[:, :base] = src.V[:, :base]
    dst.Ks[:, :base] = src.Ks[:, :base]
    dst.Vs[:, :base] = src.Vs[:, :base]
    restore_cache(snap, [dst], "q8", dict(MODEL, layers=1), max_seq_len=64, history=ids[:base], cache_len=base)
    for x, y in ((src.K, dst.K), (src.V, dst.V), (src.Ks, dst.Ks), (src.Vs, dst.Vs)):
        assert torch.equal(x[:, :L], y[:, :L])


@pytest.mark.parametrize("mode", ["f16", "q8"])
def test_sink_mode_ring_equals_compacted(ops, mode):
    """Version-2 snapshot: a ring cache after evictions gives the bytes of the reference's
    compacted cache (logical order, unroped keys), and restoring it into a fresh ring reproduces
    the rope-at-read attention output."""
    from bitgpu_b200.snapshot import restore_cache, save_cache
    rng = np.random.default_rng(13)
    B, H, KV, D, SINKS, MAX = 1, 16, 8, 128, 4, 132
    c, s = OR.synth_rope(D, MAX, 1e6, "yarn", 4.0, 8192)
    cos_t, sin_t = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
    ring = ops.KVCache(B, MAX, KV, D, mode=mode, sinks=SINKS, window=MAX - SINKS)
    lin = ops.KVCache(B, MAX, KV, D, mode=mode, sinks=SINKS)
    fill = 0
    for _ in range(300):
        f_r, f_l = ring.evict_for(fill, 1, MAX), lin.evict_for(fill, 1, MAX)
        assert f_r == f_l
        fill = f_r
        k = torch.from_numpy(rand(rng, B, 1, KV, D)).cuda()
        v = torch.from_numpy(rand(rng, B, 1, KV, D)).cuda()
        ring.append_kv(k, v, fill)
        lin.append_kv(k, v, fill)
        fill += 1
    assert ring.ring_head != 0
    roll = {"sinkTokens": SINKS, "cacheLen": fill}
    ids = list(range(400))
    sr = save_cache([ring], ids, mode, dict(MODEL, layers=1), roll=roll)
    sl = save_cache([lin], ids, mode, dict(MODEL, layers=1), roll=roll)
    assert sr["version"] == 2 and sr["data"] == sl["data"] == packed_reference_bytes(lin, 0, 0, fill)
    back = ops.KVCache(B, MAX, KV, D, mode=mode, sinks=SINKS, window=MAX - SINKS)
    back.ring_head = 77
    restore_cache(sr, [back], mode, dict(MODEL, layers=1), max_seq_len=MAX, sinks=SINKS)
    assert back.ring_head == 0
    q = torch.from_numpy(rand(rng, B, 1, H, D)).cuda()
    a = ops.attention(q, ring, fill - 1, cos_t=cos_t, sin_t=sin_t)
    b = ops.attention(q, back, fill - 1, cos_t=cos_t, sin_t=sin_t)
    assert (a - b).abs().max().item() <= 5e-4


def test_hybrid_states_appended(ops):
    """Hybrid: full-attention K/V first, then each linear layer's DeltaNet + conv state."""
    from bitgpu_b200.snapshot import restore_cache, save_cache
    rng = np.random.default_rng(9)
    KV, D, L = 2, 256, 12
    att = ops.KVCache(1, 32, KV, D, mode="f32")
    att.append_kv(torch.from_numpy(rand(rng, 1, L, KV, D)).cuda(), torch.from_numpy(rand(rng, 1, L, KV, D)).cuda(), 0)
    states = [(torch.randn(4, 128, 128, device="cuda"), torch.randn(3, 640, device="cuda")) for _ in range(3)]
    model = {"layers": 4, "kvHeads": KV, "headDim": D, "hidden": 256, "vocab": 256}
    snap = save_cache([att], list(range(L + 1)), "f32", model, linear_states=states)
    tail = b"".join(t.cpu().numpy().tobytes() for st in states for t in st)
    assert snap["data"] == packed_reference_bytes(att, 0, 0, L) + tail
    att2 = ops.KVCache(1, 32, KV, D, mode="f32")
    states2 = [(torch.zeros_like(a), torch.zeros_like(b)) for a, b in states]
    restore_cache(snap, [att2], "f32", model, max_seq_len=32, linear_states=states2)
    assert torch.equal(att.K[:, :L], att2.K[:, :L])
    for (a, b), (c, d) in zip(states, states2):
        assert torch.equal(a, c) and torch.equal(b, d)
