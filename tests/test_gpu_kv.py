"""GPU parity: KV writers (append, fused RMSNorm+RoPE+write) and sink eviction."""
import numpy as np
import pytest
import torch

from gpu_util import fill_cache, gate_ok, rand
from oracle import attention as OA
from oracle import evict as OE
from oracle import kvcodec
from oracle import rope as OR

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from bitgpu_b200 import ops
    return ops


@pytest.mark.parametrize("mode", ["f32", "f16", "q8", "q8r"])
@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("src_f16", [False, True])
def test_append_bit_exact(ops, mode, D, src_f16):
    """copy.wgsl / copy_kv16.wgsl / copy_kv8.wgsl: stored bytes equal the oracle codec's."""
    if mode == "q8r" and D % 128:
        pytest.skip()
    rng = np.random.default_rng(D + 3 * src_f16)
    B, S, KV, pos0 = 3, 7, 4, 11
    src = rand(rng, B, S, KV, D, scale=3.0)
    src[0, 1, 2, :32] = 0.0       # an all-zero q8 block
    if src_f16:
        src = src.astype(np.float16).astype(np.float32)
    cache = ops.KVCache(B, pos0 + S + 2, KV, D, mode=mode)
    t = torch.from_numpy(src).cuda()
    cache.append(0, t.half() if src_f16 else t, pos0)
    cache.append(1, (-t).half() if src_f16 else -t, pos0)
    enc, s = kvcodec.encode(mode, src)
    encv, sv = kvcodec.encode(mode, -src)
    got = cache.K[:, pos0:pos0 + S].cpu().numpy()
    assert np.array_equal(got.view(np.uint8) if mode in ("q8", "q8r") else got,
                          enc.view(np.uint8) if mode in ("q8", "q8r") else enc)
    gotv = cache.V[:, pos0:pos0 + S].cpu().numpy()
    assert np.array_equal(gotv.view(np.uint8) if mode in ("q8", "q8r") else gotv,
                          encv.view(np.uint8) if mode in ("q8", "q8r") else encv)
    if s is not None:
        assert np.array_equal(cache.Ks[:, pos0:pos0 + S].cpu().numpy(), s)
        assert np.array_equal(cache.Vs[:, pos0:pos0 + S].cpu().numpy(), sv)
    # rows outside the written range untouched
    assert not cache.K[:, :pos0].float().abs().sum().item()


@pytest.mark.parametrize("mode", ["f32", "f16", "q8"])
@pytest.mark.parametrize("rope", [True, False])
def test_rmsnorm_rope_write(ops, mode, rope):
    """rmsnorm_rope_sg{,_kv16,_kv8}.wgsl: normed+roped K straight into the cache at `pos`."""
    rng = np.random.default_rng(11)
    B, KV, D, pos, eps = 2, 8, 128, 37, 1e-6
    x = rand(rng, B, KV, D)
    gamma = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    c, s = OR.synth_rope(D, 64, 1e6, "yarn", 4.0, 8192)
    cf = np.concatenate([c[pos], c[pos]]).astype(np.float32)
    sf = np.concatenate([s[pos], s[pos]]).astype(np.float32)
    inv = np.float32(1.0) / np.sqrt((x * x).sum(-1, keepdims=True) / np.float32(D) + np.float32(eps))
    nd = (x * inv * gamma).astype(np.float32)
    exp = OR.rope_rotate_half(nd, cf, sf) if rope else nd
    cache = ops.KVCache(B, 64, KV, D, mode=mode)
    y = torch.empty(B, KV, D, device="cuda")
    cache.write_normed_k(torch.from_numpy(x).cuda(), torch.from_numpy(gamma).cuda(), eps, pos,
                         cos=torch.from_numpy(cf).cuda() if rope else None,
                         sin=torch.from_numpy(sf).cuda() if rope else None, y=y)
    assert np.abs(y.cpu().numpy() - exp).max() < 1e-5
    # the cache holds the codec of the kernel's own f32 result (bit-exact encode)
    enc, sc = kvcodec.encode(mode, y.cpu().numpy())
    got = cache.K[:, pos].cpu().numpy()
    assert np.array_equal(got.view(np.uint8) if mode == "q8" else got, enc.view(np.uint8) if mode == "q8" else enc)
    if sc is not None:
        assert np.array_equal(cache.Ks[:, pos].cpu().numpy(), sc)


@pytest.mark.parametrize("mode", ["f16", "q8"])
def test_evict_compaction_matches_engine(ops, mode):
    """bg_kv_evict moves rows exactly like engine.ts:1188-1212 (scales included)."""
    rng = np.random.default_rng(12)
    B, KV, D, SINKS, MAX = 2, 2, 128, 4, 100
    cache = ops.KVCache(B, MAX, KV, D, mode=mode, sinks=SINKS)
    Kraw, Vraw = rand(rng, B, MAX, KV, D), rand(rng, B, MAX, KV, D)
    fill_cache(cache, Kraw, Vraw)
    before = [t.clone() for t in (cache.K, cache.V) + ((cache.Ks, cache.Vs) if cache.Ks is not None else ())]
    lw = OE.LogicalWindow(SINKS, MAX)
    lw.append(range(MAX))
    nf = cache.evict_for(MAX, 1, MAX)
    lw.append([-1])
    assert nf == lw.fill - 1
    src_rows = torch.tensor(lw.slots[:nf])
    after = [cache.K, cache.V] + ([cache.Ks, cache.Vs] if cache.Ks is not None else [])
    for b0, a0 in zip(before, after):
        assert torch.equal(a0[:, :nf], b0[:, src_rows])


def test_ring_equals_compaction(ops):
    """Attention over a ring cache after ring evictions == over a compacted linear cache.

    Both caches hold the same bytes per logical slot; the rope-at-read kernel cuts its tiles at
    the ring's physical discontinuities, so the two summation orders (and the f16 rounding of the
    softmax weights against different running maxima) may differ at the kernel's rounding level,
    ~1e-4; a layout error would show as O(0.1)."""
    rng = np.random.default_rng(13)
    B, H, KV, D, SINKS, MAX = 2, 16, 8, 128, 4, 132
    c, s = OR.synth_rope(D, MAX, 1e6, "yarn", 4.0, 8192)
    cos_t, sin_t = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
    ring = ops.KVCache(B, MAX, KV, D, mode="q8", sinks=SINKS, window=MAX - SINKS)
    lin = ops.KVCache(B, MAX, KV, D, mode="q8", sinks=SINKS)
    fill = 0
    for step in range(300):
        fill_r = ring.evict_for(fill, 1, MAX)
        fill_l = lin.evict_for(fill, 1, MAX)
        assert fill_r == fill_l
        fill = fill_r
        k = torch.from_numpy(rand(rng, B, 1, KV, D)).cuda()
        v = torch.from_numpy(rand(rng, B, 1, KV, D)).cuda()
        for cc in (ring, lin):
            cc.append(0, k, fill)
            cc.append(1, v, fill)
        fill += 1
        if step % 37 == 0 or step == 299:
            q = torch.from_numpy(rand(rng, B, 1, H, D)).cuda()
            a = ops.attention(q, ring, fill - 1, cos_t=cos_t, sin_t=sin_t)
            b = ops.attention(q, lin, fill - 1, cos_t=cos_t, sin_t=sin_t)
            err = (a - b).abs().max().item()
            assert err <= 5e-4, (step, err)
    assert ring.ring_head != 0


def test_roll_stream_vs_oracle(ops):
    """Short sink-mode stream (q8, 4 sinks) checked against the oracle at sampled steps."""
    rng = np.random.default_rng(14)
    B, H, KV, D, SINKS, MAX = 1, 16, 8, 128, 4, 100
    c, s = OR.synth_rope(D, MAX, 1e6, "yarn", 4.0, 8192)
    cos_t, sin_t = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
    ring = ops.KVCache(B, MAX, KV, D, mode="q8", sinks=SINKS, window=MAX - SINKS)
    lw = OE.LogicalWindow(SINKS, MAX)
    toks = {}
    fill = 0
    for step in range(260):
        fill = ring.evict_for(fill, 1, MAX)
        lw.append([step])
        assert lw.fill == fill + 1
        kv = rand(rng, 2, B, 1, KV, D)
        toks[step] = kvcodec.q8_decode(*kvcodec.q8_encode(kv))
        ring.append(0, torch.from_numpy(kv[0]).cuda(), fill)
        ring.append(1, torch.from_numpy(kv[1]).cuda(), fill)
        fill += 1
        if step in (50, 99, 100, 101, 175, 176, 259):
            q = rand(rng, B, 1, H, D)
            out = ops.attention(torch.from_numpy(q).cuda(), ring, fill - 1, cos_t=cos_t, sin_t=sin_t)
            Kl = np.concatenate([toks[t][0][0] for t in lw.slots])
            Vl = np.concatenate([toks[t][1][0] for t in lw.slots])
            exp = OA.attend(q[0], OA.rotate_keys_at_read(Kl, c, s), Vl, fill - 1)
            ok, mad, cos_ = gate_ok(out[0].cpu().numpy(), exp)
            assert ok, (step, mad, cos_)


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("modes", [("f16", "q8"), ("f32", "q8r"), ("q8", "f16")])
def test_append_kv_pair_equals_two_appends(ops, D, modes):
    """bg_kv_append_kv_pair writes the same bytes as one bg_kv_append_kv per cache (codecs, scales,
    a ring cache's wrap and an f16 source included)."""
    if "q8r" in modes and D % 128:
        pytest.skip("q8r needs head_dim % 128")
    B, S, KV, pos0 = 3, 37, 4, 11
    g = torch.Generator(device="cuda").manual_seed(D)
    k = torch.randn((B, S, KV, D), generator=g, device="cuda").half()
    v = torch.randn((B, S, KV, D), generator=g, device="cuda").half()
    mk = lambda m: ops.KVCache(B, 0, KV, D, mode=m, sinks=4, window=60)
    a0, a1, b0, b1 = mk(modes[0]), mk(modes[1]), mk(modes[0]), mk(modes[1])
    for c in (a0, a1, b0, b1):
        c.ring_head = 50
    a0.append_kv_pair(a1, k, v, pos0)
    b0.append_kv(k, v, pos0)
    b1.append_kv(k, v, pos0)
    for x, y in ((a0, b0), (a1, b1)):
        assert torch.equal(x.K, y.K) and torch.equal(x.V, y.V)
        if x.Ks is not None:
            assert torch.equal(x.Ks, y.Ks) and torch.equal(x.Vs, y.Vs)
