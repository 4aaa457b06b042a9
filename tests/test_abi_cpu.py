"""CPU checks of the C ABI: the library loads, exports every symbol include/bgattn.h declares,
and its host-only logic (validation, ring eviction bookkeeping) behaves -- no kernel launches."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "bgattn.h")).read()
    return sorted(set(re.findall(r"\b(bg_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def L():
    from bitgpu_b200._lib import lib
    return lib()


def test_exports_match_header(L):
    from bitgpu_b200._lib import EXPORTS
    syms = header_symbols()
    assert syms == sorted(EXPORTS)
    for s in syms:
        assert hasattr(L, s), s


def test_strerror_version(L):
    assert L.bg_version() >= 1
    assert L.bg_strerror(-1) == b"invalid argument"
    assert L.bg_strerror(-5) == b"unsupported shape or mode"


def test_validation_without_launch(L):
    """Bad parameters are rejected before any CUDA call (engine.ts:232-235,372-373)."""
    from bitgpu_b200._lib import AttnParams, KVCacheDesc, BG_EINVAL, BG_EUNSUPPORTED
    kv = KVCacheDesc(1, 1, None, None, 64, 1, 0, 0, 0)
    p = AttnParams(1, 8, 3, 128, 0, 1)                    # H % KV != 0
    rc = L.bg_attention(C.byref(p), 1, C.c_void_p(1), 0, C.byref(kv), None, None, 0.0, None, C.c_void_p(1), 0,
                        None, 0, None)
    assert rc == BG_EINVAL
    p = AttnParams(1, 8, 2, 96, 0, 1)                     # head_dim not built
    assert L.bg_attention(C.byref(p), 1, C.c_void_p(1), 0, C.byref(kv), None, None, 0.0, None, C.c_void_p(1), 0,
                          None, 0, None) == BG_EUNSUPPORTED
    p = AttnParams(2, 8, 2, 128, 5, 6)                    # Ltot != posBase + S
    assert L.bg_attention(C.byref(p), 1, C.c_void_p(1), 0, C.byref(kv), None, None, 0.0, None, C.c_void_p(1), 0,
                          None, 0, None) == BG_EINVAL
    kvq = KVCacheDesc(1, 1, None, None, 64, 2, 0, 0, 0)   # q8 without scale buffers
    p = AttnParams(1, 8, 2, 128, 0, 1)
    assert L.bg_attention(C.byref(p), 1, C.c_void_p(1), 0, C.byref(kvq), None, None, 0.0, None, C.c_void_p(1), 0,
                          None, 0, None) == BG_EINVAL
    p = AttnParams(1, 8, 2, 128, 64, 65)                  # past the cache capacity
    assert L.bg_attention(C.byref(p), 1, C.c_void_p(1), 0, C.byref(kv), None, None, 0.0, None, C.c_void_p(1), 0,
                          None, 0, None) == BG_EINVAL


def test_workspace_size(L):
    from bitgpu_b200._lib import AttnParams
    p = AttnParams(1, 32, 8, 128, 32767, 32768)
    n = L.bg_attention_workspace_size(C.byref(p), 64)
    assert n > 0 and n % (130 * 4) == 0


def test_ring_evict_schedule_matches_engine(L):
    """bg_kv_ring_evict reproduces engine.ts:1188-1212's new fill and advances the head by
    the evicted batch."""
    from bitgpu_b200._lib import KVCacheDesc
    from oracle.evict import evict_plan
    for sinks, mx, fill, need in [(4, 4100, 4100, 1), (4, 100, 100, 1), (4, 100, 100, 500), (1, 65, 65, 3),
                                  (4, 4100, 3000, 2000)]:
        kv = KVCacheDesc(1, 1, None, None, mx, 2, sinks, mx - sinks, 17)
        nf = C.c_uint32()
        assert L.bg_kv_ring_evict(C.byref(kv), fill, need, mx, C.byref(nf)) == 0
        batch, exp = evict_plan(fill, need, sinks, mx)
        assert nf.value == exp
        if exp > sinks:
            assert kv.ring_head == (17 + batch) % (mx - sinks)
