"""KV snapshot format: host-side validation of restoreCache (engine.ts:2808-2848), on CPU."""
import pytest

from bitgpu_b200 import ops
from bitgpu_b200.snapshot import SnapshotError, restore_cache

MODEL = {"layers": 2, "kvHeads": 2, "headDim": 64, "hidden": 128, "vocab": 100}


def layers(mode="q8", sinks=0, window=0):
    return [ops.KVCache(1, 32, 2, 64, mode=mode, sinks=sinks, window=window, device="cpu") for _ in range(2)]


def snap(**kw):
    s = {"version": 1, "kvCache": "q8", "model": dict(MODEL), "ids": [1, 2, 3, 4], "data": b""}
    s.update(kw)
    return s


def bytes_for(L, count):
    from bitgpu_b200.snapshot import _layer_bytes
    return b"\0" * sum(_layer_bytes(c, count) for c in L)


@pytest.mark.parametrize("bad,msg", [
    ({"version": 3}, "unsupported snapshot version 3"),
    ({"version": 2, "roll": {"sinkTokens": 4, "cacheLen": 3}}, "saved under overflow 'sinks'"),
    ({"kvCache": "f16"}, "snapshots do not convert across modes"),
    ({"model": dict(MODEL, headDim=128)}, "different model"),
    ({"ids": []}, "holds no tokens"),
    ({"data": b"\0" * 7}, "snapshot data is 7 bytes"),
])
def test_restore_rejects(bad, msg):
    L = layers()
    with pytest.raises(SnapshotError, match=msg):
        restore_cache(snap(**bad), L, "q8", MODEL, max_seq_len=32)


def test_restore_rejects_sink_mismatch_and_capacity():
    L = layers(sinks=4, window=28)
    s = snap(version=2, roll={"sinkTokens": 2, "cacheLen": 3})
    with pytest.raises(SnapshotError, match="uses 2 sink tokens but this engine uses 4"):
        restore_cache(s, L, "q8", MODEL, max_seq_len=32, sinks=4)
    with pytest.raises(SnapshotError, match="saved under overflow 'error'"):
        restore_cache(snap(), L, "q8", MODEL, max_seq_len=32, sinks=4)
    L = layers()
    with pytest.raises(SnapshotError, match="needs 4 cache slots but maxSeqLen is 3"):
        restore_cache(snap(data=bytes_for(L, 3)), L, "q8", MODEL, max_seq_len=3)


def test_delta_restore_checks_prefix():
    L = layers()
    s = snap(base=2, data=bytes_for(L, 1))
    with pytest.raises(SnapshotError, match="expects the cache at position 2"):
        restore_cache(s, L, "q8", MODEL, max_seq_len=32, history=[1, 2], cache_len=1)
    with pytest.raises(SnapshotError, match=r"prefix does not match the current prewarm \(token 1\)"):
        restore_cache(s, L, "q8", MODEL, max_seq_len=32, history=[1, 9], cache_len=2)


def test_snapshot_bytes_layout_sizes():
    from bitgpu_b200.snapshot import _layer_bytes
    for mode, per in (("f32", 2 * 2 * 64 * 4), ("f16", 2 * 2 * 64 * 2), ("q8", 2 * 2 * 64 + 2 * 2 * 2 * 4)):
        c = ops.KVCache(1, 32, 2, 64, mode=mode, device="cpu")
        assert _layer_bytes(c, 5) == 5 * per   # K, V rows (+ K, V scale rows), engine.ts:2740-2747
