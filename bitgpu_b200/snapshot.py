"""KV snapshot save / restore in the reference's wire format (``src/engine.ts:2719-2872``,
``KvSnapshot`` in ``src/types.ts:364-390``).

A snapshot is a plain dict ``{version, kvCache, model, ids, [base], [roll], data}``:

* ``version`` 1 (default mode, roped keys) or 2 (sink mode: unroped keys, rolled window,
  ``roll = {sinkTokens, cacheLen}``);
* ``data`` (bytes): for each KV-bearing layer the K rows, V rows and, under q8, the K and V
  block-scale rows of cache positions ``[base, len)`` in logical order; then, for the hybrid
  model, each linear layer's DeltaNet state and conv left context.  ``len`` is
  ``len(ids) - 1`` (version 1: the last token's K/V is re-written when the conversation
  continues) or ``roll.cacheLen`` (version 2).

The per-layer bytes come from ``bg_kv_snapshot_save`` / ``bg_kv_snapshot_restore``, which gather
the logical order out of a physical ring cache, so snapshots taken here restore in the reference
engine and vice versa.  Validation and its error texts follow ``restoreCache``.
"""
import ctypes as C

import torch

from ._lib import check, lib


class SnapshotError(ValueError):
    pass


def _layer_bytes(cache, count):
    d = cache.desc()
    return int(lib().bg_kv_snapshot_bytes(C.byref(d), cache.KV, cache.D, count))


def save_cache(layers, ids, kv_mode, model, roll=None, base=0, seq=0, linear_states=()):
    """``layers``: the KV-bearing layers' ``KVCache`` objects in layer order; ``ids``: the full
    token history; ``kv_mode``: 'f32' | 'f16' | 'q8'; ``model``: the architecture stamp dict;
    ``roll``: ``{'sinkTokens', 'cacheLen'}`` in sink mode; ``base``: delta start;
    ``linear_states``: ``(deltanet_state, conv_state)`` tensors per linear layer."""
    if len(ids) == 0:
        return None
    n = roll["cacheLen"] if roll else len(ids) - 1
    base = max(0, min(int(base), n))
    if base > 0 and roll:
        raise SnapshotError("saveCache: delta snapshots ({ from }) are not supported under overflow 'sinks'")
    if base > 0 and linear_states:
        raise SnapshotError("saveCache: delta snapshots ({ from }) are not supported for the qwen3_5 hybrid backbone")
    count = n - base
    sizes = [_layer_bytes(c, count) for c in layers]
    extra = [t.numel() * t.element_size() for st in linear_states for t in st]
    data = torch.empty(sum(sizes) + sum(extra), dtype=torch.uint8, pin_memory=True)
    stream = torch.cuda.current_stream()
    off = 0
    for c, sz in zip(layers, sizes):
        d = c.desc()
        check("bg_kv_snapshot_save", lib().bg_kv_snapshot_save(C.byref(d), seq, c.KV, c.D, base, count,
                                                                C.c_void_p(data.data_ptr() + off),
                                                                C.c_void_p(stream.cuda_stream)))
        off += sz
    for st in linear_states:
        for t in st:
            nb = t.numel() * t.element_size()
            data[off:off + nb].copy_(t.contiguous().view(torch.uint8).view(-1), non_blocking=True)
            off += nb
    stream.synchronize()
    snap = {"version": 2 if roll else 1, "kvCache": kv_mode, "model": dict(model), "ids": list(ids),
            "data": bytes(data.numpy().tobytes())}
    if base > 0:
        snap["base"] = base
    if roll:
        snap["roll"] = {"sinkTokens": roll["sinkTokens"], "cacheLen": roll["cacheLen"]}
    return snap


def restore_cache(snap, layers, kv_mode, model, max_seq_len, sinks=None, seq=0, linear_states=(), history=(),
                  cache_len=0):
    """Validate ``snap`` against this engine state and write it into ``layers`` (and the linear
    layers' states).  ``sinks``: the engine's sink count in sink mode, None otherwise;
    ``history`` / ``cache_len``: the current state (checked by delta restores).
    Returns ``(ids, cache_len)`` of the restored conversation."""
    roll = sinks is not None
    if not snap or snap.get("version") not in (1, 2):
        raise SnapshotError(f"restoreCache: unsupported snapshot version {snap.get('version') if snap else None}")
    if (snap["version"] == 2) != roll:
        raise SnapshotError(
            "restoreCache: snapshot was saved under overflow 'sinks' (unroped keys); this engine runs overflow 'error'"
            if snap["version"] == 2 else
            "restoreCache: snapshot was saved under overflow 'error' (roped keys); this engine runs overflow 'sinks'")
    if snap["version"] == 2 and snap.get("roll", {}).get("sinkTokens") != sinks:
        raise SnapshotError(f"restoreCache: snapshot uses {snap.get('roll', {}).get('sinkTokens')} sink tokens but "
                            f"this engine uses {sinks}")
    if snap.get("kvCache") != kv_mode:
        raise SnapshotError(f"restoreCache: snapshot was saved under kvCache '{snap.get('kvCache')}' but this engine "
                            f"runs '{kv_mode}' - snapshots do not convert across modes")
    m = snap.get("model")
    if not m or any(m.get(k) != model.get(k) for k in ("layers", "kvHeads", "headDim", "hidden", "vocab")):
        raise SnapshotError("restoreCache: snapshot is from a different model (architecture mismatch)")
    ids = snap.get("ids")
    if not isinstance(ids, list) or len(ids) == 0:
        raise SnapshotError("restoreCache: snapshot holds no tokens")
    n = snap["roll"]["cacheLen"] if snap["version"] == 2 else len(ids) - 1
    base = max(0, int(snap.get("base", 0) or 0))
    if base > 0 and linear_states:
        raise SnapshotError("restoreCache: delta snapshots are not supported for the qwen3_5 hybrid backbone")
    count = n - base
    need = n + (0 if snap["version"] == 2 else 1)
    if need > max_seq_len:
        raise SnapshotError(f"restoreCache: snapshot needs {need} cache slots but maxSeqLen is {max_seq_len}")
    expect = sum(_layer_bytes(c, count) for c in layers) + \
        sum(t.numel() * t.element_size() for st in linear_states for t in st)
    if len(snap["data"]) != expect:
        raise SnapshotError(f"restoreCache: snapshot data is {len(snap['data'])} bytes, expected {expect}")
    if base > 0:
        if cache_len != base:
            raise SnapshotError(f"restoreCache: delta snapshot expects the cache at position {base} (prewarm the "
                                f"shared prefix first); it is at {cache_len}")
        for i in range(base):
            if history[i] != ids[i]:
                raise SnapshotError(f"restoreCache: delta snapshot prefix does not match the current prewarm "
                                    f"(token {i})")
    data = torch.frombuffer(bytearray(snap["data"]), dtype=torch.uint8).pin_memory() if expect else None
    stream = torch.cuda.current_stream()
    off = 0
    for c in layers:
        if roll:
            c.ring_head = 0  # the snapshot holds the compacted logical order
        sz = _layer_bytes(c, count)
        d = c.desc()
        check("bg_kv_snapshot_restore", lib().bg_kv_snapshot_restore(C.byref(d), seq, c.KV, c.D, base,
                                                                      count, C.c_void_p(data.data_ptr() + off),
                                                                      C.c_void_p(stream.cuda_stream)))
        off += sz
    for st in linear_states:
        for t in st:
            nb = t.numel() * t.element_size()
            t.view(torch.uint8).view(-1).copy_(data[off:off + nb], non_blocking=True)
            off += nb
    stream.synchronize()
    return list(ids), n
