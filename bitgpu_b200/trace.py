"""Per-CTA timing trace of the head_dim-256 decode and the split-KV exchange step.

Needs a trace build of the library (the shipped one has no trace), loaded through BGATTN_LIB:

    python -m bitgpu_b200.build --trace /tmp/libbgattn_trace.so
    BGATTN_LIB=/tmp/libbgattn_trace.so python -m bitgpu_b200.trace 16384 131072
    BGATTN_LIB=/tmp/libbgattn_trace.so python -m torch.distributed.run --nproc-per-node 2 \\
        --master-addr 127.0.0.1 -m bitgpu_b200.trace --peer 131072

The decode kernel records, per CTA, %globaltimer stamps at entry, first tile ready, loop end and
partials written; the exchange kernel records, per row, entry, local merge done, counters raised,
every rank's row arrived and output written.  Times print in microseconds from the first decode
CTA's entry of the last call.  Shapes are config 5b's (24 query / 4 kv heads, head_dim 256, f16).
"""
import ctypes as C
import os
import sys

import numpy as np
import torch

H, KV, D = 24, 4, 256


def _fill(ops, n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    cache = ops.KVCache(1, n, KV, D, mode="f16", device="cuda")
    for p0 in range(0, n, 8192):
        m = min(8192, n - p0)
        for w in (0, 1):
            cache.append(w, torch.randn((1, m, KV, D), generator=g, device="cuda"), p0)
    return cache


def _read(lib, name, n):
    fn = getattr(lib, name)
    fn.argtypes = [C.c_void_p, C.c_size_t]
    buf = (C.c_ulonglong * n)()
    if fn(buf, n) != 0:
        raise RuntimeError(f"{name} failed")
    return np.array(buf, dtype=np.int64)


def decode_trace(ctxs):
    from . import lib, ops
    L = lib()
    if not hasattr(L, "bg_trace_read"):
        raise RuntimeError("not a trace build: set BGATTN_LIB to a library built with --trace")
    for ctx in ctxs:
        cache = _fill(ops, ctx, 1)
        gq = torch.Generator(device="cuda").manual_seed(2)
        q = torch.randn((1, 1, H, D), generator=gq, device="cuda")
        gate = torch.randn((1, 1, H, D), generator=gq, device="cuda")
        out = torch.empty_like(q)
        for _ in range(5):
            ops.attention(q, cache, ctx - 1, scale=D ** -0.5, gate=gate, out=out)
        torch.cuda.synchronize()
        a = _read(L, "bg_trace_read", 148 * 8).reshape(148, 8)
        t0 = a[:, 0].min()
        print(f"ctx {ctx}")
        for name, c in (("entry", 0), ("first tile", 1), ("loop end", 2), ("partials", 5)):
            r = (a[:, c] - t0) / 1e3
            print(f"  {name:10s} min {r.min():7.2f} med {np.median(r):7.2f} max {r.max():7.2f} us")
        del cache


def peer_trace(ctx):
    import torch.distributed as dist
    from . import lib, ops
    from .splitkv import SplitKVDecoder
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl")
    L = lib()
    dec = SplitKVDecoder(ctx)
    cache = _fill(ops, dec.hi - dec.lo, 11 + rank)
    gq = torch.Generator(device="cuda").manual_seed(12)
    q = torch.randn((1, 1, H, D), generator=gq, device="cuda")
    gate = torch.randn((1, 1, H, D), generator=gq, device="cuda")
    step = ops.Graphed(lambda: dec.step(q, cache, ctx - 1, gate=gate, scale=D ** -0.5))
    for _ in range(20):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(100):
        step()
    e1.record()
    torch.cuda.synchronize()
    a = _read(L, "bg_trace_read", 148 * 8).reshape(148, 8)
    b = _read(L, "bg_ptrace_read", 512 * 4).reshape(512, 4)
    t0 = a[:, 0].min()
    us = lambda x: (x - t0) / 1e3
    rows = H
    line = (f"rank {rank}: step {e0.elapsed_time(e1) * 10:.1f} us | decode first tile med {np.median(us(a[:, 1])):.1f} "
            f"partials max {us(a[:, 5]).max():.1f} | exchange entry min {us(b[:rows, 0]).min():.1f} "
            f"local merge max {us(b[:rows, 1]).max():.1f} counters max {us(b[:rows, 2]).max():.1f} "
            f"arrived min/max {us(b[256:256 + rows, 0]).min():.1f}/{us(b[256:256 + rows, 0]).max():.1f} "
            f"output max {us(b[:rows, 3]).max():.1f}")
    lines = [None] * dist.get_world_size()
    dist.all_gather_object(lines, line)
    if rank == 0:
        print("\n".join(lines))
    dec.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    args = sys.argv[1:]
    if args and args[0] == "--peer":
        peer_trace(int(args[1]) if len(args) > 1 else 131072)
    else:
        decode_trace([int(x) for x in args] or [16384, 131072])
