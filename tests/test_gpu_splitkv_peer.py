"""Split-KV decode over two GPUs with the peer-memory exchange (config 5b's path): every rank's
partial rows go straight into every rank's gather buffer over NVLink and the merge waits on
arrival counters.  Run as two child processes, one per GPU (skipped with fewer than two GPUs).

* parity: three consecutive steps (both parities of the double-buffered gather slots, the device
  step counter) over f16, q8 and f32 caches equal single-GPU attention over the whole cache, with
  the exchange as push + merge kernels and as the fused epilogue of the tensor-core kernel;
* a CUDA-graph replay of the step gives the same result;
* a rank that skips a step (stays alive, pushes nothing) makes the other rank's merge give up
  after its bounded wait and report BG_ETIMEOUT -- no hang, no fault."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, ret, fused):
    import sys
    os.environ["BGATTN_PEER_FUSED"] = fused   # read once, when the library is first used
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device(f"cuda:{rank}"))
    from bitgpu_b200 import ops
    from bitgpu_b200._lib import BG_ETIMEOUT, lib
    from bitgpu_b200.splitkv import SplitKVDecoder
    H, KV, D, L = 24, 4, 256, 6000
    g = torch.Generator(device="cuda").manual_seed(3)      # identical full cache on every rank
    Kf = torch.randn((1, L, KV, D), generator=g, device="cuda")
    Vf = torch.randn((1, L, KV, D), generator=g, device="cuda")
    errs = []
    decs = []
    # f16 / q8: tensor-core split kernel; f32: CUDA-core split kernel; then the exchange
    for mode in ("f16", "q8", "f32"):
        full = ops.KVCache(1, L, KV, D, mode=mode)
        full.append(0, Kf, 0)
        full.append(1, Vf, 0)
        dec = SplitKVDecoder(L, spin_limit=20000)
        assert dec.exchange == "peer"
        lo, hi = dec.lo, dec.hi
        loc = ops.KVCache(1, hi - lo, KV, D, mode=mode)
        loc.append(0, Kf[:, lo:hi].contiguous(), 0)
        loc.append(1, Vf[:, lo:hi].contiguous(), 0)
        for step in range(3):
            pos = L - 1 - 7 * step                               # a shorter context each step
            q = torch.randn((1, 1, H, D), generator=g, device="cuda")
            gate = torch.randn((1, 1, H, D), generator=g, device="cuda")
            out = dec.step(q, loc, pos, gate=gate, scale=1 / 16)
            ref = ops.attention(q, full, pos, scale=1 / 16, gate=gate)
            errs.append((mode, float((out - ref).abs().max())))
        decs.append(dec)
    dec = decs[0]
    # the same step replayed from a CUDA graph (f16)
    full = ops.KVCache(1, L, KV, D, mode="f16")
    full.append(0, Kf, 0)
    full.append(1, Vf, 0)
    loc = ops.KVCache(1, dec.hi - dec.lo, KV, D, mode="f16")
    loc.append(0, Kf[:, dec.lo:dec.hi].contiguous(), 0)
    loc.append(1, Vf[:, dec.lo:dec.hi].contiguous(), 0)
    q = torch.randn((1, 1, H, D), generator=g, device="cuda")
    gate = torch.randn((1, 1, H, D), generator=g, device="cuda")
    G = ops.Graphed(lambda: dec.step(q, loc, L - 1, gate=gate, scale=1 / 16))
    ref = ops.attention(q, full, L - 1, scale=1 / 16, gate=gate)
    for _ in range(3):
        errs.append(("graph", float((G() - ref).abs().max())))
    status = lib().bg_device_status(None)
    dist.barrier()
    # rank 1 skips the next step's push: rank 0's merge must time out, report it and return
    store = dist.distributed_c10d._get_default_store()
    timeout_rc = None
    if rank == 0:
        ops.attention_peer(q, loc, L - 1, dec.lo, dec.hi, dec.px, scale=1 / 16, gate=gate)
        timeout_rc = lib().bg_device_status(None)
        store.set("rank0_done", "1")
    else:
        store.wait(["rank0_done"])
    ret[rank] = (errs, status, timeout_rc, BG_ETIMEOUT)
    del G
    for d in decs:
        d.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("fused", ["0", "1"])
def test_splitkv_peer_two_gpus(fused):
    """fused "0": split kernel, push kernel, merge kernel (default); "1": the tensor-core kernel
    finishes the step in its last CTA per group."""
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ret, fused)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(2):
        errs, status, _, _ = ret[r]
        assert status == 0, (r, status)
        assert max(e for _, e in errs) < 1e-3, (r, errs)
    _, _, trc, tcode = ret[0]
    assert trc == tcode
