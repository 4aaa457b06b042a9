"""World-size-2 CPU test of the split-KV host path (gloo backend): slicing, the all-gather of
partial rows and the LSE merge reproduce single-device gated attention.  The per-rank kernels are
stood in for by the oracle (the CUDA path is covered by the GPU tests); what runs here is the
collective orchestration of bitgpu_b200.splitkv."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_partials(q, cache, pos_base, lo, hi, scale):
    from oracle import attention as OA
    K, V = cache
    qn = q.numpy()
    rows = []
    for b in range(qn.shape[0]):
        m, l, o = OA.attend_partials(qn[b], K[b], V[b], pos_base, lo, hi, scale=scale or None)
        rows.append(np.concatenate([o, m[..., None] * 1.0, l[..., None]], -1).reshape(-1, o.shape[-1] + 2))
    return torch.from_numpy(np.concatenate(rows).astype(np.float32))


def _oracle_merge(gathered, out_shape, gate):
    from oracle import attention as OA
    g = gathered.numpy()
    D = g.shape[-1] - 2
    out = OA.lse_merge([x[:, D] for x in g], [x[:, D + 1] for x in g], [x[:, :D] for x in g])
    out = out.reshape(out_shape)
    if gate is not None:
        out = out / (1 + np.exp(-gate.numpy()))
    return torch.from_numpy(out.astype(np.float32))


def _worker(rank, world, port, L, q, K, V, gate, pos_base, ret):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from bitgpu_b200.splitkv import SplitKVDecoder
    dec = SplitKVDecoder(L, partials_fn=lambda q_, c, pb, lo, hi, sc: _oracle_partials(q_, c, pb, lo, hi, sc),
                         merge_fn=_oracle_merge)
    lo, hi = dec.lo, dec.hi
    local = (np.ascontiguousarray(K[:, :]), np.ascontiguousarray(V[:, :]))  # oracle reads absolute positions
    out = dec.step(torch.from_numpy(q), local, pos_base, gate=torch.from_numpy(gate))
    ret[rank] = (lo, hi, out.numpy())
    dist.destroy_process_group()


@pytest.mark.parametrize("L", [1001, 64])
def test_splitkv_two_ranks_matches_single(L):
    from bitgpu_b200.splitkv import split_bounds
    from oracle import attention as OA
    assert split_bounds(10, 3) == [(0, 4), (4, 7), (7, 10)]
    rng = np.random.default_rng(L)
    B, S, H, KV, D = 1, 2, 6, 2, 256
    pos_base = L - S
    q = rng.standard_normal((B, S, H, D)).astype(np.float32)
    K = rng.standard_normal((B, L, KV, D)).astype(np.float32)
    V = rng.standard_normal((B, L, KV, D)).astype(np.float32)
    gate = rng.standard_normal((B, S, H, D)).astype(np.float32)
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    ret = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, L, q, K, V, gate, pos_base, ret)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    exp = OA.attend(q[0], K[0], V[0], pos_base, gate=gate[0])
    (lo0, hi0, o0), (lo1, hi1, o1) = ret[0], ret[1]
    assert (lo0, hi1) == (0, L) and hi0 == lo1
    for o in (o0, o1):                       # every rank ends with the full result
        assert np.abs(o[0] - exp).max() < 1e-5


def _failing_worker(rank, world, port, how, ret):
    """Rank 1 fails between steps (``raise``: an exception ends the process; ``stall``: it stays
    alive but never joins step 2); rank 0 must come back from step 2 with PeerFailure."""
    import datetime
    import sys
    import time
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from bitgpu_b200.splitkv import PeerFailure, SplitKVDecoder
    rng = np.random.default_rng(0)
    L, B, S, H, KV, D = 96, 1, 1, 2, 1, 64
    K = rng.standard_normal((B, L, KV, D)).astype(np.float32)
    V = rng.standard_normal((B, L, KV, D)).astype(np.float32)
    q = torch.from_numpy(rng.standard_normal((B, S, H, D)).astype(np.float32))
    dec = SplitKVDecoder(L, partials_fn=lambda q_, c, pb, lo, hi, sc: _oracle_partials(q_, c, pb, lo, hi, sc),
                         merge_fn=_oracle_merge)
    dec.step(q, (K, V), L - 1)                     # step 1 completes on both ranks
    if rank == 1:
        if how == "raise":
            raise SystemExit(3)                    # the process ends between steps
        time.sleep(30)                             # alive, but never joins step 2
        return
    t0 = time.time()
    try:
        dec.step(q, (K, V), L - 1)
        ret[0] = ("no error", time.time() - t0)
    except PeerFailure as e:
        ret[0] = ("PeerFailure", time.time() - t0, str(e)[:200])
    os._exit(0)                                    # the group is broken; skip its teardown


@pytest.mark.parametrize("how", ["raise", "stall"])
def test_splitkv_peer_failure_is_reported(how):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    ret = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, how, ret)) for r in range(2)]
    for p in procs:
        p.start()
    procs[0].join(90)
    alive = procs[0].is_alive()
    for p in procs:
        if p.is_alive():
            p.kill()
        p.join(10)
    assert not alive, "the surviving rank hung"
    assert ret[0][0] == "PeerFailure", ret.get(0)
    assert ret[0][1] < 60
