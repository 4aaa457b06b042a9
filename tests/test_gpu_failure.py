"""Failure detection on the device, without a GPU fault: a bounded wait that runs out.

Every mbarrier wait in the library's kernels gives up after a poll limit, records BG_ETIMEOUT and
returns (the reference's counterpart is the engine's device-lost path, engine.ts:400-409).  Here
a self-test kernel waits on a barrier nothing arrives on, with a short caller-set limit, so the
wait expires for certain; the host must then read BG_ETIMEOUT from bg_device_status, the flag
must clear, and the context must still run real work correctly."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_reports_timeout():
    from bitgpu_b200 import ops
    from bitgpu_b200._lib import BG_EINVAL, BG_ETIMEOUT, BG_OK, lib
    L = lib()
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.bg_device_status(st) == BG_OK
    assert L.bg_selftest_wait_expiry(0, st) == BG_EINVAL          # a wait needs a limit
    assert L.bg_selftest_wait_expiry(1000, st) == BG_OK            # launched
    assert L.bg_device_status(st) == BG_ETIMEOUT                   # the wait gave up and said so
    assert L.bg_device_status(st) == BG_OK                         # read-and-clear
    # the context is intact: a decode step after the timeout is still exact
    g = torch.Generator(device="cuda").manual_seed(9)
    cache = ops.KVCache(1, 300, 2, 128, mode="f16")
    for w in (0, 1):
        cache.append(w, torch.randn((1, 300, 2, 128), generator=g, device="cuda"), 0)
    q = torch.randn((1, 1, 8, 128), generator=g, device="cuda")
    out = ops.attention(q, cache, 299).cpu().numpy()
    from oracle import attention as OA
    K = cache.K[0].float().cpu().numpy()
    V = cache.V[0].float().cpu().numpy()
    exp = OA.attend(q[0].cpu().numpy(), K, V, 299)
    assert np.abs(out[0] - exp).max() < 2e-3
    assert L.bg_device_status(st) == BG_OK
