"""bg_attention_noalloc: the attention entry point for callers that cannot allocate device memory
(their device memory belongs to another allocator, or their token loop must not call cudaMalloc).
It keeps its scratch in a fixed 8 MiB array inside the library instead of taking a workspace.

Checked through the C ABI against bg_attention (the entry point that takes a caller workspace) on
two calls in a row with different shapes and data, so contents left in the shared array by one
call cannot leak into the next.  This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _call_pair(L, ops, mode, B, S, H, KV, D, pos_base, seed, gated):
    from bitgpu_b200._lib import AttnParams, DT_F32
    g = torch.Generator(device="cuda").manual_seed(seed)
    cache = ops.KVCache(B, pos_base + S + 3, KV, D, mode=mode)
    cache.append(0, torch.randn((B, pos_base + S, KV, D), generator=g, device="cuda"), 0)
    cache.append(1, torch.randn((B, pos_base + S, KV, D), generator=g, device="cuda"), 0)
    q = torch.randn((B, S, H, D), generator=g, device="cuda")
    gate = torch.randn((B, S, H, D), generator=g, device="cuda") if gated else None
    p = AttnParams(S, H, KV, D, pos_base, pos_base + S)
    d = cache.desc()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    gp = C.c_void_p(gate.data_ptr()) if gated else None
    ref = torch.empty_like(q)
    ws = torch.empty(max(L.bg_attention_workspace_size(C.byref(p), B), 1), dtype=torch.uint8, device="cuda")
    rc = L.bg_attention(C.byref(p), B, C.c_void_p(q.data_ptr()), DT_F32, C.byref(d), None, None, 0.0, gp,
                        C.c_void_p(ref.data_ptr()), DT_F32, C.c_void_p(ws.data_ptr()), ws.numel(), stream)
    assert rc == 0
    out = torch.full_like(q, float("nan"))
    rc = L.bg_attention_noalloc(C.byref(p), B, C.c_void_p(q.data_ptr()), DT_F32, C.byref(d), None, None, 0.0, gp,
                                C.c_void_p(out.data_ptr()), DT_F32, stream)
    assert rc == 0
    torch.cuda.synchronize()
    a, b = out.cpu().numpy(), ref.cpu().numpy()
    assert np.isfinite(a).all()
    assert np.abs(a - b).max() < TOL


def test_noalloc_matches_workspace_entry_point_twice():
    from bitgpu_b200 import ops
    from bitgpu_b200._lib import lib
    L = lib()
    _call_pair(L, ops, "f16", B=4, S=1, H=32, KV=8, D=128, pos_base=4095, seed=1, gated=False)
    # second call: different shape, cache codec and gate; reuses the same scratch array
    _call_pair(L, ops, "q8", B=1, S=3, H=24, KV=4, D=256, pos_base=2000, seed=2, gated=True)


def test_noalloc_rejects_oversized_scratch(monkeypatch):
    """A call whose split partials would exceed the fixed scratch (bg_attention_noalloc_limit(),
    8 MiB) is refused (BG_ENOMEM) before any launch.  The split-count override forces 64 splits of
    2048 rows (68 MB of partials)."""
    from bitgpu_b200 import ops
    from bitgpu_b200._lib import AttnParams, BG_ENOMEM, DT_F32, lib
    L = lib()
    monkeypatch.setenv("BGATTN_NSPLIT", "64")
    B, S, H, KV, D = 64, 1, 32, 8, 128
    p = AttnParams(S, H, KV, D, 32767, 32768)
    assert L.bg_attention_noalloc_limit() == 8 << 20
    assert L.bg_attention_workspace_size(C.byref(p), B) > L.bg_attention_noalloc_limit()
    cache = ops.KVCache(1, 8, KV, D, mode="f16")
    d = cache.desc()
    rc = L.bg_attention_noalloc(C.byref(p), B, C.c_void_p(1), DT_F32, C.byref(d), None, None, 0.0, None,
                                C.c_void_p(1), DT_F32, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == BG_ENOMEM
