"""Helpers shared by the GPU parity tests: seeded inputs, caches filled through the oracle's
codec (so GPU and CPU consume identical bytes), and the reference's pass gate."""
import numpy as np
import torch

from oracle import kvcodec

TOL = 2e-3  # attention / DeltaNet max-abs bar (scripts/verify-kernels.mjs:104)


def rand(rng, *shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float32)


def fill_cache(cache, Kraw, Vraw, fill=None):
    """Encode logical rows ``Kraw/Vraw[B, L, KV, D]`` with the oracle codec, store them in the
    device cache at their physical rows (ring mapping honoured) and return the float32 values
    the kernels must reconstruct at read (``[B, L, KV, D]``)."""
    mode = cache.mode
    B, L = Kraw.shape[:2]
    rows = cache.logical_rows(L).numpy()
    outs = []
    for raw, data, sc in ((Kraw, cache.K, cache.Ks), (Vraw, cache.V, cache.Vs)):
        enc, s = kvcodec.encode(mode, raw)
        dev = torch.from_numpy(np.ascontiguousarray(enc.view(np.int8) if mode in ("q8", "q8r") else enc))
        data[:, rows] = dev.to(data.device)
        if s is not None:
            sc[:, rows] = torch.from_numpy(s).to(sc.device)
        outs.append(kvcodec.decode(mode, enc, s))
    return outs


def gate_ok(out, exp, tol=TOL, cos_min=0.99999):
    out = np.asarray(out, np.float64).ravel()
    exp = np.asarray(exp, np.float64).ravel()
    mad = float(np.abs(out - exp).max())
    cos = float(out @ exp / (np.linalg.norm(out) * np.linalg.norm(exp) + 1e-9))
    return mad < tol and cos > cos_min, mad, cos
