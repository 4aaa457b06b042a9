"""KV-cache storage codecs (f32 / f16 / q8) restated from the reference WGSL.

Layout (reference): one cache row per (position, kv head), row index ``pos*KV + kvh``
(``shaders/attention_sg.wgsl:11-12,32``).

* f16: one f32->f16 rounding at append (``shaders/copy_kv16.wgsl:13``), widened to f32 at
  read (``shaders/attention_sg_kv16.wgsl:1-4,35,41``).
* q8 (reference default, q8_0 style): per 32-element block, scale ``s = max(absmax, 1e-30)``
  (``shaders/copy_kv8.wgsl:30-35``) and code ``pack4x8snorm(v/s)``
  (``copy_kv8.wgsl:39``), i.e. ``floor(0.5 + 127*clamp(v/s,-1,1))`` as int8 (WGSL spec
  definition of pack4x8snorm: ties round up).  Read: ``unpack4x8snorm(code)*s`` =
  ``max(code/127, -1) * s`` (``shaders/attention_sg_kv8.wgsl:40,51``).
  Storage: codes int8 ``[rows, D]`` (== u32 words ``[rows, D/4]`` little-endian, component 0
  in the low byte), scales f32 ``[rows, D/32]``.
* q8_row128 (the BASELINE.json variant, not in the reference): one scale per row of 128,
  ``scale = absmax/127``, ``code = round-half-even(v/scale)`` clamped to +-127,
  read ``code*scale``.  Provided as an explicit extra mode only.
"""
import numpy as np

F32 = np.float32


def f16_round(x):
    return np.asarray(x, F32).astype(np.float16)


def f16_read(x16):
    return np.asarray(x16, np.float16).astype(F32)


def q8_encode(rows):
    """rows ``[..., D]`` f32 -> (codes int8 ``[..., D]``, scales f32 ``[..., D/32]``)."""
    x = np.asarray(rows, F32)
    D = x.shape[-1]
    assert D % 32 == 0
    xb = x.reshape(x.shape[:-1] + (D // 32, 32))
    s = np.maximum(np.abs(xb).max(-1), F32(1e-30)).astype(F32)
    e = (xb / s[..., None]).astype(F32)
    e = np.clip(e, F32(-1.0), F32(1.0))
    codes = np.floor(F32(0.5) + F32(127.0) * e).astype(np.int8)
    return codes.reshape(x.shape), s


def q8_decode(codes, scales):
    c = np.asarray(codes, np.int8)
    D = c.shape[-1]
    u = np.maximum(c.astype(F32) / F32(127.0), F32(-1.0)).astype(F32)
    ub = u.reshape(c.shape[:-1] + (D // 32, 32))
    return (ub * np.asarray(scales, F32)[..., None]).astype(F32).reshape(c.shape)


def q8r_encode(rows, block=128):
    """BASELINE variant: one absmax/127 scale per ``block`` elements, round-half-even."""
    x = np.asarray(rows, F32)
    D = x.shape[-1]
    xb = x.reshape(x.shape[:-1] + (D // block, block))
    s = (np.abs(xb).max(-1) / F32(127.0)).astype(F32)
    sd = np.where(s > 0, s, F32(1.0)).astype(F32)
    codes = np.clip(np.rint(xb / sd[..., None]), -127, 127).astype(np.int8)
    return codes.reshape(x.shape), s


def q8r_decode(codes, scales, block=128):
    c = np.asarray(codes, np.int8)
    D = c.shape[-1]
    cb = c.reshape(c.shape[:-1] + (D // block, block)).astype(F32)
    return (cb * np.asarray(scales, F32)[..., None]).astype(F32).reshape(c.shape)


def encode(mode, rows):
    """Encode f32 rows into the storage of ``mode`` ('f32'|'f16'|'q8'|'q8r').
    Returns (data, scales-or-None)."""
    if mode == "f32":
        return np.asarray(rows, F32).copy(), None
    if mode == "f16":
        return f16_round(rows), None
    if mode == "q8":
        return q8_encode(rows)
    if mode == "q8r":
        return q8r_encode(rows)
    raise ValueError(mode)


def decode(mode, data, scales=None):
    if mode == "f32":
        return np.asarray(data, F32)
    if mode == "f16":
        return f16_read(data)
    if mode == "q8":
        return q8_decode(data, scales)
    if mode == "q8r":
        return q8r_decode(data, scales)
    raise ValueError(mode)
