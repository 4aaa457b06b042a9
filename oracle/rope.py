"""RoPE tables as the reference engine builds them.

``synth_rope`` follows ``src/engine.ts:117-147`` (``synthRope``): per-frequency inverse
wavelengths in float64 (plain or YaRN with beta_fast 32 / beta_slow 1 and
mscale = f32(0.1*ln(factor)+1)), angle = position * inv in float64, one rounding to float32
per table entry.  ``tools/reference.py:120-152`` implements the identical recipe.  Tables are
``[positions, rotary_dim/2]`` float32, the layout the roll attention kernels index as
``cosT[j*half + d%half]`` (``shaders/attention_sg_roll.wgsl:49``).
"""
import math

import numpy as np


def synth_rope(head_dim, positions, rope_theta, rope_type=None, factor=1.0,
               original_max_position_embeddings=0, rotary_dim=None):
    rot = head_dim if rotary_dim is None else rotary_dim
    half = rot // 2
    base = float(rope_theta)
    f = float(factor) if rope_type == "yarn" else 1.0
    j = np.arange(half, dtype=np.float64)
    pf = base ** ((2.0 * j) / rot)
    if f == 1.0:
        inv = 1.0 / pf
        mscale = 1.0
    else:
        orig = float(original_max_position_embeddings)
        lo = max(0, math.floor(rot * math.log(orig / (32 * 2 * math.pi)) / (2 * math.log(base))))
        hi = min(half - 1, math.ceil(rot * math.log(orig / (2 * math.pi)) / (2 * math.log(base))))
        ramp = np.clip((j - lo) / (hi - lo), 0.0, 1.0)
        inv = (1.0 / (f * pf)) * ramp + (1.0 / pf) * (1.0 - ramp)
        mscale = float(np.float32(0.1 * math.log(f) + 1.0))
    ang = np.outer(np.arange(positions, dtype=np.float64), inv)
    return (np.cos(ang) * mscale).astype(np.float32), (np.sin(ang) * mscale).astype(np.float32)


def rope_rotate_half(x, cos_full, sin_full):
    """``x*cos + rotate_half(x)*sin`` with full-width (``[.., D]``) tables, the operand order
    of ``shaders/rmsnorm_rope_sg.wgsl:27-32`` (``nd*cos[i] + rot*sin[i]``)."""
    x = np.asarray(x, np.float32)
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], -1)
    return (x * cos_full + rot * sin_full).astype(np.float32)
