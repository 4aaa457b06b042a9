"""CPU oracle for the bitgpu attention hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (float32 arithmetic, like the reference), the math of
bitgpu's attention / DeltaNet kernels so the CUDA path can be checked against it.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it, and only as the checker or the timed CPU baseline.  The product path
(``bitgpu_b200``) never imports it and has no CPU fallback.

Pinning: ``oracle.deltanet`` (recurrent + chunked delta rule, g/beta, gated norm) and the
head_dim-256 / head_dim-128 causal attention in ``oracle.attention`` are checked against
golden vectors produced by the reference's own numpy code (``tools/qwen35_numpy.py``,
``tools/gen-kernel-cases.py``; see ``tests/golden/make_golden.py``).  The q8 codec, the
rolling-window rope-at-read and the sink-eviction schedule exist only as WGSL/TypeScript in
the reference (no runnable CPU code there), so those restatements are "parity unpinned" at
kernel level: they follow the cited shader / engine lines and are cross-checked for
internal consistency (f32 roll path == plain path before the first eviction, etc.).
"""
from . import attention, deltanet, evict, glue, hybrid, kvcodec, rope  # noqa: F401
