"""bitgpu_b200 -- B200-native (sm_100a) attention hot path of bitgpu.

``libbgattn.so`` (C ABI, ``include/bgattn.h``) holds the CUDA kernels; ``ops`` is the torch-facing
host mirror of the reference engine's operator surface.  Build with ``python -m bitgpu_b200.build``.
"""
from ._lib import LIB_PATH, BgError, lib  # noqa: F401

__version__ = "0.1.0"
