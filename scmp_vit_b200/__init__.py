"""scmp_vit_b200 -- B200-native stochastic-computing matmul engine.

Host side mirrors the reference's Python API (``scmp_kernels.sc``,
``scmp_kernels.mp``, ``sc_integration.*``); the arithmetic runs in
hand-written sm_100a CUDA behind the C ABI of ``include/scmp_b200.h``.
"""
from __future__ import annotations

__version__ = "0.1.0"

from .sc import sc_matmul  # noqa: E402,F401
