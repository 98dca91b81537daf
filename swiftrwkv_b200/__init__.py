"""B200 (sm_100a) implementation of SwiftRWKV's two hot paths.

* WKV-7 recurrence: forward, training forward with checkpoints, backward,
  one-token decode step and fused tail (``swiftrwkv_b200.kernel``, mirroring
  Sources/RWKVKernel).
* Quantised-weight dequant / GEMV: the MLX affine container of the QLoRA base
  and the .rwkvq sb6 / sym formats (``swiftrwkv_b200.quant``).

Everything computes in ``librwkvcuda.so`` (hand-written CUDA, C ABI in
``include/rwkv_cuda.h``), loaded through ctypes by ``swiftrwkv_b200._lib``.
"""
from ._lib import LIB_PATH, RWKVError, lib  # noqa: F401

__all__ = ["LIB_PATH", "RWKVError", "lib"]
