"""B200-native EXL3 trellis-decode matmul backend.

Host side (Python/PyTorch) of ``libexl3b200.so``: the kernels live in
``sglang-exl3_b200/csrc`` behind the C ABI declared in ``include/exl3_b200.h``.
"""

from . import _lib, ops, workspace  # noqa: F401

__all__ = ["ops", "workspace"]
