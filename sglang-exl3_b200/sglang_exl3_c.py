"""Drop-in replacement for the reference's compiled module ``sglang_exl3_c``.

The reference's Python layer imports a pybind module of this name
(``src/sglang_exl3/ops.py:20-26``, ``src/sglang_exl3/exl3.py:384-399``) and calls
its functions with the signatures registered in ``csrc/bindings.cpp:169-200``.
This module exposes the same names, signatures and ``P2B_MOE_ABI_VERSION``
attribute, implemented on ``libexl3b200.so``; putting ``sglang-exl3_b200`` on
``sys.path`` ahead of the reference's build makes the reference's plugin run on
the B200 kernels unchanged.  Unlike the reference module there is no CPU path:
CPU tensors raise.
"""

from exl3_b200.moe import (exl3_fat_gemm, exl3_fat_gemm_scatter, p2b_fused_moe,  # noqa: F401
                           p2b_gemv_batched)
from exl3_b200.ops import dequant_trellis, exl3_gemm, exl3_gemv  # noqa: F401

P2B_MOE_ABI_VERSION = 2

__all__ = ["P2B_MOE_ABI_VERSION", "dequant_trellis", "exl3_gemv", "exl3_gemm", "p2b_gemv_batched",
           "p2b_fused_moe", "exl3_fat_gemm", "exl3_fat_gemm_scatter"]
