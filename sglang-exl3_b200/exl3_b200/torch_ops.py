"""``torch.ops.sglang_exl3.*`` registrations over the B200 kernels.

Same op names, schemas and fake (meta) kernels as the reference's registry
(``src/sglang_exl3/ops.py:29-230``), so SGLang's CUDA-graph runner and
``torch.compile`` trace them unchanged.  Each op additionally takes a trailing
``cb: int = -1`` codebook override (0 = 3INST, 1 = MCG, 2 = mul1; -1 keeps the
reference's ``mcg`` mapping).  The real implementations call
``libexl3b200.so``; there is no fallback.
"""

from __future__ import annotations

import logging

import torch

from . import moe as _moe
from . import ops as _ops

logger = logging.getLogger("sglang.exl3.b200.ops")

_REGISTERED = False
NAMESPACE = "sglang_exl3"


def register_custom_ops() -> bool:
    """Register the ops once per process (idempotent)."""
    global _REGISTERED
    if _REGISTERED:
        return True

    @torch.library.custom_op(f"{NAMESPACE}::dequant_trellis", mutates_args=())
    def dequant_trellis(trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, bits: int, mcg: bool,
                        cb: int = -1) -> torch.Tensor:
        return _ops.dequant_trellis(trellis, suh, svh, bits, mcg, cb=None if cb < 0 else cb)

    @dequant_trellis.register_fake
    def _(trellis, suh, svh, bits, mcg, cb=-1):
        return torch.empty((trellis.size(0) * 16, trellis.size(1) * 16), dtype=torch.float16, device=trellis.device)

    @torch.library.custom_op(f"{NAMESPACE}::exl3_gemv", mutates_args=())
    def exl3_gemv(x: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int,
                  mcg: bool, mmode: int = 1, cb: int = -1) -> torch.Tensor:
        return _ops.exl3_gemv(x, trellis, suh, svh, K, mcg, mmode, cb=None if cb < 0 else cb)

    @exl3_gemv.register_fake
    def _(x, trellis, suh, svh, K, mcg, mmode=1, cb=-1):
        out_dim = svh.size(0) if svh.ndim == 1 else trellis.size(1) * 16
        return torch.empty((x.shape[0], out_dim), dtype=x.dtype, device=x.device)

    @torch.library.custom_op(f"{NAMESPACE}::exl3_gemm", mutates_args=())
    def exl3_gemm(x: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int,
                  mcg: bool, cb: int = -1) -> torch.Tensor:
        return _ops.exl3_gemm(x, trellis, suh, svh, K, mcg, cb=None if cb < 0 else cb)

    @exl3_gemm.register_fake
    def _(x, trellis, suh, svh, K, mcg, cb=-1):
        out_dim = svh.size(0) if svh.ndim == 1 else trellis.size(1) * 16
        return torch.empty((x.shape[0], out_dim), dtype=x.dtype, device=x.device)

    @torch.library.custom_op(f"{NAMESPACE}::p2b_gemv_batched", mutates_args=())
    def p2b_gemv_batched(x: torch.Tensor, trellis_ptrs: torch.Tensor, suh_ptrs: torch.Tensor,
                         svh_ptrs: torch.Tensor, expert_indices: torch.Tensor, K: int, mcg: bool,
                         mmode: int = 1, cb: int = -1) -> torch.Tensor:
        return _moe.p2b_gemv_batched(x, trellis_ptrs, suh_ptrs, svh_ptrs, expert_indices, K, mcg, mmode,
                                     cb=None if cb < 0 else cb)

    @p2b_gemv_batched.register_fake
    def _(x, trellis_ptrs, suh_ptrs, svh_ptrs, expert_indices, K, mcg, mmode=1, cb=-1):
        e = expert_indices.numel()
        m = x.size(1) if x.dim() == 3 else x.size(0)
        n = mmode if mmode > 0 else 2048
        return torch.empty((e, m, n), dtype=x.dtype, device=x.device)

    @torch.library.custom_op(f"{NAMESPACE}::p2b_fused_moe", mutates_args=("out",))
    def p2b_fused_moe(x: torch.Tensor, out: torch.Tensor,
                      gate_trellis_ptrs: torch.Tensor, gate_suh_ptrs: torch.Tensor, gate_svh_ptrs: torch.Tensor,
                      up_trellis_ptrs: torch.Tensor, up_suh_ptrs: torch.Tensor, up_svh_ptrs: torch.Tensor,
                      down_trellis_ptrs: torch.Tensor, down_suh_ptrs: torch.Tensor, down_svh_ptrs: torch.Tensor,
                      expert_indices: torch.Tensor, routing_weights: torch.Tensor, K_gate: int, K_up: int,
                      K_down: int, mcg: bool, intermediate_size: int = 2048, swiglu_limit: float = 0.0,
                      cb: int = -1) -> None:
        _moe.p2b_fused_moe(x, out, gate_trellis_ptrs, gate_suh_ptrs, gate_svh_ptrs, up_trellis_ptrs,
                           up_suh_ptrs, up_svh_ptrs, down_trellis_ptrs, down_suh_ptrs, down_svh_ptrs,
                           expert_indices, routing_weights, K_gate, K_up, K_down, mcg, intermediate_size,
                           swiglu_limit, cb=None if cb < 0 else cb)

    @p2b_fused_moe.register_fake
    def _(x, out, *args, **kwargs):
        return None

    @torch.library.custom_op(f"{NAMESPACE}::exl3_fat_gemm", mutates_args=("out",))
    def exl3_fat_gemm(a: torch.Tensor, packed: torch.Tensor, out: torch.Tensor, svh: torch.Tensor, K: int,
                      mcg: bool, mul1: bool, cb: int = -1) -> None:
        _moe.exl3_fat_gemm(a, packed, out, svh, K, mcg, mul1, cb=None if cb < 0 else cb)

    @exl3_fat_gemm.register_fake
    def _(a, packed, out, svh, K, mcg, mul1, cb=-1):
        return None

    @torch.library.custom_op(f"{NAMESPACE}::exl3_fat_gemm_scatter", mutates_args=("out",))
    def exl3_fat_gemm_scatter(a: torch.Tensor, packed: torch.Tensor, out: torch.Tensor, svh: torch.Tensor,
                              token_idx: torch.Tensor, route_weight: torch.Tensor, K: int, mcg: bool,
                              mul1: bool, cb: int = -1) -> None:
        _moe.exl3_fat_gemm_scatter(a, packed, out, svh, token_idx, route_weight, K, mcg, mul1,
                                   cb=None if cb < 0 else cb)

    @exl3_fat_gemm_scatter.register_fake
    def _(a, packed, out, svh, token_idx, route_weight, K, mcg, mul1, cb=-1):
        return None

    _REGISTERED = True
    logger.info("registered torch.ops.%s.* over libexl3b200", NAMESPACE)
    return True
