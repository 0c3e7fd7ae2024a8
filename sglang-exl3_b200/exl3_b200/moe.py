"""Routed-MoE and batched-expert EXL3 ops (reference op surface).

``moe_forward`` is the general routed SwiGLU MoE over device pointer tables
(``libexl3b200.exl3b200_moe``: routing, gate/up, SwiGLU, down and the weighted
combine all on the device, no host synchronisation).  The reference-named
functions keep the signatures of ``sglang_exl3_c``
(``csrc/bindings.cpp:149-200``) and of the ``torch.ops.sglang_exl3`` registry
(``src/sglang_exl3/ops.py:96-226``).
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from . import _lib, workspace
from .ops import (_OUT_DTYPES, _require_cuda, _stream_ptr, codebook_id, legacy_codebook, matmul, matmul_combine)

MOE_MAX_PAIRS = 65536
MOE_MAX_EXPERTS = 2048
# average routed rows per local expert from which the tensor-core pipeline is used
# (the kernel-shape map's crossover, exl3b200_select_shape)
MOE_TC_MIN_ROWS = 12


def _table(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.int64 or t.dim() != 1:
        raise RuntimeError(f"{name} must be an int64 pointer table")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    return t.contiguous()


def p2b_gemv_batched(x: torch.Tensor, trellis_ptrs: torch.Tensor, suh_ptrs: torch.Tensor, svh_ptrs: torch.Tensor,
                     expert_indices: torch.Tensor, K: int, mcg: bool, mmode: int = 1,
                     cb: Optional[int] = None, out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """``sglang_exl3_c.p2b_gemv_batched`` (``csrc/p2b_batched.cu:69-101``): for each
    selected expert e, ``x_e @ W[expert_indices[e]]`` -> ``[E, m, N]`` with N =
    mmode (> 0) else 2048, x ``[m, K]`` shared or ``[E, m, K]`` per expert.  Any
    codebook (the reference requires MCG)."""
    if x.dtype != torch.float16:
        raise RuntimeError("batched GEMV requires CUDA fp16")
    ids = expert_indices
    if ids.dtype != torch.int32:
        ids = ids.to(torch.int32)
    ids = ids.contiguous()
    dev = _require_cuda(x, trellis_ptrs, suh_ptrs, svh_ptrs, ids)
    tp = _table(trellis_ptrs, "trellis_ptrs")
    sp = _table(suh_ptrs, "suh_ptrs")
    vp = _table(svh_ptrs, "svh_ptrs")
    e = ids.numel()
    k = x.size(-1)
    per_expert = x.dim() == 3
    m = x.size(1) if per_expert else x.size(0)
    n = int(mmode) if mmode > 0 else 2048
    if K not in (2, 3, 4):
        raise RuntimeError("batched GEMV supports K=2,3,4")
    if per_expert and x.size(0) != e:
        raise RuntimeError("per-expert x must be [E, m, K]")
    x = x.contiguous()
    c = legacy_codebook(mcg, cb)
    out = torch.empty((e, m, n), dtype=out_dtype, device=dev)
    if e == 0:
        return out
    L = _lib.lib()
    with torch.cuda.device(dev):
        state = workspace.state_buffer(dev, L.exl3b200_batched_state_size(e, m, n))
        scratch = workspace.scratch_buffer(dev, L.exl3b200_batched_scratch_size(e, m, k))
        st = L.exl3b200_batched_gemv(x.data_ptr(), int(per_expert), k, m, k, n, int(K), c, tp.data_ptr(),
                                     sp.data_ptr(), vp.data_ptr(), tp.numel(), ids.data_ptr(), e, out.data_ptr(),
                                     _OUT_DTYPES[out_dtype], state.data_ptr(), state.numel(), scratch.data_ptr(),
                                     scratch.numel(), _stream_ptr(dev))
    _lib.check(st, "exl3b200_batched_gemv")
    return out


def workspace_tokens(tokens: int, chunk: int) -> int:
    """Token capacity to size the MoE workspaces for: the next power of two of the
    tokens of one launch (so a captured graph keeps its buffers while batch sizes
    vary below it), at most one chunk."""
    cap = 1
    while cap < min(tokens, chunk):
        cap <<= 1
    return min(cap, chunk)


def moe_path(tokens: int, topk: int, experts: int) -> str:
    """``"tc"`` (tensor-core pipeline, codes decoded once per 256 rows of an expert)
    when the kernel-shape map says so (``MOE_TC_MIN_ROWS`` rows per expert on
    average), else ``"small"``
    (small-M pipeline, once per 16 rows).  ``EXL3_B200_MOE_PATH`` = small / tc
    forces one.  Decided from host-known sizes only (no synchronisation)."""
    forced = os.environ.get("EXL3_B200_MOE_PATH", "auto").lower()
    if forced in ("small", "tc"):
        return forced
    from .ops import select_shape

    shape = select_shape(max(1, tokens), 128, 128, 3, 0, max(1, experts), max(1, topk))
    return "tc" if shape == _lib.SHAPE_MOE_TC else "small"


def moe_forward(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, tables: dict,
                K_gate: int, K_up: int, K_down: int, cb: int, intermediate_size: int,
                swiglu_limit: float = 0.0, out: Optional[torch.Tensor] = None, accumulate: bool = False,
                max_tokens: Optional[int] = None, path: Optional[str] = None) -> torch.Tensor:
    """Routed SwiGLU MoE: ``out[t] (+)= sum_j w[t,j] * down_e(silu(gate_e x_t) * up_e x_t)``.

    ``tables`` holds the nine int64 device pointer tables of the local experts
    (``gate_trellis`` ... ``down_svh``, as built by ``build_exl3_fused_state``,
    ``src/sglang_exl3/exl3.py:579-607``).  Ids outside ``[0, E)`` are skipped.
    ``path``: ``"small"``, ``"tc"`` or None (``moe_path``).  Returns fp32 ``[T, H]``."""
    if x.dim() != 2 or x.dtype != torch.float16:
        raise RuntimeError("MoE input must be fp16 [tokens, hidden]")
    T, H = x.shape
    ids = topk_ids.reshape(T, -1)
    topk = ids.size(1)
    ids = ids.to(torch.int32).contiguous()
    w = topk_weights.reshape(T, topk).to(torch.float32).contiguous()
    names = ("gate_trellis", "gate_suh", "gate_svh", "up_trellis", "up_suh", "up_svh",
             "down_trellis", "down_suh", "down_svh")
    tabs = [_table(tables[nm], nm) for nm in names]
    E = tabs[0].numel()
    if any(t.numel() != E for t in tabs):
        raise RuntimeError("MoE pointer tables must be equally sized")
    dev = _require_cuda(x, ids, w, *tabs)
    if max_tokens is None:
        max_tokens = T
    if T > max_tokens or max_tokens * topk > MOE_MAX_PAIRS:
        raise RuntimeError(f"fused MoE supports tokens * topk <= {MOE_MAX_PAIRS}")
    if E > MOE_MAX_EXPERTS:
        raise RuntimeError(f"fused MoE supports at most {MOE_MAX_EXPERTS} local experts")
    x = x if (x.stride(-1) == 1 and x.stride(0) % 2 == 0) else x.contiguous()
    if out is None:
        if accumulate:
            raise RuntimeError("accumulate needs an output tensor")
        out = torch.empty((T, H), dtype=torch.float32, device=dev)
    if out.dtype != torch.float32 or out.dim() != 2 or out.stride(-1) != 1 or out.size(0) < T:
        raise RuntimeError("MoE output must be float32 [tokens, hidden]")
    L = _lib.lib()
    path = path or moe_path(T, topk, E)
    if path == "tc":
        if out.data_ptr() % 16 or out.stride(0) % 4:
            raise RuntimeError("tensor-core MoE output must be 16-byte aligned with a row stride multiple of 4")
        with torch.cuda.device(dev):
            nbytes = L.exl3b200_moe_tc_scratch_size(max_tokens, topk, E, H, intermediate_size)
            scratch = workspace.scratch_buffer(dev, nbytes)
            st = L.exl3b200_moe_tc(x.data_ptr(), x.stride(0), T, H, intermediate_size, ids.data_ptr(), w.data_ptr(),
                                   topk, E, *[t.data_ptr() for t in tabs], int(K_gate), int(K_up), int(K_down),
                                   int(cb), float(swiglu_limit if swiglu_limit is not None else 0.0), out.data_ptr(),
                                   out.stride(0), int(accumulate), int(max_tokens), scratch.data_ptr(),
                                   scratch.numel(), _stream_ptr(dev))
        _lib.check(st, "exl3b200_moe_tc")
        return out
    if path != "small":
        raise RuntimeError(f"unknown MoE path {path!r}")
    with torch.cuda.device(dev):
        state = workspace.state_buffer(dev, L.exl3b200_moe_state_size(max_tokens, topk, H, intermediate_size))
        scratch = workspace.scratch_buffer(dev, L.exl3b200_moe_scratch_size(max_tokens, topk, H, intermediate_size))
        st = L.exl3b200_moe(x.data_ptr(), x.stride(0), T, H, intermediate_size, ids.data_ptr(), w.data_ptr(), topk, E,
                            *[t.data_ptr() for t in tabs], int(K_gate), int(K_up), int(K_down), int(cb),
                            float(swiglu_limit if swiglu_limit is not None else 0.0), out.data_ptr(), out.stride(0),
                            int(accumulate), int(max_tokens), state.data_ptr(), state.numel(), scratch.data_ptr(),
                            scratch.numel(), _stream_ptr(dev))
    _lib.check(st, "exl3b200_moe")
    return out


def p2b_fused_moe(x: torch.Tensor, out: torch.Tensor, gate_trellis_ptrs, gate_suh_ptrs, gate_svh_ptrs,
                  up_trellis_ptrs, up_suh_ptrs, up_svh_ptrs, down_trellis_ptrs, down_suh_ptrs, down_svh_ptrs,
                  expert_indices: torch.Tensor, routing_weights: torch.Tensor, K_gate: int, K_up: int, K_down: int,
                  mcg: bool, intermediate_size: int = 2048, swiglu_limit: float = 0.0,
                  cb: Optional[int] = None) -> torch.Tensor:
    """``sglang_exl3_c.p2b_fused_moe`` (``csrc/p2b_moe.cu:418-468``): writes
    ``out = sum_j rw[j] * down_{ids[j]}(swiglu(gate x, up x))`` in out's dtype.
    The reference takes exactly one row with hidden 4096 and intermediate
    1024/2048; here x may be ``[T, H]`` with ids/weights ``[T, topk]`` (or ``[topk]``
    for one row), any hidden/intermediate multiple of 128, any codebook."""
    if not (x.is_cuda and x.dtype == torch.float16):
        raise RuntimeError("fused MoE requires CUDA fp16 input")
    if out.shape != x.shape:
        raise RuntimeError("fused MoE output shape must match input")
    if not (swiglu_limit is not None and float(swiglu_limit) >= 0.0 and float(swiglu_limit) != float("nan")):
        raise RuntimeError("fused MoE SwiGLU limit must be finite and nonnegative (0 disables clipping)")
    x2 = x.reshape(-1, x.shape[-1])
    T = x2.size(0)
    ids = expert_indices.reshape(T, -1)
    rw = routing_weights.reshape(T, -1)
    if ids.numel() == 0 or rw.shape != ids.shape:
        raise RuntimeError("fused MoE requires one routing weight per expert index")
    tables = dict(gate_trellis=gate_trellis_ptrs, gate_suh=gate_suh_ptrs, gate_svh=gate_svh_ptrs,
                  up_trellis=up_trellis_ptrs, up_suh=up_suh_ptrs, up_svh=up_svh_ptrs,
                  down_trellis=down_trellis_ptrs, down_suh=down_suh_ptrs, down_svh=down_svh_ptrs)
    y = moe_forward(x2, ids, rw, tables, K_gate, K_up, K_down, legacy_codebook(mcg, cb), intermediate_size,
                    swiglu_limit)
    out.view(T, -1).copy_(y)
    return out


def exl3_fat_gemm(a: torch.Tensor, packed: torch.Tensor, out: torch.Tensor, svh: torch.Tensor, K: int, mcg: bool,
                  mul1: bool, cb: Optional[int] = None) -> None:
    """``sglang_exl3_c.exl3_fat_gemm`` (``csrc/exl3_fat_gemm.cu:269-283``): ``out`` fp32
    ``[M, N] = H128(a @ W_raw) / sqrt(128) * svh`` with ``a`` already rotated.
    Any K in 2..4 and codebook (the reference requires K=4 MCG)."""
    if out.dtype != torch.float32 or a.dtype != torch.float16 or packed.dtype != torch.int16:
        raise RuntimeError("exl3_fat_gemm: a fp16, packed int16, out fp32")
    if out.size(0) != a.size(0) or out.size(1) != svh.numel():
        raise RuntimeError("out shape must be [M, N]")
    c = codebook_id(mcg, mul1, cb)
    matmul(a, packed, None, svh, int(K), c, out=out, input_rotated=True)


def exl3_fat_gemm_scatter(a: torch.Tensor, packed: torch.Tensor, out: torch.Tensor, svh: torch.Tensor,
                          token_idx: torch.Tensor, route_weight: torch.Tensor, K: int, mcg: bool, mul1: bool,
                          cb: Optional[int] = None) -> None:
    """``sglang_exl3_c.exl3_fat_gemm_scatter`` (``csrc/exl3_fat_gemm.cu:286-305``):
    ``out[token_idx[i]] += route_weight[i] * (H128(a_i @ W_raw) / sqrt(128) * svh)``."""
    if out.dtype != torch.float32:
        raise RuntimeError("out must be float32")
    if token_idx.numel() != a.size(0) or route_weight.numel() != a.size(0):
        raise RuntimeError("routing tensors must have M elements")
    c = codebook_id(mcg, mul1, cb)
    matmul_combine(a, packed, None, svh, int(K), c, out, token_idx.reshape(-1), route_weight.reshape(-1),
                   input_rotated=True)
