"""Tensor-level EXL3 ops over the C ABI, with the reference's op surface.

Functions here take torch tensors, validate them with the reference's error
messages (``TORCH_CHECK`` -> ``RuntimeError``), fetch persistent workspaces and
call ``libexl3b200.so`` on the current CUDA stream.  ``register_custom_ops``
registers them as ``torch.ops.sglang_exl3.*`` with the schemas and fake kernels
of the reference (``src/sglang_exl3/ops.py:29-230``), so callers written for the
reference run unchanged.

Codebook selection: the reference ops take ``mcg: bool`` and reach only MCG
(cb 1) or mul1 (cb 2) (``csrc/bindings.cpp:48``, ``csrc/exl3_gemv.cu:32``).  Every
op here also accepts ``cb`` (0 = 3INST, 1 = MCG, 2 = mul1); ``cb=None`` keeps
the legacy mapping.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from . import workspace

_OUT_DTYPES = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}


def codebook_id(mcg: bool = False, mul1: bool = False, cb: Optional[int] = None) -> int:
    """Codebook id from the reference's flags (``dense.py:151-157``): explicit cb wins."""
    if cb is not None and int(cb) >= 0:
        if int(cb) not in (0, 1, 2):
            raise RuntimeError(f"unsupported EXL3 codebook {cb}")
        return int(cb)
    if mcg and mul1:
        raise ValueError("EXL3 linear has both mcg and mul1 markers set")
    return 1 if mcg else (2 if mul1 else 0)


def legacy_codebook(mcg: bool, cb: Optional[int] = None) -> int:
    """The ``sglang_exl3_c`` binding's mapping: mcg -> 1, else mul1 (2)."""
    if cb is not None and int(cb) >= 0:
        return codebook_id(cb=cb)
    return 1 if mcg else 2


def bits_of(trellis: torch.Tensor) -> int:
    """K from the trellis' last dimension (16*K int16 per tile, ``dense.py:149-150``)."""
    k = trellis.shape[-1] // 16
    if trellis.shape[-1] != 16 * k:
        raise RuntimeError("trellis last dimension must be 16*K")
    return int(k)


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("EXL3 B200 ops require CUDA tensors (there is no CPU path)")
        if t.device != dev:
            raise RuntimeError("EXL3 tensors must share a CUDA device")
    return dev


# ---------------------------------------------------------------------------
# dequant
# ---------------------------------------------------------------------------

def dequant(trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: Optional[int] = None,
            cb: int = 0, rounding: str = "rn", out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp16 weight ``W [k, n]`` with ``y = x @ W``.  ``rounding="rn"``: codebook
    rounded to nearest (reference device decode); ``"trunc"``: bit-identical to
    the reference's CPU ``dequant_trellis`` (``csrc/bindings.cpp:15-132``)."""
    if K is None:
        K = bits_of(trellis)
    if K not in range(1, 9):
        raise RuntimeError("K must be one of 1..8")
    if trellis.dim() != 3 or trellis.dtype != torch.int16:
        raise RuntimeError("trellis must be int16 [rows/16, cols/16, 16*K]")
    if trellis.size(2) != 16 * K:
        raise RuntimeError("trellis last dimension must be 16*K")
    if trellis.size(0) <= 0 or trellis.size(1) <= 0:
        raise RuntimeError("trellis dimensions must be positive")
    if suh.dtype != torch.float16 or svh.dtype != torch.float16:
        raise RuntimeError("suh and svh must be float16")
    rows, cols = trellis.size(0) * 16, trellis.size(1) * 16
    if suh.numel() < rows or svh.numel() < cols:
        raise RuntimeError("suh/svh are too short")
    if rows % 128 or cols % 128:
        raise RuntimeError("trellis dimensions must reconstruct whole 128-element Hadamard blocks")
    dev = _require_cuda(trellis, suh, svh)
    trellis, suh, svh = trellis.contiguous(), suh.contiguous(), svh.contiguous()
    if out is None:
        out = torch.empty((rows, cols), dtype=torch.float16, device=dev)
    mode = {"rn": 0, "trunc": 1}[rounding]
    with torch.cuda.device(dev):
        st = _lib.lib().exl3b200_dequant(trellis.data_ptr(), trellis.size(0), trellis.size(1), K, cb,
                                         suh.data_ptr(), svh.data_ptr(), out.data_ptr(), mode, _stream_ptr(dev))
    _lib.check(st, "exl3b200_dequant")
    return out


# ---------------------------------------------------------------------------
# input transform
# ---------------------------------------------------------------------------

def hadamard_in(x: torch.Tensor, suh: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp16 ``H128(x * suh) / sqrt(128)`` over 128-blocks of the last dimension."""
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.float16:
        raise RuntimeError("hadamard_in requires fp16 input")
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m, k = x2.shape
    dev = _require_cuda(x2) if suh is None else _require_cuda(x2, suh)
    if out is None:
        out = torch.empty((m, k), dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        st = _lib.lib().exl3b200_hadamard_in(x2.data_ptr(), x2.stride(0), m, k,
                                             suh.contiguous().data_ptr() if suh is not None else None,
                                             out.data_ptr(), out.stride(0), _stream_ptr(dev))
    _lib.check(st, "exl3b200_hadamard_in")
    return out.view(*x.shape[:-1], k)


# ---------------------------------------------------------------------------
# matmul
# ---------------------------------------------------------------------------

def _gemv_into(x2: torch.Tensor, trellis: torch.Tensor, suh: Optional[torch.Tensor], svh: torch.Tensor,
               K: int, cb: int, out: torch.Tensor, flags: int) -> None:
    m, k = x2.shape
    n = trellis.size(1) * 16
    dev = x2.device
    L = _lib.lib()
    state_n = L.exl3b200_gemv_state_size(n)
    scratch_n = L.exl3b200_gemv_scratch_size(m, k)
    with torch.cuda.device(dev):
        state = workspace.state_buffer(dev, state_n)
        scratch = workspace.scratch_buffer(dev, scratch_n)
        st = L.exl3b200_gemv(x2.data_ptr(), x2.stride(0), m, k, trellis.data_ptr(), n, K, cb,
                             suh.data_ptr() if suh is not None else None, svh.data_ptr(),
                             out.data_ptr(), out.stride(0), _OUT_DTYPES[out.dtype], flags,
                             state.data_ptr(), state.numel(), scratch.data_ptr(), scratch.numel(),
                             _stream_ptr(dev))
    _lib.check(st, "exl3b200_gemv")


def _check_linear(x2: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int):
    if x2.dtype != torch.float16:
        raise RuntimeError("CUDA GEMV requires fp16 input")
    if trellis.dim() != 3 or trellis.dtype != torch.int16:
        raise RuntimeError("trellis must be int16 [rows/16, cols/16, 16*K]")
    if trellis.size(2) != 16 * K:
        raise RuntimeError("trellis last dimension must be 16*K")
    if x2.size(-1) != trellis.size(0) * 16:
        raise RuntimeError("x feature dimension does not match trellis")
    if svh.numel() != trellis.size(1) * 16:
        raise RuntimeError("svh N dimension does not match trellis")
    if suh is not None and suh.numel() != trellis.size(0) * 16:
        raise RuntimeError("suh K dimension does not match trellis")


_SHAPES = {}


def select_shape(m: int, k: int, n: int, K: int, cb: int, experts: int = 0, topk: int = 0) -> int:
    """The library's kernel-shape map (``exl3b200_select_shape``): ``_lib.SHAPE_*``."""
    key = (m, k, n, K, cb, experts, topk)
    shape = _SHAPES.get(key)
    if shape is None:
        shape = int(_lib.lib().exl3b200_select_shape(m, k, n, K, cb, experts, topk))
        if shape <= 0:
            raise RuntimeError(f"no kernel shape for m={m} k={k} n={n} K={K} cb={cb}")
        if len(_SHAPES) < 65536:
            _SHAPES[key] = shape
    return shape


def _tc_rows(m: int, k: int, n: int, K: int, cb: int) -> bool:
    return select_shape(m, k, n, K, cb) == _lib.SHAPE_TC


def _gemm_into(x2: torch.Tensor, trellis: torch.Tensor, suh: Optional[torch.Tensor], svh: torch.Tensor,
               K: int, cb: int, out: torch.Tensor, flags: int) -> None:
    m, k = x2.shape
    n = trellis.size(1) * 16
    dev = x2.device
    L = _lib.lib()
    if svh.data_ptr() % 16:
        svh = svh.clone()
    with torch.cuda.device(dev):
        state = workspace.state_buffer(dev, L.exl3b200_gemm_state_size())
        scratch = workspace.scratch_buffer(dev, L.exl3b200_gemm_scratch_size(m, k))
        st = L.exl3b200_gemm(x2.data_ptr(), x2.stride(0), m, k, trellis.data_ptr(), n, K, cb,
                             suh.data_ptr() if suh is not None else None, svh.data_ptr(),
                             out.data_ptr(), out.stride(0), _OUT_DTYPES[out.dtype], flags,
                             state.data_ptr(), state.numel(), scratch.data_ptr(), scratch.numel(),
                             _stream_ptr(dev))
    _lib.check(st, "exl3b200_gemm")


def device_status(device: Optional[torch.device] = None, reset: bool = True) -> int:
    """The library's sticky device-side status (0, or e.g. ``ETIMEOUT`` when a
    tensor-core kernel's bounded wait gave up); synchronises the current stream."""
    import ctypes

    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    host = torch.zeros(1, dtype=torch.int32).pin_memory()
    with torch.cuda.device(dev):
        st = _lib.lib().exl3b200_device_status(ctypes.c_void_p(host.data_ptr()), int(reset), _stream_ptr(dev))
        _lib.check(st, "exl3b200_device_status")
        torch.cuda.current_stream(dev).synchronize()
    return int(host.item())


def set_wait_limit(seconds: Optional[float]) -> None:
    """Limit of the library's bounded device-side waits for kernels launched from now
    on (tensor-core pipeline barriers, decode peer exchange); ``None`` restores the
    defaults.  Process-wide."""
    ns = 0 if seconds is None else max(1, int(seconds * 1e9))
    _lib.check(_lib.lib().exl3b200_set_wait_limit(ns), "exl3b200_set_wait_limit")


def matmul(x: torch.Tensor, trellis: torch.Tensor, suh: Optional[torch.Tensor], svh: torch.Tensor,
           K: Optional[int] = None, cb: int = 0, out_dtype: torch.dtype = torch.float16,
           out: Optional[torch.Tensor] = None, input_rotated: bool = False,
           variant: Optional[int] = None, path: Optional[str] = None) -> torch.Tensor:
    """``y = x @ W`` for any number of rows: ``x [..., k]`` fp16 -> ``[..., n]``.

    Where the kernel-shape map says so (17 rows and more; or ``path="tc"``), one
    tensor-core GEMM over all rows (512-row CTA-pair tiles from 2048 rows when k >= 16384;
    ``path="tc1"`` keeps single-CTA tiles, ``path="tc2"`` takes pair tiles at any row
    count); below, the small-M kernel in chunks of at most 16 rows (``path="gemv"``).
    Replaces ``exl3_gemm_cuda`` (``csrc/exl3_gemm.cu:9-31``).  ``out`` may be a
    row-strided 2D view (e.g. a column slice of a fused qkv output)."""
    if K is None:
        K = bits_of(trellis)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1 or (x2.stride(0) % 2):
        x2 = x2.contiguous()
    _check_linear(x2, trellis, suh, svh, K)
    dev = _require_cuda(x2, trellis, svh)
    m = x2.size(0)
    n = trellis.size(1) * 16
    if out is None:
        out2 = torch.empty((m, n), dtype=out_dtype, device=dev)
    else:
        out2 = out.reshape(m, n) if out.dim() != 2 else out
        if out2.stride(-1) != 1:
            raise RuntimeError("out must have unit stride in its last dimension")
        if out2.dtype not in _OUT_DTYPES:
            raise RuntimeError("out must be fp16, bf16 or fp32")
    flags = _lib.FLAG_INPUT_ROTATED if input_rotated else 0
    if variant is not None:
        flags |= (int(variant) & 3) << 8
    if path not in (None, "tc", "tc1", "tc2", "gemv"):
        raise RuntimeError("path must be None, 'tc', 'tc1', 'tc2' or 'gemv'")
    if path == "tc1":  # the tensor-core kernel without CTA-pair tiles
        flags |= _lib.FLAG_SINGLE_CTA
    elif path == "tc2":  # CTA-pair tiles at any row count
        flags |= _lib.FLAG_PAIR_CTA
    use_tc = path in ("tc", "tc1", "tc2") or (path is None and trellis.data_ptr() % 16 == 0 and _tc_rows(m, x2.size(1), n, K, cb))
    if use_tc:
        _gemm_into(x2, trellis.contiguous(), suh, svh, K, cb, out2, flags)
    else:
        for r0 in range(0, m, _lib.GEMV_MAX_M):
            r1 = min(m, r0 + _lib.GEMV_MAX_M)
            _gemv_into(x2[r0:r1], trellis, suh, svh, K, cb, out2[r0:r1], flags)
    if out is not None:
        return out
    return out2.view(*lead, n)


# ---------------------------------------------------------------------------
# reference-named entry points (semantics of sglang_exl3_c, csrc/bindings.cpp)
# ---------------------------------------------------------------------------

def dequant_trellis(trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, bits: int, mcg: bool,
                    cb: Optional[int] = None, rounding: str = "trunc") -> torch.Tensor:
    """``sglang_exl3_c.dequant_trellis`` (``csrc/bindings.cpp:117-132``).  The
    reference op's output is the truncating CPU decode; ``rounding="trunc"`` (the
    default here) reproduces it bit for bit, ``"rn"`` gives the device decode."""
    if bits not in (2, 3, 4, 8) and cb is None:
        raise RuntimeError("K must be one of 2, 3, 4, or 8")
    return dequant(trellis, suh, svh, int(bits), legacy_codebook(mcg, cb), rounding)


def exl3_gemv(x: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int,
              mcg: bool, mmode: int = 1, cb: Optional[int] = None) -> torch.Tensor:
    """``sglang_exl3_c.exl3_gemv`` (``csrc/bindings.cpp:134-147``): fp16 ``[m, n]``,
    1 <= m <= 16 (the reference allows 8)."""
    if x.dim() < 2:
        raise RuntimeError("x must have shape [..., in_features]")
    m = x.numel() // x.size(-1)
    if not (1 <= m <= _lib.GEMV_MAX_M):
        raise RuntimeError(f"native GEMV supports 1 <= m <= {_lib.GEMV_MAX_M}")
    if x.size(-1) != trellis.size(0) * 16:
        raise RuntimeError("x feature dimension does not match trellis")
    if mmode not in (0, 1):
        raise RuntimeError("mmode must be 0 or 1")
    return matmul(x.reshape(m, x.size(-1)), trellis, suh, svh, int(K), legacy_codebook(mcg, cb))


def exl3_gemm(x: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int,
              mcg: bool, cb: Optional[int] = None) -> torch.Tensor:
    """``sglang_exl3_c.exl3_gemm`` (``csrc/exl3_gemm.cu:9-31``): fp16 ``[m, n]``."""
    x2 = x.contiguous().view(x.numel() // x.size(-1), x.size(-1))
    return matmul(x2, trellis, suh, svh, int(K), legacy_codebook(mcg, cb))


def mlp(x: torch.Tensor, gate_up, down, K_gate_up: int, cb_gate_up: int, K_down: int, cb_down: int,
        swiglu_limit: float = 0.0, out_dtype: torch.dtype = torch.float16,
        out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Dense SwiGLU MLP block ``down(silu(gate(x)) * up(x))`` in one library call, the
    activation fused into the gate|up matmul's epilogue (``exl3b200_mlp``).
    ``gate_up`` = (trellis, suh, svh) of the fused gate|up linear (n = 2 * inter, gate
    columns first: the reference's packed13 layout, ``exl3.py:1199-1218``), ``down`` =
    (trellis, suh, svh).  Small-M kernels up to 16 rows, tensor cores from 17."""
    import ctypes

    from .decode import linear_desc

    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.float16:
        raise RuntimeError("mlp requires fp16 input")
    if x2.stride(-1) != 1 or (x2.stride(0) % 2):
        x2 = x2.contiguous()
    gtr, gsu, gsv = gate_up
    dtr, dsu, dsv = down
    _check_linear(x2, gtr, gsu, gsv, K_gate_up)
    inter = gtr.size(1) * 8
    if dtr.size(0) * 16 != inter or dtr.size(1) * 16 != x2.size(1):
        raise RuntimeError("down projection does not match the gate|up linear")
    _check_linear(torch.empty((0, inter), dtype=torch.float16, device=x2.device), dtr, dsu, dsv, K_down)
    dev = _require_cuda(x2, gtr, gsv, dtr, dsv)
    m, hidden = x2.shape
    if out is None:
        out2 = torch.empty((m, hidden), dtype=out_dtype, device=dev)
    else:
        out2 = out.reshape(m, hidden) if out.dim() != 2 else out
        if out2.stride(-1) != 1 or out2.dtype not in _OUT_DTYPES:
            raise RuntimeError("out must be fp16 / bf16 / fp32 with unit column stride")
    L = _lib.lib()
    aligned = [t if t.data_ptr() % 16 == 0 else t.clone() for t in (gsv, dsu, dsv)]
    gsv, dsu, dsv = aligned
    st_n, sc_n = ctypes.c_size_t(), ctypes.c_size_t()
    _lib.check(L.exl3b200_mlp_workspace(m, hidden, inter, K_gate_up, cb_gate_up, ctypes.byref(st_n),
                                        ctypes.byref(sc_n)), "exl3b200_mlp_workspace")
    args = _lib.MlpArgs(x2.data_ptr(), x2.stride(0), m, hidden, inter, linear_desc(gtr.contiguous(), gsu, gsv),
                        K_gate_up, cb_gate_up, linear_desc(dtr.contiguous(), dsu, dsv), K_down, cb_down,
                        float(swiglu_limit), out2.data_ptr(), out2.stride(0), _OUT_DTYPES[out2.dtype])
    with torch.cuda.device(dev):
        state = workspace.state_buffer(dev, st_n.value)
        scratch = workspace.scratch_buffer(dev, sc_n.value)
        st = L.exl3b200_mlp(ctypes.byref(args), state.data_ptr(), state.numel(), scratch.data_ptr(), scratch.numel(),
                            _stream_ptr(dev))
    _lib.check(st, "exl3b200_mlp")
    if out is not None:
        return out
    return out2.view(*lead, hidden)


def _ptr_array(vals) -> "ctypes.Array":
    import ctypes

    arr = (ctypes.c_void_p * len(vals))()
    for i, v in enumerate(vals):
        arr[i] = v
    return arr


def matmul_multi(x: torch.Tensor, linears, K: int, cb: int, outs=None,
                 out_dtype: torch.dtype = torch.float16, variant: Optional[int] = None):
    """Several linears ``(trellis, suh, svh)`` over one input in one launch sequence
    (fused q/k/v or gate/up; replaces the upstream ``exl3_mgemm`` pair GEMM the
    reference calls, ``src/sglang_exl3/dense.py:91-119``).  Returns the list of
    outputs (or writes into ``outs``: 2D row-strided views, e.g. column slices of one
    fused output)."""
    import ctypes

    count = len(linears)
    if not 1 <= count <= _lib.MULTI_MAX:
        raise RuntimeError(f"matmul_multi takes 1..{_lib.MULTI_MAX} linears")
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1 or (x2.stride(0) % 2):
        x2 = x2.contiguous()
    for tr, su, sv in linears:
        _check_linear(x2, tr, su, sv, K)
    dev = _require_cuda(x2, *[t for lin in linears for t in lin])
    m, k = x2.shape
    ns = [tr.size(1) * 16 for tr, _, _ in linears]
    if outs is None:
        outs = [torch.empty((m, n), dtype=out_dtype, device=dev) for n in ns]
    for o, n in zip(outs, ns):
        if o.dim() != 2 or o.shape != (m, n) or o.stride(-1) != 1:
            raise RuntimeError("matmul_multi outputs must be [m, n] with unit column stride")
        if o.dtype != outs[0].dtype:
            raise RuntimeError("matmul_multi outputs must share a dtype")
    L = _lib.lib()
    flags = 0 if variant is None else (int(variant) & 3) << 8
    if _tc_rows(m, k, max(ns), K, cb) and all(lin[0].data_ptr() % 16 == 0 for lin in linears):
        # one tensor-core GEMM per linear: codes streamed once per 256 rows
        for (tr, su, sv), o in zip(linears, outs):
            _gemm_into(x2, tr.contiguous(), su, sv, K, cb, o, 0)
        return outs
    for r0 in range(0, m, _lib.GEMV_MAX_M):
        r1 = min(m, r0 + _lib.GEMV_MAX_M)
        mc = r1 - r0
        state_n = sum(L.exl3b200_gemv_state_size(n) for n in ns)
        scratch_n = count * L.exl3b200_gemv_scratch_size(mc, k)
        with torch.cuda.device(dev):
            state = workspace.state_buffer(dev, state_n)
            scratch = workspace.scratch_buffer(dev, scratch_n)
            oc = [o[r0:r1] for o in outs]
            st = L.exl3b200_gemv_multi(
                count, x2[r0:r1].data_ptr(), x2.stride(0), mc, k, K, cb,
                _ptr_array([lin[0].data_ptr() for lin in linears]), (ctypes.c_int * count)(*ns),
                _ptr_array([lin[1].data_ptr() for lin in linears]), _ptr_array([lin[2].data_ptr() for lin in linears]),
                _ptr_array([o.data_ptr() for o in oc]), (ctypes.c_longlong * count)(*[o.stride(0) for o in oc]),
                _OUT_DTYPES[outs[0].dtype], flags, state.data_ptr(), state.numel(), scratch.data_ptr(),
                scratch.numel(), _stream_ptr(dev))
        _lib.check(st, "exl3b200_gemv_multi")
    return outs


def matmul_combine(x: torch.Tensor, trellis: torch.Tensor, suh: Optional[torch.Tensor], svh: torch.Tensor,
                   K: int, cb: int, out: torch.Tensor, rows: torch.Tensor, scale: Optional[torch.Tensor] = None,
                   input_rotated: bool = False) -> torch.Tensor:
    """``out[rows[r]] += scale[r] * (x[r] @ W)`` (fp32 out; rows int32, scale fp32).

    Up to 16 rows: the small-M kernel (rows must be distinct).  More: one
    tensor-core launch that decodes the codes once per 256 rows and adds with
    atomics (repeated rows add up; out 16-byte aligned, row stride a multiple of 4)."""
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1 or (x2.stride(0) % 2):
        x2 = x2.contiguous()
    _check_linear(x2, trellis, suh, svh, K)
    dev = _require_cuda(x2, trellis, svh, out, rows)
    if out.dtype != torch.float32 or out.dim() != 2 or out.stride(-1) != 1:
        raise RuntimeError("out must be a float32 [rows, N] tensor")
    rows = rows.to(torch.int32).contiguous()
    scale = None if scale is None else scale.to(torch.float32).contiguous()
    m, k = x2.shape
    n = trellis.size(1) * 16
    L = _lib.lib()
    flags = _lib.FLAG_INPUT_ROTATED if input_rotated else 0
    if m > _lib.GEMV_MAX_M and out.data_ptr() % 16 == 0 and out.stride(0) % 4 == 0:
        with torch.cuda.device(dev):
            scratch = workspace.scratch_buffer(dev, L.exl3b200_gemm_combine_scratch_size(m, k, n))
            st = L.exl3b200_gemm_combine(
                x2.data_ptr(), x2.stride(0), m, k, trellis.data_ptr(), n, K, cb,
                suh.data_ptr() if suh is not None else None, svh.data_ptr(), out.data_ptr(), out.stride(0),
                rows.data_ptr(), scale.data_ptr() if scale is not None else None, flags, scratch.data_ptr(),
                scratch.numel(), _stream_ptr(dev))
        _lib.check(st, "exl3b200_gemm_combine")
        return out
    for r0 in range(0, m, _lib.GEMV_MAX_M):
        r1 = min(m, r0 + _lib.GEMV_MAX_M)
        with torch.cuda.device(dev):
            state = workspace.state_buffer(dev, L.exl3b200_gemv_state_size(n))
            scratch = workspace.scratch_buffer(dev, L.exl3b200_gemv_scratch_size(r1 - r0, k))
            st = L.exl3b200_gemv_combine(
                x2[r0:r1].data_ptr(), x2.stride(0), r1 - r0, k, trellis.data_ptr(), n, K, cb,
                suh.data_ptr() if suh is not None else None, svh.data_ptr(), out.data_ptr(), out.stride(0),
                rows[r0:r1].data_ptr(), scale[r0:r1].data_ptr() if scale is not None else None, flags,
                state.data_ptr(), state.numel(), scratch.data_ptr(), scratch.numel(), _stream_ptr(dev))
        _lib.check(st, "exl3b200_gemv_combine")
    return out
