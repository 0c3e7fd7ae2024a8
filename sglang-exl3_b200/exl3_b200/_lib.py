"""ctypes binding of ``libexl3b200.so`` (declared in ``include/exl3_b200.h``).

The library is the only compute path: if it is missing or fails to load, every
op raises; there is no CPU or eager-torch fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libexl3b200.so")

OK = 0
STATUS_NAMES = {
    0: "EXL3B200_OK",
    1: "EXL3B200_EBADSHAPE",
    2: "EXL3B200_EBADBITS",
    3: "EXL3B200_EBADCODEBOOK",
    4: "EXL3B200_EUNALIGNED",
    5: "EXL3B200_ELAUNCH",
    6: "EXL3B200_EWORKSPACE",
    7: "EXL3B200_ENULL",
    8: "EXL3B200_EBADARG",
    9: "EXL3B200_ETIMEOUT",
    10: "EXL3B200_EIO",
}

EBADSHAPE, EBADBITS, EBADCODEBOOK, EUNALIGNED, ELAUNCH, EWORKSPACE, ENULL, EBADARG, ETIMEOUT, EIO = range(1, 11)

DTYPE_F16, DTYPE_BF16, DTYPE_F32 = 0, 1, 2
FLAG_INPUT_ROTATED = 1
FLAG_SINGLE_CTA = 2
FLAG_PAIR_CTA = 4
GEMV_MAX_M = 16

_vp = ctypes.c_void_p
_i = ctypes.c_int
_ll = ctypes.c_longlong
_sz = ctypes.c_size_t



class Linear(ctypes.Structure):
    """``exl3b200_linear``: one EXL3 linear for the decode-layer entry points."""

    _fields_ = [("trellis", _vp), ("suh", _vp), ("svh", _vp), ("k", _i), ("n", _i)]


class ShapeDesc(ctypes.Structure):
    """``exl3b200_shape_desc``: one entry of the kernel-shape map."""

    _fields_ = [("name", ctypes.c_char_p), ("max_rows", ctypes.c_int), ("tile_rows", ctypes.c_int),
                ("tile_cols", ctypes.c_int), ("ctas_per_sm", ctypes.c_int)]


SHAPE_GV8, SHAPE_GV8_NARROW, SHAPE_GV16, SHAPE_TC, SHAPE_MOE_SMALL, SHAPE_MOE_TC = range(1, 7)


class MlpArgs(ctypes.Structure):
    """``exl3b200_mlp_args``: one fused SwiGLU MLP block."""

    _fields_ = [("x", _vp), ("x_stride", _ll), ("m", _i), ("hidden", _i), ("inter", _i), ("gate_up", Linear),
                ("K_gate_up", _i), ("cb_gate_up", _i), ("down", Linear), ("K_down", _i), ("cb_down", _i),
                ("swiglu_limit", ctypes.c_float), ("out", _vp), ("out_stride", _ll), ("out_dtype", _i)]


class EpArgs(ctypes.Structure):
    """``exl3b200_ep_args``: one expert-parallel MoE call."""

    _fields_ = [("x", _vp), ("x_stride", _ll), ("tokens", _i), ("max_tokens", _i), ("hidden", _i), ("inter", _i),
                ("topk_ids", _vp), ("topk_weights", _vp), ("topk", _i), ("experts", _i), ("tables", _vp),
                ("K_gate", _i), ("K_up", _i), ("K_down", _i), ("cb", _i), ("swiglu_limit", ctypes.c_float),
                ("out", _vp), ("out_stride", _ll), ("path", _i)]


class DecodeLayer(ctypes.Structure):
    """``exl3b200_decode_layer``: one decoder layer's norms and linears (pointers to
    ``Linear`` descriptors, which the caller keeps alive)."""

    _fields_ = [("attn_norm_w", _vp), ("q", _vp), ("k", _vp), ("v", _vp), ("o", _vp), ("mlp_norm_w", _vp),
                ("gate", _vp), ("up", _vp), ("down", _vp)]


class Peers(ctypes.Structure):
    """``exl3b200_peers``: every rank's peer buffer as mapped in this process."""

    _fields_ = [("buffers", _vp * 8), ("world", _i), ("rank", _i), ("max_rows", _i), ("hidden", _i)]


_f = ctypes.c_float

# name -> (restype, argtypes); one entry per declaration in include/exl3_b200.h
SIGNATURES = {
    "exl3b200_abi_version": (_i, []),
    "exl3b200_num_shapes": (_i, []),
    "exl3b200_select_shape": (_i, [_i, _i, _i, _i, _i, _i, _i]),
    "exl3b200_shape_compat": (_i, [_i, _i, _i, _i, _i]),
    "exl3b200_shape_info": (_i, [_i, _vp]),
    "exl3b200_status_string": (ctypes.c_char_p, [_i]),
    "exl3b200_dequant": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _i, _vp]),
    "exl3b200_gemv_state_size": (_sz, [_i]),
    "exl3b200_gemv_scratch_size": (_sz, [_i, _i]),
    "exl3b200_gemv": (_i, [_vp, _ll, _i, _i, _vp, _i, _i, _i, _vp, _vp, _vp, _ll, _i, _i, _vp, _sz, _vp, _sz, _vp]),
    "exl3b200_hadamard_in": (_i, [_vp, _ll, _i, _i, _vp, _vp, _ll, _vp]),
    "exl3b200_gemv_multi": (_i, [_i, _vp, _ll, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp, _sz, _vp,
                                 _sz, _vp]),
    "exl3b200_gemv_combine": (_i, [_vp, _ll, _i, _i, _vp, _i, _i, _i, _vp, _vp, _vp, _ll, _vp, _vp, _i, _vp, _sz,
                                   _vp, _sz, _vp]),
    "exl3b200_batched_state_size": (_sz, [_i, _i, _i]),
    "exl3b200_batched_scratch_size": (_sz, [_i, _i, _i]),
    "exl3b200_batched_gemv": (_i, [_vp, _i, _ll, _i, _i, _i, _i, _i, _vp, _vp, _vp, _i, _vp, _i, _vp, _i, _vp, _sz,
                                   _vp, _sz, _vp]),
    "exl3b200_gemv_noalloc": (_i, [_vp, _ll, _i, _i, _vp, _i, _i, _i, _vp, _vp, _vp, _ll, _i, _vp]),
    "exl3b200_gemm_state_size": (_sz, []),
    "exl3b200_gemm_scratch_size": (_sz, [_i, _i]),
    "exl3b200_gemm": (_i, [_vp, _ll, _i, _i, _vp, _i, _i, _i, _vp, _vp, _vp, _ll, _i, _i, _vp, _sz, _vp, _sz, _vp]),
    "exl3b200_device_status": (_i, [_vp, _i, _vp]),
    "exl3b200_set_wait_limit": (_i, [ctypes.c_ulonglong]),
    "exl3b200_decode_attention_workspace": (_i, [_i, _i, _i, _i, _i, _vp, _vp]),
    "exl3b200_decode_mlp_workspace": (_i, [_i, _i, _i, _vp, _vp]),
    "exl3b200_decode_attention": (_i, [_i, _i, _i, _i, _i, _i, _vp, _ll, _vp, _vp, _vp, _f, _vp, _vp, _vp, _vp,
                                       _vp, _vp, _i, _vp, _vp, _vp, _ll, _vp, _vp, _sz, _vp, _sz, _vp]),
    "exl3b200_decode_attention_rows": (_i, [_i, _i, _i, _i, _i, _i, _i, _vp, _ll, _vp, _vp, _vp, _f, _vp, _vp, _vp,
                                            _vp, _vp, _vp, _i, _vp, _vp, _vp, _ll, _vp, _vp, _sz, _vp, _sz, _vp]),
    "exl3b200_decode_mlp": (_i, [_i, _i, _i, _i, _i, _vp, _ll, _vp, _vp, _vp, _f, _vp, _vp, _vp, _f, _vp, _ll, _vp,
                                 _vp, _sz, _vp, _sz, _vp]),
    "exl3b200_peer_buffer_size": (_sz, [_i, _i]),
    "exl3b200_peer_buffer_alloc": (_i, [_sz, _vp, _vp]),
    "exl3b200_peer_buffer_open": (_i, [_vp, _vp]),
    "exl3b200_peer_buffer_close": (_i, [_vp]),
    "exl3b200_peer_buffer_free": (_i, [_vp]),
    "exl3b200_peer_reset": (_i, [_vp, _vp]),
    "exl3b200_ep_buffer_size": (_sz, [_i, _i, _i, _i]),
    "exl3b200_ep_workspace": (_i, [_vp, _vp, _vp, _vp]),
    "exl3b200_ep_moe": (_i, [_vp, _vp, _vp, _sz, _vp, _sz, _vp]),
    "exl3b200_residual_add": (_i, [_i, _i, _vp, _ll, _vp, _ll, _vp, _vp]),
    "exl3b200_decode_layer_workspace": (_i, [_i, _i, _i, _i, _i, _i, _vp, _vp]),
    "exl3b200_decode_layer_step": (_i, [_i, _i, _i, _i, _i, _i, _i, _i, _vp, _ll, _vp, _vp, _f, _vp, _vp, _i, _vp,
                                        _vp, _i, _vp, _vp, _f, _vp, _vp, _sz, _vp, _sz, _vp]),
    "exl3b200_mlp_workspace": (_i, [_i, _i, _i, _i, _i, _vp, _vp]),
    "exl3b200_mlp": (_i, [_vp, _vp, _sz, _vp, _sz, _vp]),
    "exl3b200_moe_tc_scratch_size": (_sz, [_i, _i, _i, _i, _i]),
    "exl3b200_moe_tc": (_i, [_vp, _ll, _i, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i,
                             _i, _i, _i, ctypes.c_float, _vp, _ll, _i, _i, _vp, _sz, _vp]),
    "exl3b200_gemm_combine_scratch_size": (_sz, [_i, _i, _i]),
    "exl3b200_gemm_combine": (_i, [_vp, _ll, _i, _i, _vp, _i, _i, _i, _vp, _vp, _vp, _ll, _vp, _vp, _i, _vp, _sz,
                                   _vp]),
    "exl3b200_read_ranges": (_i, [_i, _vp, _vp, _vp, _i, _i, _vp, _sz, _i, _i, _vp]),
    "exl3b200_moe_state_size": (_sz, [_i, _i, _i, _i]),
    "exl3b200_moe_scratch_size": (_sz, [_i, _i, _i, _i]),
    "exl3b200_moe": (_i, [_vp, _ll, _i, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i,
                          _i, _i, _i, ctypes.c_float, _vp, _ll, _i, _i, _vp, _sz, _vp, _sz, _vp]),
}
MULTI_MAX = 8

_lib = None
_lock = threading.Lock()


class Exl3LibraryError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """Load (once) and return the CUDA library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise Exl3LibraryError(
                    f"{LIB_PATH} is not built; run `python sglang-exl3_b200/build.py`. "
                    "The EXL3 B200 ops have no CPU fallback.")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def status_string(status: int) -> str:
    return lib().exl3b200_status_string(int(status)).decode()


def check(status: int, what: str) -> None:
    if status != OK:
        raise RuntimeError(f"{what} failed: {status_string(status)} ({STATUS_NAMES.get(status, status)})")
