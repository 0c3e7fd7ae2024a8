"""Fused decode sub-layers (RMSNorm -> q/k/v -> RoPE + KV append -> attention -> o
-> residual, and RMSNorm -> gate/up -> SwiGLU -> down -> residual) over the C ABI.

The residual stream ``h`` is fp32 ``[batch, hidden]``; ``ss`` holds two per-row
sum-of-squares buffers that the sub-layers alternate between: a sub-layer reads
``ss_in`` for its RMSNorm, zeroes ``ss_out`` and accumulates the new sum of
squares into it with its residual add.  With tensor parallelism either the
sub-layer stores its partial output in ``y`` and, after an NCCL all-reduce,
``residual_add`` completes it, or (``peers``: a ``PeerExchange``) the sub-layer
exchanges the partials itself over NVLink and adds their sum.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import _lib
from . import workspace


def linear_desc(trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor) -> _lib.Linear:
    if trellis.dtype != torch.int16 or trellis.dim() != 3 or not trellis.is_contiguous():
        raise RuntimeError("trellis must be a contiguous int16 [k/16, n/16, 16K] tensor")
    return _lib.Linear(trellis.data_ptr(), suh.data_ptr(), svh.data_ptr(), trellis.size(0) * 16, trellis.size(1) * 16)


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _ws(dev: torch.device, state_n: int, scratch_n: int):
    return workspace.state_buffer(dev, state_n), workspace.scratch_buffer(dev, scratch_n)


def _check_state(h: torch.Tensor, ss_in: torch.Tensor, ss_out: torch.Tensor, norm_w: torch.Tensor):
    if h.dtype != torch.float32 or h.dim() != 2 or h.stride(1) != 1:
        raise RuntimeError("h must be fp32 [batch, hidden] with unit column stride")
    for s in (ss_in, ss_out):
        if s.dtype != torch.float32 or s.numel() < h.size(0) or not s.is_contiguous():
            raise RuntimeError("sum-of-squares buffers must be contiguous fp32 [batch]")
    if norm_w.dtype != torch.bfloat16 or norm_w.numel() != h.size(1) or not norm_w.is_contiguous():
        raise RuntimeError("norm weight must be contiguous bf16 [hidden]")


def _peers_arg(peers):
    return ctypes.byref(peers.struct) if peers is not None else None


def decode_attention(h: torch.Tensor, ss_in: torch.Tensor, ss_out: torch.Tensor, norm_w: torch.Tensor, eps: float,
                     qkv: Sequence, o: Sequence, K: int, cb: int, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     pos: torch.Tensor, inv_freq: torch.Tensor, y: Optional[torch.Tensor] = None,
                     peers=None, rows_per_seq: int = 1) -> None:
    """Attention sub-layer.  ``rows_per_seq = 1``: one new token per row of ``h``, each
    row a sequence; ``rows_per_seq = R`` (speculative verify): rows ``R s + j`` are
    sequence ``s`` at position ``pos + j``, causal among themselves.  ``qkv`` = three
    (trellis, suh, svh) linears, ``o`` one; caches bf16 [sequences, kv_heads, max_ctx, 128]."""
    _check_state(h, ss_in, ss_out, norm_w)
    B, H = h.shape
    R = int(rows_per_seq)
    if R < 1 or B % R:
        raise RuntimeError("rows must be a multiple of rows_per_seq")
    if k_cache.dtype != torch.bfloat16 or k_cache.dim() != 4 or k_cache.size(-1) != 128 or not k_cache.is_contiguous():
        raise RuntimeError("caches must be contiguous bf16 [sequences, kv_heads, max_ctx, 128]")
    if v_cache.shape != k_cache.shape or not v_cache.is_contiguous() or k_cache.size(0) != B // R:
        raise RuntimeError("k and v caches must match and have one row per sequence")
    if pos.dtype != torch.int64 or inv_freq.dtype != torch.float32 or inv_freq.numel() != 64:
        raise RuntimeError("pos must be int64 and inv_freq fp32 [64]")
    kv_heads, max_ctx = k_cache.size(1), k_cache.size(2)
    q_heads = qkv[0][0].size(1) * 16 // 128
    dev = h.device
    L = _lib.lib()
    st_n, sc_n = ctypes.c_size_t(), ctypes.c_size_t()
    _lib.check(L.exl3b200_decode_attention_workspace(B, H, q_heads, kv_heads, max_ctx, ctypes.byref(st_n),
                                                     ctypes.byref(sc_n)), "exl3b200_decode_attention_workspace")
    lq, lk, lv = (linear_desc(*lin) for lin in qkv)
    lo = linear_desc(*o)
    with torch.cuda.device(dev):
        state, scratch = _ws(dev, st_n.value, sc_n.value)
        rc = L.exl3b200_decode_attention_rows(
            B, R, H, q_heads, kv_heads, int(K), int(cb), h.data_ptr(), h.stride(0), ss_in.data_ptr(), ss_out.data_ptr(),
            norm_w.data_ptr(), float(eps), ctypes.byref(lq), ctypes.byref(lk), ctypes.byref(lv), ctypes.byref(lo),
            k_cache.data_ptr(), v_cache.data_ptr(), max_ctx, pos.data_ptr(), inv_freq.data_ptr(),
            y.data_ptr() if y is not None else None, y.stride(0) if y is not None else 0, _peers_arg(peers),
            state.data_ptr(), state.numel(), scratch.data_ptr(), scratch.numel(), _stream(dev))
    _lib.check(rc, "exl3b200_decode_attention")


def decode_mlp(h: torch.Tensor, ss_in: torch.Tensor, ss_out: torch.Tensor, norm_w: torch.Tensor, eps: float,
               gate: Sequence, up: Sequence, down: Sequence, K: int, cb: int, swiglu_limit: float = 0.0,
               y: Optional[torch.Tensor] = None, peers=None) -> None:
    """SwiGLU MLP sub-layer."""
    _check_state(h, ss_in, ss_out, norm_w)
    B, H = h.shape
    inter = gate[0].size(1) * 16
    dev = h.device
    L = _lib.lib()
    st_n, sc_n = ctypes.c_size_t(), ctypes.c_size_t()
    _lib.check(L.exl3b200_decode_mlp_workspace(B, H, inter, ctypes.byref(st_n), ctypes.byref(sc_n)),
               "exl3b200_decode_mlp_workspace")
    lg, lu, ld = linear_desc(*gate), linear_desc(*up), linear_desc(*down)
    with torch.cuda.device(dev):
        state, scratch = _ws(dev, st_n.value, sc_n.value)
        rc = L.exl3b200_decode_mlp(
            B, H, inter, int(K), int(cb), h.data_ptr(), h.stride(0), ss_in.data_ptr(), ss_out.data_ptr(),
            norm_w.data_ptr(), float(eps), ctypes.byref(lg), ctypes.byref(lu), ctypes.byref(ld), float(swiglu_limit),
            y.data_ptr() if y is not None else None, y.stride(0) if y is not None else 0, _peers_arg(peers),
            state.data_ptr(), state.numel(), scratch.data_ptr(), scratch.numel(), _stream(dev))
    _lib.check(rc, "exl3b200_decode_mlp")


class LayerDesc:
    """One decoder layer for ``decode_layer``: the ``exl3b200_decode_layer`` struct and
    the ``Linear`` descriptors it points to (kept alive with the tensors' pointers)."""

    def __init__(self, attn_norm_w: torch.Tensor, qkv: Sequence, o: Sequence, mlp_norm_w: torch.Tensor,
                 gate: Sequence, up: Sequence, down: Sequence):
        for w in (attn_norm_w, mlp_norm_w):
            if w.dtype != torch.bfloat16 or not w.is_contiguous():
                raise RuntimeError("norm weights must be contiguous bf16 [hidden]")
        self.norms = (attn_norm_w, mlp_norm_w)
        self.lins = [linear_desc(*lin) for lin in (*qkv, o, gate, up, down)]
        q, k, v, lo, g, u, d = (ctypes.addressof(lin) for lin in self.lins)
        self.struct = _lib.DecodeLayer(attn_norm_w.data_ptr(), q, k, v, lo, mlp_norm_w.data_ptr(), g, u, d)
        self.q_heads = qkv[0][0].size(1) * 16 // 128
        self.inter = gate[0].size(1) * 16


def decode_layer(h: torch.Tensor, ss_a: torch.Tensor, ss_b: torch.Tensor, eps: float, layer: LayerDesc,
                 next_layer: Optional[LayerDesc], input_ready: bool, K: int, cb: int, k_cache: torch.Tensor,
                 v_cache: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor, swiglu_limit: float = 0.0,
                 peers=None, rows_per_seq: int = 1) -> None:
    """A whole decoder layer (attention, then MLP) with the RMSNorm input stages folded
    into the residual epilogues.  ``ss_a``: the rows' sum of squares of ``h`` on entry
    and of the new ``h`` on return; ``ss_b`` a second [rows] buffer.  With
    ``next_layer`` the MLP's residual epilogue writes that layer's q/k/v inputs and its
    call passes ``input_ready=True`` (same rows and shapes: the workspace is shared)."""
    _check_state(h, ss_a, ss_b, layer.norms[0])
    B, H = h.shape
    R = int(rows_per_seq)
    if R < 1 or B % R:
        raise RuntimeError("rows must be a multiple of rows_per_seq")
    if k_cache.dtype != torch.bfloat16 or k_cache.dim() != 4 or k_cache.size(-1) != 128 or not k_cache.is_contiguous():
        raise RuntimeError("caches must be contiguous bf16 [sequences, kv_heads, max_ctx, 128]")
    if v_cache.shape != k_cache.shape or not v_cache.is_contiguous() or k_cache.size(0) != B // R:
        raise RuntimeError("k and v caches must match and have one row per sequence")
    if pos.dtype != torch.int64 or inv_freq.dtype != torch.float32 or inv_freq.numel() != 64:
        raise RuntimeError("pos must be int64 and inv_freq fp32 [64]")
    kv_heads, max_ctx = k_cache.size(1), k_cache.size(2)
    dev = h.device
    L = _lib.lib()
    st_n, sc_n = ctypes.c_size_t(), ctypes.c_size_t()
    _lib.check(L.exl3b200_decode_layer_workspace(B, H, layer.q_heads, kv_heads, layer.inter, max_ctx,
                                                 ctypes.byref(st_n), ctypes.byref(sc_n)),
               "exl3b200_decode_layer_workspace")
    with torch.cuda.device(dev):
        state, scratch = _ws(dev, st_n.value, sc_n.value)
        rc = L.exl3b200_decode_layer_step(
            B, R, H, layer.q_heads, kv_heads, layer.inter, int(K), int(cb), h.data_ptr(), h.stride(0),
            ss_a.data_ptr(), ss_b.data_ptr(), float(eps), ctypes.byref(layer.struct),
            ctypes.byref(next_layer.struct) if next_layer is not None else None, int(bool(input_ready)),
            k_cache.data_ptr(), v_cache.data_ptr(), max_ctx, pos.data_ptr(), inv_freq.data_ptr(),
            float(swiglu_limit), _peers_arg(peers), state.data_ptr(), state.numel(), scratch.data_ptr(),
            scratch.numel(), _stream(dev))
    _lib.check(rc, "exl3b200_decode_layer_step")


def residual_add(h: torch.Tensor, y: torch.Tensor, ss_out: torch.Tensor) -> None:
    """``h += y`` and the new per-row sum of squares into (zeroed) ``ss_out``."""
    if y.dtype != torch.float32 or y.shape != h.shape:
        raise RuntimeError("y must be fp32 shaped like h")
    dev = h.device
    with torch.cuda.device(dev):
        rc = _lib.lib().exl3b200_residual_add(h.size(0), h.size(1), h.data_ptr(), h.stride(0), y.data_ptr(),
                                              y.stride(0), ss_out.data_ptr(), _stream(dev))
    _lib.check(rc, "exl3b200_residual_add")


class PeerExchange:
    """Peer buffers of one tensor-parallel group for the fused decode sub-layers:
    each rank allocates its buffer, the 64-byte CUDA IPC handles are exchanged with
    ``all_gather_object`` and every rank maps the others' buffers.  ``close`` (all
    ranks, before the process group goes away) unmaps and frees them."""

    def __init__(self, max_rows: int, hidden: int, group=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise RuntimeError("peer exchange supports at most 8 ranks")
        L = _lib.lib()
        size = L.exl3b200_peer_buffer_size(max_rows, hidden)
        if size == 0:
            raise RuntimeError("bad peer buffer shape")
        handle = (ctypes.c_char * 64)()
        own = ctypes.c_void_p()
        _lib.check(L.exl3b200_peer_buffer_alloc(size, ctypes.byref(own), handle), "exl3b200_peer_buffer_alloc")
        self._own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        ptrs = []
        for q in range(self.world):
            if q == self.rank:
                ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            buf = (ctypes.c_char * 64).from_buffer_copy(handles[q])
            _lib.check(L.exl3b200_peer_buffer_open(buf, ctypes.byref(p)), "exl3b200_peer_buffer_open")
            self._opened.append(p.value)
            ptrs.append(p.value)
        self.struct = _lib.Peers((ctypes.c_void_p * 8)(*(ptrs + [None] * (8 - len(ptrs)))), self.world, self.rank,
                                 max_rows, hidden)
        dist.barrier(group)

    def reset(self) -> None:
        """Re-arm the exchange after a device wait gave up (every rank, together):
        drain this rank's work, wait for every rank, re-arm the own buffer, wait again."""
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(self.group)
        _lib.check(_lib.lib().exl3b200_peer_reset(self._own, torch.cuda.current_stream().cuda_stream),
                   "exl3b200_peer_reset")
        torch.cuda.synchronize()
        dist.barrier(self.group)

    def close(self) -> None:
        import torch.distributed as dist

        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(self.group)
        L = _lib.lib()
        for p in self._opened:
            L.exl3b200_peer_buffer_close(p)
        self._opened = []
        dist.barrier(self.group)
        L.exl3b200_peer_buffer_free(self._own)
        self._own = None
