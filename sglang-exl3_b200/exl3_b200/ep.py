"""Expert-parallel routed MoE: all-to-all dispatch and combine around the device
MoE pipeline.

The experts of a layer are split evenly over the ranks of a process group
(rank r owns global experts ``[r*E/W, (r+1)*E/W)``: the reference's EP layout,
whose id mapping is ``map_topk_to_local`` / ``_get_expert_map``,
``src/sglang_exl3/exl3.py:485-509``).  Two exchange modes:

* static (default): every token row goes to every rank with its top-k ids
  rewritten to that rank's local ids (-1 where another rank owns the expert) and
  its routing weights, so every ``all_to_all_single`` has equal splits of T rows.
  Nothing is read on the host: a call is stream-ordered end to end (NCCL in the
  stream) and can be captured in a CUDA graph.  Each rank runs its local experts
  on the W*T received rows (``local_fn``: the fused device MoE pipeline, which
  skips id -1, so rows with no local expert cost routing only), the fp32 results
  come back with the reverse exchange and the W contributions are summed per
  token.  The price is bandwidth: W*T rows of H fp16 out and fp32 back per rank.
* variable (``static=False``): a token goes only to the ranks that own one of its
  experts; the per-destination counts are exchanged first and read on the host to
  size the row exchanges (one host synchronisation per call).

Collectives are ``torch.distributed`` calls, so the module runs over NCCL on
GPUs and over gloo on CPU (the tests use gloo with a host-side expert function).
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

LocalFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


class ExpertParallelMoE:
    """Dispatch/combine for ``n_experts`` experts over ``world`` ranks."""

    def __init__(self, n_experts: int, world: int, rank: int, group=None, static: bool = True):
        if world < 1 or n_experts % world:
            raise ValueError(f"{n_experts} experts do not split evenly over {world} ranks")
        self.n_experts = n_experts
        self.world = world
        self.rank = rank
        self.group = group
        self.static = static
        self.per_rank = n_experts // world
        self.last_counts: Optional[tuple] = None  # variable mode: (send, recv) row counts of the last call

    def local_ids(self, topk_ids: torch.Tensor) -> torch.Tensor:
        """``[W, T, k]`` int32: each rank's view of the ids (local id, or -1 when the
        expert is invalid or lives on another rank)."""
        ids = topk_ids.to(torch.long)
        valid = (ids >= 0) & (ids < self.n_experts)
        owner = torch.where(valid, ids // self.per_rank, torch.full_like(ids, -1))
        ranks = torch.arange(self.world, device=ids.device).view(-1, 1, 1)
        local = ids.unsqueeze(0) - ranks * self.per_rank
        return torch.where(owner.unsqueeze(0) == ranks, local, torch.full_like(local, -1)).to(torch.int32)

    def _static(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, local_fn: LocalFn) -> torch.Tensor:
        T, H = x.shape
        k = ids.size(1)
        W = self.world
        meta = torch.cat([self.local_ids(ids), w.unsqueeze(0).expand(W, T, k).contiguous().view(torch.int32)],
                         dim=2).contiguous()  # [W, T, 2k]
        send_x = x.unsqueeze(0).expand(W, T, H).contiguous()
        recv_x = torch.empty_like(send_x)
        recv_meta = torch.empty_like(meta)
        dist.all_to_all_single(recv_x, send_x, group=self.group)
        dist.all_to_all_single(recv_meta, meta, group=self.group)
        rows = W * T
        recv_ids = recv_meta[:, :, :k].reshape(rows, k)
        recv_w = recv_meta[:, :, k:].reshape(rows, k).contiguous().view(torch.float32)
        # rows with a local expert first (stable, on the device): when local_fn works in
        # chunks of rows, the chunks past them route no pair and stream no codes
        order = torch.argsort((recv_ids < 0).all(1).to(torch.int8), stable=True)
        y_c = local_fn(recv_x.view(rows, H).index_select(0, order), recv_ids.index_select(0, order).contiguous(),
                       recv_w.index_select(0, order).contiguous()).to(torch.float32)
        if y_c.shape != (rows, H):
            raise RuntimeError("local expert function must return [rows, hidden]")
        y = torch.empty_like(y_c)
        y.index_copy_(0, order, y_c)
        back = torch.empty_like(y)
        dist.all_to_all_single(back, y, group=self.group)
        return back.view(W, T, H).sum(0)

    def plan(self, topk_ids: torch.Tensor):
        """Destination rows of a call: token index per send row (grouped by
        destination rank), the destination rank of each row and the per-rank counts."""
        ids = topk_ids.to(torch.long)
        valid = (ids >= 0) & (ids < self.n_experts)
        dest = torch.where(valid, ids // self.per_rank, torch.full_like(ids, -1))
        T = ids.size(0)
        mask = torch.zeros((T, self.world + 1), dtype=torch.bool, device=ids.device)
        mask.scatter_(1, torch.where(dest < 0, torch.full_like(dest, self.world), dest), True)
        pairs = mask[:, : self.world].t().nonzero()  # (rank, token), rank-major then token order
        send_rank = pairs[:, 0]
        send_tok = pairs[:, 1]
        counts = torch.bincount(send_rank, minlength=self.world)
        return send_tok, send_rank, dest, counts

    def __call__(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                 local_fn: LocalFn) -> torch.Tensor:
        """``out [T, H]`` fp32 = sum over each token's experts (wherever they live)."""
        if x.dim() != 2:
            raise RuntimeError("EP MoE input must be [tokens, hidden]")
        T, H = x.shape
        k = topk_ids.shape[-1]
        ids = topk_ids.reshape(T, k).to(torch.long)
        w = topk_weights.reshape(T, k).to(torch.float32)
        if self.static:
            if T == 0:
                return torch.zeros((0, H), dtype=torch.float32, device=x.device)
            return self._static(x, ids, w, local_fn)
        send_tok, send_rank, dest, counts = self.plan(ids)

        # rows to send: the token, its ids local to the destination (-1 elsewhere), weights
        row_dest = dest[send_tok]
        local_ids = torch.where(row_dest == send_rank[:, None], ids[send_tok] - send_rank[:, None] * self.per_rank,
                                torch.full_like(row_dest, -1)).to(torch.int32)
        meta = torch.cat([local_ids, w[send_tok].contiguous().view(torch.int32)], dim=1).contiguous()
        send_x = x[send_tok].contiguous()

        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        send_splits = counts.tolist()
        recv_splits = recv_counts.tolist()
        self.last_counts = (tuple(send_splits), tuple(recv_splits))
        R = int(sum(recv_splits))

        recv_x = torch.empty((R, H), dtype=x.dtype, device=x.device)
        recv_meta = torch.empty((R, 2 * k), dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_x, send_x, recv_splits, send_splits, group=self.group)
        dist.all_to_all_single(recv_meta, meta, recv_splits, send_splits, group=self.group)
        recv_ids = recv_meta[:, :k].contiguous()
        recv_w = recv_meta[:, k:].contiguous().view(torch.float32)

        if R > 0:
            y = local_fn(recv_x, recv_ids, recv_w).to(torch.float32).contiguous()
        else:
            y = torch.empty((0, H), dtype=torch.float32, device=x.device)
        if y.shape != (R, H):
            raise RuntimeError("local expert function must return [rows, hidden]")
        back = torch.empty((send_tok.numel(), H), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(back, y, send_splits, recv_splits, group=self.group)
        out = torch.zeros((T, H), dtype=torch.float32, device=x.device)
        out.index_add_(0, send_tok, back)
        return out


_TABLE_NAMES = ("gate_trellis", "gate_suh", "gate_svh", "up_trellis", "up_suh", "up_svh",
                "down_trellis", "down_suh", "down_svh")


class PeerExpertParallelMoE:
    """Expert parallelism with the dispatch and the combine over NVLink peer memory
    (``exl3b200_ep_moe``): a token row goes once to every rank that owns one of its
    experts, each rank runs its local experts on what it received, and the weighted
    results come back to the token's rank, all on the device (no NCCL, no host
    synchronisation, graph-capturable).  Each rank holds its own tokens (at most
    ``max_tokens``).  The peer buffers are allocated once and mapped into every rank
    through CUDA IPC handles exchanged with ``all_gather_object``; ``close`` (every
    rank, before the process group goes away) unmaps and frees them.  Without a
    process group (``world == 1``) the exchange runs with the rank itself."""

    def __init__(self, n_experts: int, max_tokens: int, topk: int, hidden: int, group=None):
        import ctypes

        from . import _lib

        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        if self.world > 8 or n_experts % self.world:
            raise RuntimeError(f"{n_experts} experts over {self.world} ranks (at most 8, evenly) are not supported")
        self.group = group
        self.n_experts, self.max_tokens, self.topk, self.hidden = n_experts, max_tokens, topk, hidden
        L = _lib.lib()
        size = L.exl3b200_ep_buffer_size(self.world, max_tokens, topk, hidden)
        if size == 0:
            raise RuntimeError("bad expert-parallel buffer shape")
        handle = (ctypes.c_char * 64)()
        own = ctypes.c_void_p()
        _lib.check(L.exl3b200_peer_buffer_alloc(size, ctypes.byref(own), handle), "exl3b200_peer_buffer_alloc")
        self._own = own.value
        self._opened = []
        ptrs = [self._own]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
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
            dist.barrier(group)
        self.struct = _lib.Peers((ctypes.c_void_p * 8)(*(ptrs + [None] * (8 - len(ptrs)))), self.world, self.rank,
                                 max_tokens, hidden)

    def __call__(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, tables: dict,
                 K_gate: int, K_up: int, K_down: int, cb: int, intermediate_size: int, swiglu_limit: float = 0.0,
                 path: int = -1, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``out [T, H]`` fp32: every token's routed SwiGLU experts, wherever they live.
        ``tables``: the nine int64 device pointer tables of this rank's experts."""
        import ctypes

        from . import _lib, workspace

        T, H = x.shape
        if H != self.hidden or T > self.max_tokens:
            raise RuntimeError("expert-parallel input does not fit the buffers")
        if x.dtype != torch.float16:
            raise RuntimeError("expert-parallel input must be fp16")
        if x.stride(-1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
            x = x.contiguous()
        ids = topk_ids.reshape(T, -1).to(torch.int32).contiguous()
        w = topk_weights.reshape(T, -1).to(torch.float32).contiguous()
        if ids.size(1) != self.topk:
            raise RuntimeError("top-k does not match the buffers")
        if out is None:
            out = torch.empty((T, H), dtype=torch.float32, device=x.device)
        tabs = [tables[nm].contiguous() for nm in _TABLE_NAMES]
        tab_ptrs = (ctypes.c_void_p * 9)(*[t.data_ptr() for t in tabs])
        args = _lib.EpArgs(x.data_ptr(), x.stride(0), T, self.max_tokens, H, int(intermediate_size), ids.data_ptr(),
                           w.data_ptr(), self.topk, self.n_experts, ctypes.cast(tab_ptrs, ctypes.c_void_p), int(K_gate),
                           int(K_up), int(K_down), int(cb), float(swiglu_limit or 0.0), out.data_ptr(), out.stride(0),
                           int(path))
        L = _lib.lib()
        st_n, sc_n = ctypes.c_size_t(), ctypes.c_size_t()
        _lib.check(L.exl3b200_ep_workspace(ctypes.byref(args), ctypes.byref(self.struct), ctypes.byref(st_n),
                                           ctypes.byref(sc_n)), "exl3b200_ep_workspace")
        dev = x.device
        with torch.cuda.device(dev):
            state = workspace.state_buffer(dev, max(256, st_n.value))
            scratch = workspace.scratch_buffer(dev, sc_n.value)
            rc = L.exl3b200_ep_moe(ctypes.byref(args), ctypes.byref(self.struct), state.data_ptr(), state.numel(),
                                   scratch.data_ptr(), scratch.numel(), torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(rc, "exl3b200_ep_moe")
        self._keep = (ids, w, tabs, tab_ptrs)  # alive until the enqueued call ran (and for graph replays)
        return out

    def reset(self) -> None:
        """Re-arm after a wait gave up (every rank together)."""
        from . import _lib

        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(self.group)
        _lib.check(_lib.lib().exl3b200_peer_reset(self._own, torch.cuda.current_stream().cuda_stream),
                   "exl3b200_peer_reset")
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(self.group)

    def close(self) -> None:
        from . import _lib

        if self._own is None:
            return
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(self.group)
        L = _lib.lib()
        for p in self._opened:
            L.exl3b200_peer_buffer_close(p)
        self._opened = []
        if self.world > 1:
            dist.barrier(self.group)
        L.exl3b200_peer_buffer_free(self._own)
        self._own = None


def exl3_local_experts(tables: dict, K_gate: int, K_up: int, K_down: int, cb: int, intermediate_size: int,
                       swiglu_limit: float = 0.0) -> LocalFn:
    """``local_fn`` running this rank's experts with the fused device MoE pipeline
    (``exl3_b200.moe.moe_forward``), in chunks of at most 2048 (token, slot) pairs."""
    from . import moe as _moe

    def fn(xr: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        xr = xr.to(torch.float16).contiguous()
        rows, k = ids.shape
        chunk = max(1, _moe.MOE_MAX_PAIRS // k)
        cap = _moe.workspace_tokens(rows, chunk)
        out = torch.empty((rows, xr.size(1)), dtype=torch.float32, device=xr.device)
        for r0 in range(0, rows, chunk):
            r1 = min(rows, r0 + chunk)
            _moe.moe_forward(xr[r0:r1], ids[r0:r1], w[r0:r1], tables, K_gate, K_up, K_down, cb,
                             intermediate_size, swiglu_limit, out=out[r0:r1], max_tokens=cap)
        return out

    return fn
