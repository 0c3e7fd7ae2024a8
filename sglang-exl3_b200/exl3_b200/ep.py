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
