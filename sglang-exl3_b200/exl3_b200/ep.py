"""Expert-parallel routed MoE: all-to-all dispatch and combine around the device
MoE pipeline.

The experts of a layer are split evenly over the ranks of a process group
(rank r owns global experts ``[r*E/W, (r+1)*E/W)``: the reference's EP layout,
whose id mapping is ``map_topk_to_local`` / ``_get_expert_map``,
``src/sglang_exl3/exl3.py:485-509``).  One MoE call:

1. every token goes once to each rank that owns at least one of its top-k experts,
   with its top-k ids rewritten to that rank's local ids (-1 where another rank
   owns the expert) and its routing weights;
2. the per-destination row counts are exchanged (``all_to_all_single`` on the
   counts; the host reads them to size the variable exchanges), then the token
   rows (fp16) and the packed ids/weights (int32);
3. each rank runs its local experts on what it received (``local_fn``: the fused
   device MoE pipeline, which skips id -1) into fp32 rows;
4. those rows go back with the reverse exchange and are summed per token.

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

    def __init__(self, n_experts: int, world: int, rank: int, group=None):
        if world < 1 or n_experts % world:
            raise ValueError(f"{n_experts} experts do not split evenly over {world} ranks")
        self.n_experts = n_experts
        self.world = world
        self.rank = rank
        self.group = group
        self.per_rank = n_experts // world
        self.last_counts: Optional[tuple] = None  # (send, recv) row counts of the last call

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
