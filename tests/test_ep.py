"""Expert-parallel dispatch/combine (exl3_b200.ep) with two gloo ranks on CPU.

The local expert function is a host-side stand-in (expert e maps x to
x * (e + 1) + e), so the test checks the routing, the all-to-all exchanges and
the per-token combine against a single-process sum over all experts, including
invalid ids (skipped), tokens whose experts all live on one rank and a rank that
receives nothing.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from exl3_b200.ep import ExpertParallelMoE

E, H, K = 8, 16, 3


def _expert(e, x):
    return x * (e + 1) + e


def _reference(x, ids, w):
    out = torch.zeros(x.shape, dtype=torch.float32)
    for t in range(x.size(0)):
        for j in range(ids.size(1)):
            e = int(ids[t, j])
            if 0 <= e < E:
                out[t] += w[t, j] * _expert(e, x[t].float())
    return out


def _cases():
    g = torch.Generator().manual_seed(7)
    x = torch.randn(11, H, generator=g).half()
    ids = torch.randint(0, E, (11, K), generator=g)
    ids[3] = torch.tensor([-1, 9, 2])        # invalid ids are skipped
    ids[5] = torch.tensor([0, 1, 2])         # all experts on rank 0
    w = torch.rand(11, K, generator=g)
    only_low = torch.randint(0, E // 2, (6, K), generator=g)  # rank 1 receives nothing
    return [(x, ids, w), (x[:6], only_low, w[:6]), (x[:0], ids[:0], w[:0])]


def _worker(rank, world, port, results, static):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ep = ExpertParallelMoE(E, world, rank, static=static)

        def local_fn(xr, lids, lw):
            out = torch.zeros(xr.shape, dtype=torch.float32)
            for r in range(xr.size(0)):
                for j in range(lids.size(1)):
                    le = int(lids[r, j])
                    if le >= 0:
                        out[r] += lw[r, j] * _expert(rank * ep.per_rank + le, xr[r].float())
            return out

        for ci, (x, ids, w) in enumerate(_cases()):
            got = ep(x, ids, w, local_fn)
            torch.testing.assert_close(got, _reference(x, ids, w), rtol=1e-5, atol=1e-5)
            if ci == 1 and rank == 1 and not static:
                results.put(("recv_rank1_case1", ep.last_counts[1]))
        results.put(("ok", rank))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("static", [True, False])
def test_ep_dispatch_combine_two_ranks(static):
    """Both exchange modes: fixed-size (no host read) and variable-size."""
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    mp.start_processes(_worker, args=(2, _free_port(), results, static), nprocs=2, join=True, start_method="spawn")
    got = [results.get(timeout=30) for _ in range(2 if static else 3)]
    assert sorted(r for k, r in got if k == "ok") == [0, 1]
    if not static:
        assert [v for k, v in got if k == "recv_rank1_case1"] == [(0, 0)]


def test_ep_local_ids_per_rank():
    ep = ExpertParallelMoE(8, 4, 0)
    ids = torch.tensor([[0, 7, 6], [3, 2, 2], [-1, 8, 5]])
    lid = ep.local_ids(ids)
    assert lid.shape == (4, 3, 3)
    assert lid[0].tolist() == [[0, -1, -1], [-1, -1, -1], [-1, -1, -1]]
    assert lid[1].tolist() == [[-1, -1, -1], [1, 0, 0], [-1, -1, -1]]
    assert lid[2].tolist() == [[-1, -1, -1], [-1, -1, -1], [-1, -1, 1]]
    assert lid[3].tolist() == [[-1, 1, 0], [-1, -1, -1], [-1, -1, -1]]


def test_ep_plan_groups_rows_by_destination():
    ep = ExpertParallelMoE(8, 4, 0)
    ids = torch.tensor([[0, 7, 6], [3, 2, 2], [-1, 8, 5]])
    send_tok, send_rank, dest, counts = ep.plan(ids)
    # token 0 -> ranks 0 and 3, token 1 -> rank 1, token 2 -> rank 2 (ids -1 and 8 are invalid)
    assert counts.tolist() == [1, 1, 1, 1]
    assert send_rank.tolist() == [0, 1, 2, 3]
    assert send_tok.tolist() == [0, 1, 2, 0]


def test_ep_rejects_uneven_split():
    with pytest.raises(ValueError):
        ExpertParallelMoE(10, 4, 0)
