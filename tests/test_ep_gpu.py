"""Expert-parallel MoE over NCCL on two GPUs against the single-GPU fused MoE.

Each rank builds the same 16 experts (seeded), keeps its half for the EP call and
runs the whole layer alone as the reference; outputs must agree to fp32
accumulation tolerance.  Skipped unless two GPUs are visible.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

E, TOPK, H, I, K, T = 16, 4, 256, 256, 3, 37


def _worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from exl3_b200 import moe as M
        from exl3_b200.ep import ExpertParallelMoE, exl3_local_experts

        g = torch.Generator(device=dev).manual_seed(11)
        w13 = torch.randint(-32768, 32768, (E, 2, H // 16, I // 16, 16 * K), dtype=torch.int16, device=dev, generator=g)
        w2 = torch.randint(-32768, 32768, (E, I // 16, H // 16, 16 * K), dtype=torch.int16, device=dev, generator=g)

        def signs(*shape):
            return (torch.randint(0, 2, shape, device=dev, generator=g) * 2 - 1).half()

        w13_suh, w13_svh, w2_suh, w2_svh = signs(E, 2, H), signs(E, 2, I), signs(E, I), signs(E, H)

        def tables(lo, hi):
            def p(t):
                return torch.tensor([int(t[e].data_ptr()) for e in range(lo, hi)], dtype=torch.int64, device=dev)
            return {"gate_trellis": p(w13[:, 0]), "gate_suh": p(w13_suh[:, 0]), "gate_svh": p(w13_svh[:, 0]),
                    "up_trellis": p(w13[:, 1]), "up_suh": p(w13_suh[:, 1]), "up_svh": p(w13_svh[:, 1]),
                    "down_trellis": p(w2), "down_suh": p(w2_suh), "down_svh": p(w2_svh)}

        x = (torch.randn(T, H, device=dev, generator=g) * 0.5).half()
        ids = torch.randint(0, E, (T, TOPK), device=dev, generator=g)
        ids[0, 0] = -1
        w = torch.rand(T, TOPK, device=dev, generator=g)
        ref = M.moe_forward(x, ids.to(torch.int32), w, tables(0, E), K, K, K, 0, I)
        per = E // world
        local = exl3_local_experts(tables(rank * per, (rank + 1) * per), K, K, K, 0, I)
        for static in (True, False):
            ep = ExpertParallelMoE(E, world, rank, static=static)
            got = ep(x, ids, w, local)
            torch.cuda.synchronize()
            err = ((got - ref).abs().max() / ref.abs().max()).item()
            assert err < 2e-3, (static, err)

        # the static exchange has no host read: capture the whole EP layer in a CUDA
        # graph, replay it with new routing (same on both ranks: same seed)
        ep = ExpertParallelMoE(E, world, rank, static=True)
        ids_buf, w_buf = ids.clone(), w.clone()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                ep(x, ids_buf, w_buf, local)  # workspaces of the capture stream
        torch.cuda.current_stream(dev).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            out_g = ep(x, ids_buf, w_buf, local)
        try:
            for trial in range(2):
                new_ids = torch.randint(0, E, (T, TOPK), device=dev, generator=g)
                ids_buf.copy_(new_ids)
                graph.replay()
                torch.cuda.synchronize()
                ref2 = M.moe_forward(x, new_ids.to(torch.int32), w, tables(0, E), K, K, K, 0, I)
                err = ((out_g - ref2).abs().max() / ref2.abs().max()).item()
                assert err < 2e-3, ("graph", trial, err)
        finally:
            del graph  # a graph holding NCCL work goes before the process group
    finally:
        dist.destroy_process_group()


def test_ep_two_gpus_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_worker, args=(2, port), nprocs=2, join=True, start_method="spawn")
