"""Tensor-parallel fused decode with the NVLink peer exchange (two GPUs) against
the same model with NCCL all-reduces: the residual stream agrees up to the order
of the partial sums and of the row sums of squares (which moves the next RMSNorm by
about one fp16 ulp: 2e-3 normwise, as the single-GPU partial path), greedy tokens
are equal, a CUDA-graph replay of the peer path
equals its eager steps, and no device wait gave up.  Skipped without two GPUs.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _tame(m):
    for L in m.layers:
        for lin in L["qkv"] + [L["o"]] + L["gu"] + [L["down"]]:
            lin[2].mul_(float(lin[0].size(0) * 16) ** -0.5)
    return m


def _worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from exl3_b200 import ops
        from exl3_b200.harness import DecodeModel, DecoderConfig

        cfg = DecoderConfig(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, inter=1024, vocab=512, K=4, cb=0)
        group = dist.group.WORLD
        ms = [_tame(DecodeModel(cfg, batch=2, max_ctx=96, device=dev, world=world, rank=rank, group=group,
                                fused=True, peer=peer)) for peer in (False, True)]
        assert ms[1].peers is not None and ms[0].peers is None
        for m in ms:
            m.fill_random_kv(20)
            m.tokens.copy_(torch.tensor([3, 5], device=dev))
        for _ in range(3):
            for m in ms:
                m.step()
            torch.cuda.synchronize()
            err = ((ms[1].h - ms[0].h).abs().max() / ms[0].h.abs().max()).item()
            assert err < 2e-3, err
            assert torch.equal(ms[1].next_tokens, ms[0].next_tokens)
        # graph replay of the peer path continues the same sequence as eager steps
        m = ms[1]
        kv0 = (m.k_cache.clone(), m.v_cache.clone())
        pos0, tok0 = int(m.pos.item()), m.tokens.clone()
        eager = []
        for _ in range(3):
            m.step()
            eager.append(m.next_tokens.clone())
        m.k_cache.copy_(kv0[0])
        m.v_cache.copy_(kv0[1])
        m.pos.fill_(pos0)
        m.tokens.copy_(tok0)
        m.capture()
        m.pos.fill_(pos0)
        m.tokens.copy_(tok0)
        for i in range(3):
            m.decode(1)
            torch.cuda.synchronize()
            assert torch.equal(m.next_tokens, eager[i])
        assert ops.device_status(dev) == 0
        for m in ms:
            m.close()
    finally:
        dist.destroy_process_group()


def test_peer_exchange_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_worker, args=(2, port), nprocs=2, join=True, start_method="spawn")
