"""Tensor-parallel fused decode with the NVLink peer exchange (two GPUs) against
the same model with NCCL all-reduces: the residual stream agrees up to the order
of the partial sums and of the row sums of squares (which moves the next RMSNorm by
about one fp16 ulp: 2e-3 normwise, as the single-GPU partial path), greedy tokens
are equal, CUDA-graph replays of the peer paths
agree with their eager steps, and no device wait gave up.  Whole layers with the RMSNorm
folded into the exchange epilogues agree with the NCCL model to 5e-3 in the residual
stream (fp16 rounding at other points) and 1e-2 in the bf16 logits.  Skipped without two GPUs.
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
                                fused=True, peer=peer, fold=fold)) for peer, fold in ((False, False), (True, False),
                                                                                       (True, True))]
        assert ms[1].peers is not None and ms[0].peers is None and ms[2].fold and not ms[1].fold
        for m in ms:
            m.fill_random_kv(20)
            m.tokens.copy_(torch.tensor([3, 5], device=dev))
        rel = lambda a, b: ((a - b).abs().max() / b.abs().max()).item()  # noqa: E731
        for _ in range(3):
            for m in ms:
                m.step()
            torch.cuda.synchronize()
            err = rel(ms[1].h, ms[0].h)
            assert err < 2e-3, err
            assert torch.equal(ms[1].next_tokens, ms[0].next_tokens)
            # whole layers with the RMSNorm folded into the exchange epilogues
            assert rel(ms[2].h, ms[0].h) < 5e-3
            assert rel(ms[2].last_logits.float(), ms[0].last_logits.float()) < 1e-2  # bf16 logits
            ms[2].tokens.copy_(ms[0].tokens)
        # graph replay of the peer paths continues the same sequence as eager steps
        for m in ms[1:]:
            _replay_matches_eager(m, m.tokens.clone(), int(m.pos.item()), 3)
        assert ops.device_status(dev) == 0
        for m in ms:
            m.close()
    finally:
        dist.destroy_process_group()


def _replay_matches_eager(m, tokens0, pos0, steps):
    """Eager steps, then the captured graph from the same state.  Each replay is fed the
    eager step's input tokens.  The fused step is not bitwise repeatable: the order of
    the fp32 atomic sums (split-K partials, the rows' sums of squares) moves values by
    ulps, and where that flips the bf16 rounding of an appended K/V entry (2^-8) the
    attention output follows - two eager runs of this model differ by ~1e-3 of the
    residual stream.  So the residual stream must agree to 5e-3, the bf16 logits to
    1e-2, and a greedy token may differ only at a near-tie."""
    rel = lambda a, b: ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()  # noqa: E731
    kv0 = (m.k_cache.clone(), m.v_cache.clone())
    m.pos.fill_(pos0)
    m.tokens.copy_(tokens0)
    eager = []
    for _ in range(steps):
        tin = m.tokens.clone()
        m.step()
        eager.append((tin, m.h.clone(), m.last_logits.float().clone(), m.next_tokens.clone()))
    m.k_cache.copy_(kv0[0])
    m.v_cache.copy_(kv0[1])
    m.pos.fill_(pos0)
    m.tokens.copy_(tokens0)
    m.capture()
    m.pos.fill_(pos0)
    for tin, h, logits, tok in eager:
        m.tokens.copy_(tin)
        m.decode(1)
        torch.cuda.synchronize()
        assert rel(m.h, h) < 5e-3
        assert rel(m.last_logits, logits) < 1e-2
        top = logits.max(-1).values
        picked = logits.gather(-1, m.next_tokens.view(-1, 1)).squeeze(-1)
        assert bool(torch.all((m.next_tokens == tok) | (top - picked <= 2.0 ** -7 * top.abs())))
    m.release()


def test_peer_exchange_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_worker, args=(2, port), nprocs=2, join=True, start_method="spawn")
