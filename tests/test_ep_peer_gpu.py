"""Expert parallelism over NVLink peer memory (exl3b200_ep_moe) on the GPU.

One rank (no process group): the dispatch, receive, return and combine kernels run
against the rank's own buffer, and the result must equal the routed MoE pipeline
on the same experts (same rows, same weights; only the order of the fp32 atomics
differs) and the oracle; several calls in a row alternate the buffer's parity; a
CUDA graph of one call replays correctly.  A two-rank exchange whose second rank
never answers (its buffer is local memory nobody writes) must give up within the
wait limit, record EXL3B200_ETIMEOUT and recover after exl3b200_peer_reset.  On 2, 4
and 8 GPUs (skipped with fewer): every rank owns 1/world of the experts and its own
tokens; each rank's output equals the single-GPU MoE over all experts for its tokens.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import exl3_oracle as O

pytestmark = pytest.mark.gpu

# Same experts, same rows and weights; the pipeline runs over a different row count
# (the receive regions), so its MMAs group and accumulate in another order, and where
# that moves a gate/up value across an fp16 rounding boundary the SwiGLU activation
# differs by one fp16 ulp: about 2^-11 / sqrt(intermediate) ~ 2.5e-5 of the output
# norm per flipped element.  Several flips stay well below 5e-4.
TOL_SAME = 5e-4
TOL_MOE = 4e-3    # the routed-MoE oracle tolerance (fp16 SwiGLU intermediate)


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _experts(seed, E, H, I, K, cb):
    rng = np.random.default_rng(seed)
    ex = []
    for _ in range(E):
        e = {}
        for which, (k, n) in (("gate", (H, I)), ("up", (H, I)), ("down", (I, H))):
            sv = O.random_signs(rng, n)
            if which != "down":
                sv = (sv.astype(np.float32) * k ** -0.5).astype(np.float16)
            e[which] = (O.random_trellis(rng, k, n, K), O.random_signs(rng, k), sv, K, cb)
        ex.append(e)
    return ex


def _tables(experts, dev):
    keep, tabs = [], {}
    for which in ("gate", "up", "down"):
        cols = [[_t(e[which][i], dev) for e in experts] for i in range(3)]
        keep += cols[0] + cols[1] + cols[2]
        for name, ts in zip(("trellis", "suh", "svh"), cols):
            tabs[f"{which}_{name}"] = torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=dev)
    return tabs, keep


def _route(rng, T, E, topk):
    logits = rng.standard_normal((T, E))
    ids = np.argsort(-logits, axis=1)[:, :topk].astype(np.int32)
    w = np.take_along_axis(logits, ids, 1)
    return ids, (np.exp(w) / np.exp(w).sum(1, keepdims=True)).astype(np.float32)


def _rel(a, b):
    return float((a.double() - b.double()).abs().max() / b.double().abs().max())


@pytest.mark.parametrize("path", [0, 1])
def test_ep_peer_one_rank(cuda_device, path):
    from exl3_b200 import moe
    from exl3_b200.ep import PeerExpertParallelMoE

    E, H, I, K, cb, topk = 12, 256, 384, 3, 0, 4
    experts = _experts(11, E, H, I, K, cb)
    tabs, keep = _tables(experts, cuda_device)
    ep = PeerExpertParallelMoE(E, 256, topk, H)
    rng = np.random.default_rng(3)
    try:
        for T in (1, 37, 200, 5):  # several calls: the parity alternates
            x = (0.5 * rng.standard_normal((T, H))).astype(np.float16)
            ids, w = _route(rng, T, E, topk)
            xd, idd, wd = _t(x, cuda_device), _t(ids, cuda_device), _t(w, cuda_device)
            y = ep(xd, idd, wd, tabs, K, K, K, cb, I, path=path)
            ref = moe.moe_forward(xd, idd, wd, tabs, K, K, K, cb, I, path="tc" if path else "small")
            torch.cuda.synchronize()
            assert _rel(y, ref) < TOL_SAME, T
            assert O.normwise_rel_err(y.cpu().numpy(), O.moe_ref(x, experts, ids, w)) < TOL_MOE, T
        from exl3_b200 import ops
        assert ops.device_status(cuda_device) == 0
    finally:
        ep.close()


def test_ep_peer_graph_replay(cuda_device):
    from exl3_b200 import moe
    from exl3_b200.ep import PeerExpertParallelMoE

    E, H, I, K, cb, topk, T = 8, 256, 256, 4, 1, 2, 24
    experts = _experts(12, E, H, I, K, cb)
    tabs, keep = _tables(experts, cuda_device)
    ep = PeerExpertParallelMoE(E, T, topk, H)
    rng = np.random.default_rng(4)
    x = _t((0.5 * rng.standard_normal((T, H))).astype(np.float16), cuda_device)
    ids0, w0 = _route(rng, T, E, topk)
    idd, wd = _t(ids0, cuda_device), _t(w0, cuda_device)
    out = torch.empty((T, H), dtype=torch.float32, device=cuda_device)
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    try:
        with torch.cuda.stream(s):
            for _ in range(2):
                ep(x, idd, wd, tabs, K, K, K, cb, I, out=out)
        torch.cuda.current_stream(cuda_device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            ep(x, idd, wd, tabs, K, K, K, cb, I, out=out)
        for trial in range(3):  # replays alternate the parity on the device
            ids, w = _route(rng, T, E, topk)
            idd.copy_(_t(ids, cuda_device))
            wd.copy_(_t(w, cuda_device))
            g.replay()
            torch.cuda.synchronize()
            ref = moe.moe_forward(x, idd, wd, tabs, K, K, K, cb, I)
            assert _rel(out, ref) < TOL_SAME, trial
    finally:
        del g
        ep.close()


def test_ep_peer_wait_runs_out(cuda_device):
    """Two-rank exchange on one GPU whose rank 1 is a buffer nobody fills: the receive
    wait must give up (10 ms limit), record the status, poison the buffer and return
    zeros; after re-arming, a one-rank exchange on the same buffer is correct.  Both
    buffers are plain device memory sized for two ranks."""
    import ctypes

    from exl3_b200 import _lib, moe, ops
    from exl3_b200.ep import PeerExpertParallelMoE

    E, H, I, K, cb, topk, T = 8, 256, 256, 3, 0, 2, 16
    experts = _experts(13, E, H, I, K, cb)
    tabs, keep = _tables(experts, cuda_device)
    L = _lib.lib()
    size = L.exl3b200_ep_buffer_size(2, T, topk, H)
    own = torch.zeros(size, dtype=torch.uint8, device=cuda_device)
    fake = torch.zeros(size, dtype=torch.uint8, device=cuda_device)
    ep = object.__new__(PeerExpertParallelMoE)  # buffers supplied here, not allocated by the class
    ep.rank, ep.group, ep.max_tokens, ep.topk, ep.hidden = 0, None, T, topk, H
    ep.world, ep.n_experts = 2, 2 * E
    ep.struct = _lib.Peers((ctypes.c_void_p * 8)(own.data_ptr(), fake.data_ptr(), *[None] * 6), 2, 0, T, H)
    rng = np.random.default_rng(5)
    x = _t((0.5 * rng.standard_normal((T, H))).astype(np.float16), cuda_device)
    ids, w = _route(rng, T, 2 * E, topk)  # global ids over two ranks of E experts
    idd, wd = _t(ids, cuda_device), _t(w, cuda_device)
    ops.device_status(cuda_device)
    ops.set_wait_limit(0.01)
    try:
        y = ep(x, idd, wd, tabs, K, K, K, cb, I)
        torch.cuda.synchronize()
        assert ops.device_status(cuda_device) == _lib.ETIMEOUT
        assert float(y.abs().max()) == 0.0
        assert own[:16].view(torch.int32).tolist()[3] == 1  # poisoned
    finally:
        ops.set_wait_limit(None)
    _lib.check(L.exl3b200_peer_reset(own.data_ptr(), torch.cuda.current_stream(cuda_device).cuda_stream),
               "exl3b200_peer_reset")
    ep.world, ep.n_experts = 1, E
    ep.struct = _lib.Peers((ctypes.c_void_p * 8)(own.data_ptr(), *[None] * 7), 1, 0, T, H)
    ids1, w1 = _route(rng, T, E, topk)
    idd1, wd1 = _t(ids1, cuda_device), _t(w1, cuda_device)
    y = ep(x, idd1, wd1, tabs, K, K, K, cb, I)
    ref = moe.moe_forward(x, idd1, wd1, tabs, K, K, K, cb, I)
    torch.cuda.synchronize()
    assert ops.device_status(cuda_device) == 0
    assert _rel(y, ref) < TOL_SAME


def _rank_worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from exl3_b200 import moe, ops
        from exl3_b200.ep import PeerExpertParallelMoE

        E, H, I, K, cb, topk = 16, 256, 384, 3, 0, 4
        experts = _experts(21, E, H, I, K, cb)   # the same weights on every rank
        per = E // world
        local_tabs, keep = _tables(experts[rank * per:(rank + 1) * per], dev)
        all_tabs, keep2 = _tables(experts, dev)
        ep = PeerExpertParallelMoE(E, 128, topk, H, group=dist.group.WORLD)
        rng = np.random.default_rng(100 + rank)  # every rank its own tokens
        for T in (3, 128, 40):
            x = _t((0.5 * rng.standard_normal((T, H))).astype(np.float16), dev)
            ids, w = _route(rng, T, E, topk)
            idd, wd = _t(ids, dev), _t(w, dev)
            for path in (0, 1):
                y = ep(x, idd, wd, local_tabs, K, K, K, cb, I, path=path)
                # the same pipeline on one GPU (the two pipelines differ by up to the MoE tolerance)
                ref = moe.moe_forward(x, idd, wd, all_tabs, K, K, K, cb, I, path="tc" if path else "small")
                torch.cuda.synchronize()
                assert _rel(y, ref) < TOL_SAME, (rank, T, path, _rel(y, ref))
        assert ops.device_status(dev) == 0
        ep.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_peer_multi_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_rank_worker, args=(world, port), nprocs=world, join=True, start_method="spawn")
