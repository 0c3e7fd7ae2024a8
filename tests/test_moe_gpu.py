"""Grouped matmuls on the GPU against the oracle: fused multi-linear, batched
experts (p2b_gemv_batched), routed MoE (p2b_fused_moe / moe_forward), fat GEMM
and its scatter form.  Tolerance as for the matmul: normwise 2e-3 (fp32
accumulate); the MoE output passes through an fp16 activation, as in the
reference, and is held to 4e-3."""

import numpy as np
import pytest
import torch

import exl3_oracle as O
from exl3_b200 import moe, ops

pytestmark = pytest.mark.gpu

TOL = 2e-3
TOL_MOE = 4e-3


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _lin(rng, k, n, K):
    return O.random_trellis(rng, k, n, K), O.random_signs(rng, k), O.random_signs(rng, n)


@pytest.mark.parametrize("m", [5, 40])  # 40 rows: one tensor-core GEMM per linear
@pytest.mark.parametrize("K,cb", [(4, 0), (3, 1), (2, 2)])
def test_matmul_multi_qkv(cuda_device, K, cb, m):
    rng = np.random.default_rng(31 + K)
    lins = [_lin(rng, 512, n, K) for n in (512, 128, 128)]
    x = rng.standard_normal((m, 512)).astype(np.float16)
    dev_lins = [tuple(_t(a, cuda_device) for a in lin) for lin in lins]
    fused = torch.zeros((m, 768), dtype=torch.float16, device=cuda_device)
    outs = [fused[:, 0:512], fused[:, 512:640], fused[:, 640:768]]
    ops.matmul_multi(_t(x, cuda_device), dev_lins, K, cb, outs=outs)
    for (tr, su, sv), o in zip(lins, outs):
        assert O.normwise_rel_err(o.float().cpu().numpy(), O.gemv_ref(x, tr, su, sv, K, cb)) < TOL


def _experts(rng, E, H, I, K):
    ex = []
    for _ in range(E):
        ex.append({"gate": _lin(rng, H, I, K) + (K, 0), "up": _lin(rng, H, I, K) + (K, 0),
                   "down": _lin(rng, I, H, K) + (K, 0)})
    return ex


def _tables(experts, dev, cb):
    keep = []
    tabs = {}
    for which in ("gate", "up", "down"):
        tr = [_t(e[which][0], dev) for e in experts]
        su = [_t(e[which][1], dev) for e in experts]
        sv = [_t(e[which][2], dev) for e in experts]
        keep += tr + su + sv
        tabs[f"{which}_trellis"] = torch.tensor([t.data_ptr() for t in tr], dtype=torch.int64, device=dev)
        tabs[f"{which}_suh"] = torch.tensor([t.data_ptr() for t in su], dtype=torch.int64, device=dev)
        tabs[f"{which}_svh"] = torch.tensor([t.data_ptr() for t in sv], dtype=torch.int64, device=dev)
    return tabs, keep


def _with_cb(experts, cb):
    return [{w: e[w][:4] + (cb,) for w in e} for e in experts]


@pytest.mark.parametrize("cb", [0, 1, 2])
@pytest.mark.parametrize("per_expert", [False, True])
def test_p2b_gemv_batched(cuda_device, cb, per_expert):
    rng = np.random.default_rng(40 + cb + 3 * per_expert)
    E, H, I, K, m = 6, 256, 384, 3, 2
    experts = _experts(rng, E, H, I, K)
    tabs, keep = _tables(experts, cuda_device, cb)
    ids = np.array([4, 1, 1, 5], dtype=np.int32)
    x = rng.standard_normal((len(ids), m, H) if per_expert else (m, H)).astype(np.float16)
    out = moe.p2b_gemv_batched(_t(x, cuda_device), tabs["gate_trellis"], tabs["gate_suh"], tabs["gate_svh"],
                               _t(ids, cuda_device), K, False, I, cb=cb)
    assert out.shape == (len(ids), m, I)
    for j, e in enumerate(ids):
        tr, su, sv = experts[e]["gate"][:3]
        xe = x[j] if per_expert else x
        assert O.normwise_rel_err(out[j].float().cpu().numpy(), O.gemv_ref(xe, tr, su, sv, K, cb)) < TOL


@pytest.mark.parametrize("path", ["small", "tc"])
@pytest.mark.parametrize("T,topk,E", [(1, 8, 16), (5, 4, 8), (16, 8, 12), (40, 2, 6), (600, 8, 16)])
@pytest.mark.parametrize("cb", [0, 1])
def test_moe_forward(cuda_device, T, topk, E, cb, path):
    """Both pipelines at every size: the tensor-core one from 1 row per expert to
    300 (two 256-row tiles, one of them with both 128-row accumulators)."""
    rng = np.random.default_rng(1000 * T + 10 * topk + cb)
    H, I, K = 256, 384, 3
    experts = _with_cb(_experts(rng, E, H, I, K), cb)
    tabs, keep = _tables(experts, cuda_device, cb)
    x = rng.standard_normal((T, H)).astype(np.float16)
    logits = rng.standard_normal((T, E))
    ids = np.argsort(-logits, axis=1)[:, :topk].astype(np.int32)
    w = np.take_along_axis(logits, ids, 1)
    w = (np.exp(w) / np.exp(w).sum(1, keepdims=True)).astype(np.float32)
    y = moe.moe_forward(_t(x, cuda_device), _t(ids, cuda_device), _t(w, cuda_device), tabs, K, K, K, cb, I,
                        path=path)
    ref = O.moe_ref(x, experts, ids, w)
    assert O.normwise_rel_err(y.cpu().numpy(), ref) < TOL_MOE


@pytest.mark.parametrize("T,topk,E", [(40, 1, 16), (64, 2, 64)])
def test_moe_small_eight_row_problems(cuda_device, T, topk, E):
    """At most 4 rows per expert on average: the small-M pipeline groups an expert's rows
    in problems of up to 8 (one row group); a skewed routing gives one expert 20 rows
    (three problems) and leaves others empty."""
    rng = np.random.default_rng(77 + T + E)
    H, I, K, cb = 256, 384, 3, 0
    experts = _with_cb(_experts(rng, E, H, I, K), cb)
    tabs, keep = _tables(experts, cuda_device, cb)
    x = rng.standard_normal((T, H)).astype(np.float16)
    ids = rng.integers(0, E, size=(T, topk)).astype(np.int32)
    ids[:20, 0] = 3  # expert 3: at least 20 rows
    for r in range(20):  # keep a token's experts distinct
        for j in range(1, topk):
            if ids[r, j] == 3:
                ids[r, j] = 4
    w = rng.random((T, topk)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    y = moe.moe_forward(_t(x, cuda_device), _t(ids, cuda_device), _t(w, cuda_device), tabs, K, K, K, cb, I,
                        path="small")
    assert O.normwise_rel_err(y.cpu().numpy(), O.moe_ref(x, experts, ids, w)) < TOL_MOE


@pytest.mark.parametrize("path", ["small", "tc"])
def test_moe_invalid_ids_and_clip(cuda_device, path):
    rng = np.random.default_rng(77)
    T, topk, E, H, I, K, cb = 3, 3, 5, 256, 256, 4, 1
    experts = _with_cb(_experts(rng, E, H, I, K), cb)
    tabs, keep = _tables(experts, cuda_device, cb)
    x = (rng.standard_normal((T, H)) * 4).astype(np.float16)
    ids = np.array([[0, 7, 2], [-1, 4, 4], [3, 1, 9]], dtype=np.int32)  # 7, -1, 9 are not local
    w = rng.uniform(0.1, 1.0, size=(T, topk)).astype(np.float32)
    y = moe.moe_forward(_t(x, cuda_device), _t(ids, cuda_device), _t(w, cuda_device), tabs, K, K, K, cb, I,
                        swiglu_limit=1.5, path=path)
    ref = O.moe_ref(x, experts, ids, w, limit=1.5)
    assert O.normwise_rel_err(y.cpu().numpy(), ref) < TOL_MOE


@pytest.mark.parametrize("path", ["small", "tc"])
def test_moe_mixed_bits_and_accumulate(cuda_device, path):
    """gate/up/down with different K (two gate/up launches), then a shared expert
    added with accumulate."""
    rng = np.random.default_rng(78)
    T, topk, E, H, I = 4, 2, 4, 256, 256
    experts = []
    for _ in range(E):
        experts.append({"gate": _lin(rng, H, I, 2) + (2, 0), "up": _lin(rng, H, I, 3) + (3, 0),
                        "down": _lin(rng, I, H, 4) + (4, 0)})
    tabs, keep = _tables(experts, cuda_device, 0)
    shared = [{"gate": _lin(rng, H, I, 4) + (4, 0), "up": _lin(rng, H, I, 4) + (4, 0),
               "down": _lin(rng, I, H, 4) + (4, 0)}]
    stabs, keep2 = _tables(shared, cuda_device, 0)
    x = rng.standard_normal((T, H)).astype(np.float16)
    ids = np.array([[0, 3], [1, 2], [2, 2], [3, 0]], dtype=np.int32)
    w = rng.uniform(0.2, 0.8, size=(T, topk)).astype(np.float32)
    xd = _t(x, cuda_device)
    y = moe.moe_forward(xd, _t(ids, cuda_device), _t(w, cuda_device), tabs, 2, 3, 4, 0, I, path=path)
    ones = torch.ones((T, 1), dtype=torch.float32, device=cuda_device)
    zeros = torch.zeros((T, 1), dtype=torch.int32, device=cuda_device)
    moe.moe_forward(xd, zeros, ones, stabs, 4, 4, 4, 0, I, out=y, accumulate=True, path=path)
    ref = O.moe_ref(x, experts, ids, w) + O.moe_ref(x, shared, np.zeros((T, 1), np.int64), np.ones((T, 1), np.float32))
    assert O.normwise_rel_err(y.cpu().numpy(), ref) < TOL_MOE


def test_p2b_fused_moe_reference_signature(cuda_device):
    """One row, ids int32 [topk], fp16 weights, fp16 out (csrc/p2b_moe.cu:418-468)."""
    rng = np.random.default_rng(79)
    E, H, I, K = 8, 512, 256, 4
    experts = _with_cb(_experts(rng, E, H, I, K), 1)
    tabs, keep = _tables(experts, cuda_device, 1)
    x = rng.standard_normal((1, H)).astype(np.float16)
    ids = np.array([6, 0, 3, 5], dtype=np.int32)
    rw = np.array([0.4, 0.3, 0.2, 0.1], dtype=np.float16)
    out = torch.empty((1, H), dtype=torch.float16, device=cuda_device)
    moe.p2b_fused_moe(_t(x, cuda_device), out, tabs["gate_trellis"], tabs["gate_suh"], tabs["gate_svh"],
                      tabs["up_trellis"], tabs["up_suh"], tabs["up_svh"], tabs["down_trellis"], tabs["down_suh"],
                      tabs["down_svh"], _t(ids, cuda_device), _t(rw, cuda_device), K, K, K, True, I, 0.0)
    ref = O.moe_ref(x, experts, ids[None, :], rw.astype(np.float32)[None, :])
    assert O.normwise_rel_err(out.float().cpu().numpy(), ref) < TOL_MOE


@pytest.mark.parametrize("K,cb", [(4, 1), (3, 0)])
def test_fat_gemm_and_scatter(cuda_device, K, cb):
    rng = np.random.default_rng(90 + K)
    M, k, n = 37, 256, 384
    tr, su, sv = _lin(rng, k, n, K)
    x = rng.standard_normal((M, k)).astype(np.float16)
    a = O.input_transform(x, su)
    out = torch.zeros((M, n), dtype=torch.float32, device=cuda_device)
    moe.exl3_fat_gemm(_t(a, cuda_device), _t(tr, cuda_device), out, _t(sv, cuda_device), K, cb == 1, cb == 2, cb=cb)
    ref = O.fat_gemm_ref(a, tr, sv, K, cb)
    assert O.normwise_rel_err(out.cpu().numpy(), ref) < TOL
    tok = rng.integers(0, 9, size=M).astype(np.int64)
    rw = rng.uniform(0.1, 1.0, size=M).astype(np.float16)
    acc = torch.zeros((9, n), dtype=torch.float32, device=cuda_device)
    moe.exl3_fat_gemm_scatter(_t(a, cuda_device), _t(tr, cuda_device), acc, _t(sv, cuda_device),
                              _t(tok, cuda_device), _t(rw, cuda_device), K, cb == 1, cb == 2, cb=cb)
    exp = np.zeros((9, n), dtype=np.float64)
    for i in range(M):
        exp[tok[i]] += float(rw[i]) * ref[i]
    assert O.normwise_rel_err(acc.cpu().numpy(), exp) < TOL


@pytest.mark.parametrize("path", ["small", "tc"])
def test_moe_graph_capture_replay(cuda_device, path):
    rng = np.random.default_rng(81)
    T, topk, E, H, I, K = 2, 4, 8, 256, 256, 3
    experts = _with_cb(_experts(rng, E, H, I, K), 0)
    tabs, keep = _tables(experts, cuda_device, 0)
    x = _t(rng.standard_normal((T, H)).astype(np.float16), cuda_device)
    ids = _t(rng.integers(0, E, size=(T, topk)).astype(np.int32), cuda_device)
    w = _t(rng.uniform(0.1, 1, size=(T, topk)).astype(np.float32), cuda_device)
    out = torch.empty((T, H), dtype=torch.float32, device=cuda_device)
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):
        for _ in range(2):
            moe.moe_forward(x, ids, w, tabs, K, K, K, 0, I, out=out, path=path)
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        moe.moe_forward(x, ids, w, tabs, K, K, K, 0, I, out=out, path=path)
    for trial in range(2):
        new_ids = rng.integers(0, E, size=(T, topk)).astype(np.int32)
        ids.copy_(_t(new_ids, cuda_device))
        g.replay()
        torch.cuda.synchronize()
        ref = O.moe_ref(x.cpu().numpy(), experts, new_ids, w.cpu().numpy())
        assert O.normwise_rel_err(out.cpu().numpy(), ref) < TOL_MOE


@pytest.mark.parametrize("K,cb,rotated", [(4, 1, True), (3, 0, False), (2, 2, True)])
def test_matmul_combine_tensor_core(cuda_device, K, cb, rotated):
    """More than 16 rows: one tensor-core launch (exl3b200_gemm_combine); 300 rows =
    two 256-row tiles, output rows repeated (they add up), with and without scales."""
    rng = np.random.default_rng(120 + K)
    M, k, n, T = 300, 256, 384, 40
    tr, su, sv = _lin(rng, k, n, K)
    x = rng.standard_normal((M, k)).astype(np.float16)
    a = O.input_transform(x, su) if rotated else x
    ref = O.gemv_ref(x, tr, su, sv, K, cb)
    tok = rng.integers(0, T, size=M).astype(np.int32)
    for scaled in (True, False):
        rw = rng.uniform(0.1, 1.0, size=M).astype(np.float32)
        acc = torch.zeros((T, n), dtype=torch.float32, device=cuda_device)
        ops.matmul_combine(_t(a, cuda_device), _t(tr, cuda_device), None if rotated else _t(su, cuda_device),
                           _t(sv, cuda_device), K, cb, acc, _t(tok, cuda_device),
                           _t(rw, cuda_device) if scaled else None, input_rotated=rotated)
        exp = np.zeros((T, n), dtype=np.float64)
        for i in range(M):
            exp[tok[i]] += (float(rw[i]) if scaled else 1.0) * ref[i]
        assert O.normwise_rel_err(acc.cpu().numpy(), exp) < TOL
