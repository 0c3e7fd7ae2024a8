"""Parity at the full shapes of the benchmark configs.

The NumPy oracle is too slow for matrices of 8192 x 28672, so the reference here is
the one the matmul contract names: an fp32 matmul on the round-to-nearest
dequantised weights, computed on the GPU.  The weights come from the library's
``exl3b200_dequant`` (bit-exact with the oracle at every K and codebook, see
``test_dequant_gpu.py``; at full shape it is spot-checked here against the oracle
on random 128 x 128 blocks, each of which depends only on its own 8 x 8 tiles and
its slices of suh / svh), and the matmul runs in fp32 with TF32 disabled.

Tolerances (normwise: max|y - y_ref| / max|y_ref|):
* a single matmul, fp32 accumulate: 2e-3;
* a block with an fp16 intermediate (SwiGLU activation, routed MoE): 4e-3.

Shapes: config 2's fused gate+up (5120 -> 2 x 25600, 3 bpw 3INST) and down
(25600 -> 5120, 4 bpw MCG) at M in {1, 4, 16, 64, 256, 2048}, and the whole block
through the fused MLP entry point; config 4's q/k/v
group, o, gate+up and down at TP 1 and at the TP-8 shard widths, M in {1, 8, 64};
config 3's 288-expert layer (hidden 2048, intermediate 1024, 3 bpw) plus its 4-bpw
shared expert at T in {1, 8, 64, 512}; config 5's MoE layer (128 experts, hidden
4096, intermediate 1536) at 1, 16 and 64 sequences x 5 rows; both MoE pipelines.
Random codes decode to weights of order 1, so the output scales of gate/up are
multiplied by 1/sqrt(k) to keep the fp16 SwiGLU intermediate finite.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import exl3_oracle as O
from exl3_b200 import moe, ops

pytestmark = pytest.mark.gpu

TOL = 2e-3
TOL_BLOCK = 4e-3


@pytest.fixture(autouse=True)
def _fp32_matmul():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


def _gen(seed, dev):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return g


def _signs(g, shape, dev):
    return ((torch.randint(0, 2, shape, device=dev, generator=g) * 2 - 1).half()
            * (torch.rand(shape, device=dev, generator=g) + 0.5).half())


def _linear(g, k, n, K, dev, out_scale=1.0):
    tr = torch.randint(-32768, 32768, (k // 16, n // 16, 16 * K), dtype=torch.int16, device=dev, generator=g)
    su = _signs(g, (k,), dev)
    sv = _signs(g, (n,), dev)
    if out_scale != 1.0:
        sv = (sv.float() * out_scale).half()
    return tr, su, sv


def _w32(lin, K, cb):
    return ops.dequant(*lin, K, cb, "rn").float()


def _rel(got, ref):
    got = got.double()
    ref = ref.double()
    return float((got - ref).abs().max() / ref.abs().max())


def _check_blocks(lin, K, cb, w16, rng, blocks=3):
    """Random 128 x 128 blocks of the GPU dequant equal the oracle's, bit for bit."""
    tr, su, sv = lin
    kb, nb = tr.size(0) // 8, tr.size(1) // 8
    for _ in range(blocks):
        i, j = int(rng.integers(kb)), int(rng.integers(nb))
        sub = tr[8 * i:8 * i + 8, 8 * j:8 * j + 8].cpu().numpy()
        ref = O.dequant(sub, su[128 * i:128 * i + 128].cpu().numpy(), sv[128 * j:128 * j + 128].cpu().numpy(),
                        K, cb, "rn")
        got = w16[128 * i:128 * i + 128, 128 * j:128 * j + 128].cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint16), ref.view(np.uint16))


# ---------------------------------------------------------------------------
# config 2: dense SwiGLU MLP block, hidden 5120, intermediate 25600
# ---------------------------------------------------------------------------

@pytest.fixture(scope="module")
def c2(cuda_device):
    g = _gen(1, cuda_device)
    H, I = 5120, 25600
    gu = _linear(g, H, 2 * I, 3, cuda_device, out_scale=H ** -0.5)   # [gate | up], 3 bpw 3INST
    down = _linear(g, I, H, 4, cuda_device)                          # 4 bpw MCG
    w_gu16 = ops.dequant(*gu, 3, 0, "rn")
    w_d16 = ops.dequant(*down, 4, 1, "rn")
    rng = np.random.default_rng(1)
    _check_blocks(gu, 3, 0, w_gu16, rng)
    _check_blocks(down, 4, 1, w_d16, rng)
    yield {"gu": gu, "down": down, "w_gu": w_gu16.float(), "w_d": w_d16.float(), "H": H, "I": I}


@pytest.mark.parametrize("m", [1, 4, 16, 64, 256, 2048])
def test_c2_mlp_block(cuda_device, c2, m):
    H, I = c2["H"], c2["I"]
    x = torch.randn(m, H, dtype=torch.float16, device=cuda_device, generator=_gen(100 + m, cuda_device))
    y_gu = ops.matmul(x, *c2["gu"], 3, 0)
    ref_gu = x.float() @ c2["w_gu"]
    assert _rel(y_gu, ref_gu) < TOL
    act = torch.mul(F.silu(y_gu[:, :I]), y_gu[:, I:])
    y = ops.matmul(act, *c2["down"], 4, 1)
    assert _rel(y, act.float() @ c2["w_d"]) < TOL
    # the whole block against fp32 throughout (fp16 intermediate on the product side only)
    ref_act = F.silu(ref_gu[:, :I]) * ref_gu[:, I:]
    assert _rel(y, ref_act @ c2["w_d"]) < TOL_BLOCK


@pytest.mark.parametrize("m", [1, 16, 17, 64, 2048])
def test_c2_fused_mlp(cuda_device, c2, m):
    """The whole block in one call (exl3b200_mlp), SwiGLU in the gate|up epilogue."""
    H, I = c2["H"], c2["I"]
    x = torch.randn(m, H, dtype=torch.float16, device=cuda_device, generator=_gen(150 + m, cuda_device))
    y = ops.mlp(x, c2["gu"], c2["down"], 3, 0, 4, 1)
    g = x.float() @ c2["w_gu"]
    act = (F.silu(g[:, :I]) * g[:, I:]).half().float()
    assert torch.isfinite(y).all()
    assert _rel(y, act @ c2["w_d"]) < TOL_BLOCK


# ---------------------------------------------------------------------------
# config 4: Llama-70B shapes, 4 bpw 3INST, TP 1 and the TP-8 shards
# ---------------------------------------------------------------------------

def _c4_dims(tp):
    H, hd = 8192, 128
    return H, 64 * hd // tp, 8 * hd // tp, 28672 // tp


@pytest.mark.parametrize("tp", [1, 8])
@pytest.mark.parametrize("m", [1, 8, 64])
def test_c4_attention_projections(cuda_device, tp, m):
    H, q_out, kv_out, _ = _c4_dims(tp)
    g = _gen(3 + tp, cuda_device)
    qkv = [_linear(g, H, q_out, 4, cuda_device), _linear(g, H, kv_out, 4, cuda_device),
           _linear(g, H, kv_out, 4, cuda_device)]
    o = _linear(g, q_out, H, 4, cuda_device)
    x = torch.randn(m, H, dtype=torch.float16, device=cuda_device, generator=g)
    fused = torch.empty(m, q_out + 2 * kv_out, dtype=torch.float16, device=cuda_device)
    outs = [fused[:, :q_out], fused[:, q_out:q_out + kv_out], fused[:, q_out + kv_out:]]
    ops.matmul_multi(x, qkv, 4, 0, outs=outs)
    for lin, out in zip(qkv, outs):
        assert _rel(out, x.float() @ _w32(lin, 4, 0)) < TOL
    a = torch.randn(m, q_out, dtype=torch.float16, device=cuda_device, generator=g)
    w_o = _w32(o, 4, 0)
    for dtype in (torch.float16, torch.float32):
        y = ops.matmul(a, *o, 4, 0, out_dtype=dtype)
        assert y.dtype == dtype and _rel(y, a.float() @ w_o) < TOL


@pytest.mark.parametrize("tp", [1, 8])
@pytest.mark.parametrize("m", [1, 8, 64])
def test_c4_mlp_projections(cuda_device, tp, m):
    H, _, _, i_loc = _c4_dims(tp)
    g = _gen(30 + tp, cuda_device)
    gate = _linear(g, H, i_loc, 4, cuda_device)
    up = _linear(g, H, i_loc, 4, cuda_device)
    x = torch.randn(m, H, dtype=torch.float16, device=cuda_device, generator=g)
    outs = [torch.empty(m, i_loc, dtype=torch.float16, device=cuda_device) for _ in range(2)]
    ops.matmul_multi(x, [gate, up], 4, 0, outs=outs)
    for lin, out in zip((gate, up), outs):
        w = _w32(lin, 4, 0)
        assert _rel(out, x.float() @ w) < TOL
        del w
    down = _linear(g, i_loc, H, 4, cuda_device)
    a = torch.randn(m, i_loc, dtype=torch.float16, device=cuda_device, generator=g)
    assert _rel(ops.matmul(a, *down, 4, 0), a.float() @ _w32(down, 4, 0)) < TOL


def test_c4_dequant_full_shape_blocks(cuda_device):
    """The reference weights themselves: the GPU dequant of a full 8192 x 28672
    projection equals the oracle on random blocks."""
    g = _gen(33, cuda_device)
    lin = _linear(g, 8192, 28672, 4, cuda_device)
    _check_blocks(lin, 4, 0, ops.dequant(*lin, 4, 0, "rn"), np.random.default_rng(33), blocks=6)


# ---------------------------------------------------------------------------
# configs 3 and 5: routed MoE layers
# ---------------------------------------------------------------------------

def _moe_layer(seed, E, H, I, K, dev):
    g = _gen(seed, dev)
    w13 = torch.randint(-32768, 32768, (E, 2, H // 16, I // 16, 16 * K), dtype=torch.int16, device=dev, generator=g)
    w2 = torch.randint(-32768, 32768, (E, I // 16, H // 16, 16 * K), dtype=torch.int16, device=dev, generator=g)
    s13u, s13v, s2u, s2v = _signs(g, (E, 2, H), dev), _signs(g, (E, 2, I), dev), _signs(g, (E, I), dev), \
        _signs(g, (E, H), dev)
    s13v = (s13v.float() * H ** -0.5).half()

    def ptrs(t):
        return torch.tensor([int(t[e].data_ptr()) for e in range(E)], dtype=torch.int64, device=dev)

    tables = {"gate_trellis": ptrs(w13[:, 0]), "gate_suh": ptrs(s13u[:, 0]), "gate_svh": ptrs(s13v[:, 0]),
              "up_trellis": ptrs(w13[:, 1]), "up_suh": ptrs(s13u[:, 1]), "up_svh": ptrs(s13v[:, 1]),
              "down_trellis": ptrs(w2), "down_suh": ptrs(s2u), "down_svh": ptrs(s2v)}
    # fp16 dequantised experts (the reference's weights)
    wg = torch.stack([ops.dequant(w13[e, 0], s13u[e, 0], s13v[e, 0], K, 0, "rn") for e in range(E)])
    wu = torch.stack([ops.dequant(w13[e, 1], s13u[e, 1], s13v[e, 1], K, 0, "rn") for e in range(E)])
    wd = torch.stack([ops.dequant(w2[e], s2u[e], s2v[e], K, 0, "rn") for e in range(E)])
    keep = (w13, w2, s13u, s13v, s2u, s2v)
    return {"tables": tables, "wg": wg, "wu": wu, "wd": wd, "keep": keep, "E": E, "H": H, "I": I, "K": K}


def _moe_ref(x16, ids, w, layer):
    """fp32 routed SwiGLU MoE on the dequantised experts, the activation rounded to
    fp16 where the reference keeps it (p2b_moe.cu phase 3, exl3.py:1207-1215)."""
    out = torch.zeros(x16.size(0), layer["H"], dtype=torch.float32, device=x16.device)
    for e in torch.unique(ids).tolist():
        if e < 0 or e >= layer["E"]:
            continue
        ts, js = (ids == e).nonzero(as_tuple=True)
        xt = x16[ts].float()
        g = xt @ layer["wg"][e].float()
        u = xt @ layer["wu"][e].float()
        a = (F.silu(g) * u).half().float()
        out.index_add_(0, ts, w[ts, js, None].float() * (a @ layer["wd"][e].float()))
    return out


def _route(T, E, topk, dev, seed):
    g = _gen(seed, dev)
    logits = torch.randn(T, E, dtype=torch.float32, device=dev, generator=g)
    p = torch.softmax(logits, dim=-1)
    w, ids = torch.topk(p, topk, dim=-1)
    return ids.to(torch.int32), (w / w.sum(-1, keepdim=True)).float()


@pytest.fixture(scope="module")
def c3(cuda_device):
    layer = _moe_layer(2, 288, 2048, 1024, 3, cuda_device)
    g = _gen(20, cuda_device)
    H, I = 2048, 1024
    shared = [_linear(g, H, I, 4, cuda_device, out_scale=H ** -0.5), _linear(g, H, I, 4, cuda_device,
                                                                              out_scale=H ** -0.5),
              _linear(g, I, H, 4, cuda_device)]
    stables = {}
    for which, lin in zip(("gate", "up", "down"), shared):
        for name, t in zip(("trellis", "suh", "svh"), lin):
            stables[f"{which}_{name}"] = torch.tensor([t.data_ptr()], dtype=torch.int64, device=cuda_device)
    sref = {"wg": _w32(shared[0], 4, 0)[None], "wu": _w32(shared[1], 4, 0)[None], "wd": _w32(shared[2], 4, 0)[None],
            "E": 1, "H": H, "I": I}
    yield layer, shared, stables, sref


@pytest.mark.parametrize("path", ["small", "tc"])
@pytest.mark.parametrize("T", [1, 8, 64, 512])
def test_c3_moe_layer(cuda_device, c3, T, path):
    layer, shared, stables, sref = c3
    H, I, K = layer["H"], layer["I"], layer["K"]
    x = torch.randn(T, H, dtype=torch.float16, device=cuda_device, generator=_gen(200 + T, cuda_device))
    ids, w = _route(T, layer["E"], 8, cuda_device, 300 + T)
    y = moe.moe_forward(x, ids, w, layer["tables"], K, K, K, 0, I, path=path)
    ref = _moe_ref(x, ids, w, layer)
    assert torch.isfinite(y).all()
    assert _rel(y, ref) < TOL_BLOCK
    # the shared expert added into the same output (accumulate), as the config-3 layer does
    ones = torch.ones((T, 1), dtype=torch.float32, device=cuda_device)
    zeros = torch.zeros((T, 1), dtype=torch.int32, device=cuda_device)
    moe.moe_forward(x, zeros, ones, stables, 4, 4, 4, 0, I, out=y, accumulate=True, path=path)
    ref = ref + _moe_ref(x, zeros, ones, sref)
    assert _rel(y, ref) < TOL_BLOCK


@pytest.fixture(scope="module")
def c5(cuda_device):
    yield _moe_layer(4, 128, 4096, 1536, 3, cuda_device)


@pytest.mark.parametrize("path", ["small", "tc"])
@pytest.mark.parametrize("batch", [1, 16, 64])
def test_c5_moe_layer(cuda_device, c5, batch, path):
    T = 5 * batch
    H, I, K = c5["H"], c5["I"], c5["K"]
    x = torch.randn(T, H, dtype=torch.float16, device=cuda_device, generator=_gen(400 + batch, cuda_device))
    ids, w = _route(T, c5["E"], 8, cuda_device, 500 + batch)
    y = moe.moe_forward(x, ids, w, c5["tables"], K, K, K, 0, I, path=path)
    assert torch.isfinite(y).all()
    assert _rel(y, _moe_ref(x, ids, w, c5)) < TOL_BLOCK
