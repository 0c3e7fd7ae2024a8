"""The fused SwiGLU MLP block (exl3b200_mlp: activation in the gate|up epilogue) on
the GPU against the oracle.

Reference: the oracle's fp32 matmul on the dequantised fused gate|up weights, the
clipped SwiGLU rounded to fp16 where the reference keeps it, then the fp32 matmul on
the dequantised down weights.  The block carries an fp16 intermediate, so it is held
to normwise 4e-3 (as the routed MoE).  Row counts cover both kernel families (small-M
up to 16 rows, tensor cores from 17), tiles split between CTAs (300 rows) and the
CTA-pair tiles of 512 rows (600, 1030 rows).
"""

import numpy as np
import pytest
import torch

import exl3_oracle as O
from exl3_b200 import ops

pytestmark = pytest.mark.gpu

TOL_BLOCK = 4e-3


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _case(seed, m, H, I, Kg, Kd):
    rng = np.random.default_rng(seed)
    gu = (O.random_trellis(rng, H, 2 * I, Kg), O.random_signs(rng, H),
          (O.random_signs(rng, 2 * I).astype(np.float32) * H ** -0.5).astype(np.float16))
    dn = (O.random_trellis(rng, I, H, Kd), O.random_signs(rng, I), O.random_signs(rng, H))
    x = rng.standard_normal((m, H)).astype(np.float16)
    return x, gu, dn


def _ref(x, gu, dn, Kg, cbg, Kd, cbd, limit=0.0):
    y = O.gemv_ref(x, *gu, Kg, cbg)
    I = y.shape[1] // 2
    act = O.swiglu(y[:, :I], y[:, I:], limit).astype(np.float16)
    return O.gemv_ref(act, *dn, Kd, cbd)


@pytest.mark.parametrize("m", [1, 5, 16, 17, 40, 300, 600, 1030])
@pytest.mark.parametrize("Kg,cbg,Kd,cbd", [(3, 0, 4, 1), (4, 0, 4, 0), (2, 2, 3, 2)])
def test_mlp_parity(cuda_device, m, Kg, cbg, Kd, cbd):
    x, gu, dn = _case(7000 + m + 10 * Kg + cbg, m, 256, 384, Kg, Kd)
    dev = cuda_device
    y = ops.mlp(_t(x, dev), [_t(a, dev) for a in gu], [_t(a, dev) for a in dn], Kg, cbg, Kd, cbd)
    assert y.shape == (m, 256) and y.dtype == torch.float16
    assert torch.isfinite(y).all()
    assert O.normwise_rel_err(y.float().cpu().numpy(), _ref(x, gu, dn, Kg, cbg, Kd, cbd)) < TOL_BLOCK
    assert ops.device_status(dev) == 0


@pytest.mark.parametrize("m", [3, 64])
def test_mlp_clip_and_fp32_out(cuda_device, m):
    x, gu, dn = _case(7100 + m, m, 384, 256, 3, 4)
    x = (x.astype(np.float32) * 4).astype(np.float16)
    dev = cuda_device
    y = ops.mlp(_t(x, dev), [_t(a, dev) for a in gu], [_t(a, dev) for a in dn], 3, 0, 4, 1, swiglu_limit=1.5,
                out_dtype=torch.float32)
    assert y.dtype == torch.float32
    assert O.normwise_rel_err(y.cpu().numpy(), _ref(x, gu, dn, 3, 0, 4, 1, limit=1.5)) < TOL_BLOCK


@pytest.mark.parametrize("m", [2, 48])
def test_mlp_graph_replay(cuda_device, m):
    x, gu, dn = _case(7200 + m, m, 256, 256, 4, 4)
    dev = cuda_device
    xd = _t(x, dev)
    gud, dnd = [_t(a, dev) for a in gu], [_t(a, dev) for a in dn]
    out = torch.empty((m, 256), dtype=torch.float16, device=dev)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(2):
            ops.mlp(xd, gud, dnd, 4, 0, 4, 0, out=out)
    torch.cuda.current_stream(dev).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        ops.mlp(xd, gud, dnd, 4, 0, 4, 0, out=out)
    for trial in range(2):
        x2 = np.random.default_rng(trial).standard_normal((m, 256)).astype(np.float16)
        xd.copy_(_t(x2, dev))
        g.replay()
        torch.cuda.synchronize()
        assert O.normwise_rel_err(out.float().cpu().numpy(), _ref(x2, gu, dn, 4, 0, 4, 0)) < TOL_BLOCK
