"""Small-M EXL3 matmul on the GPU against the oracle.

Tolerance: the kernel accumulates in fp32, so by the target's contract the output
must be within max relative error 2e-3 of an fp32 matmul on the round-to-nearest
dequantised weights.  "Relative" is normwise: max|y - y_ref| / max|y_ref|.
bf16 outputs carry their own 2^-9 rounding, so they are held to 4e-3.
"""

import numpy as np
import pytest
import torch

import exl3_oracle as O
from exl3_b200 import ops

pytestmark = pytest.mark.gpu

TOL_F32_ACC = 2e-3
TOL_BF16_OUT = 4e-3


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _case(seed, m, k, n, K):
    rng = np.random.default_rng(seed)
    tr = O.random_trellis(rng, k, n, K)
    su = O.random_signs(rng, k)
    sv = O.random_signs(rng, n)
    x = rng.standard_normal((m, k)).astype(np.float16)
    return x, tr, su, sv


def test_hadamard_in_bit_exact(cuda_device):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((7, 1024)) * 3).astype(np.float16)
    su = O.random_signs(rng, 1024)
    got = ops.hadamard_in(_t(x, cuda_device), _t(su, cuda_device)).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint16), O.input_transform(x, su).view(np.uint16))


@pytest.mark.parametrize("K", [2, 3, 4])
@pytest.mark.parametrize("cb", [0, 1, 2])
@pytest.mark.parametrize("m", [1, 3, 8, 13, 16])
def test_gemv_parity(cuda_device, K, cb, m):
    x, tr, su, sv = _case(1000 * K + 10 * cb + m, m, 512, 384, K)
    y = ops.matmul(_t(x, cuda_device), _t(tr, cuda_device), _t(su, cuda_device), _t(sv, cuda_device), K, cb)
    ref = O.gemv_ref(x, tr, su, sv, K, cb)
    assert y.shape == (m, 384) and y.dtype == torch.float16
    assert O.normwise_rel_err(y.float().cpu().numpy(), ref) < TOL_F32_ACC


def test_gemv_c1_shape(cuda_device):
    """Config 1: K = N = 4096, 4 bpw, 3INST, seed 0, x ~ N(0, 1) [1, 4096]."""
    x, tr, su, sv = _case(0, 1, 4096, 4096, 4)
    y = ops.matmul(_t(x, cuda_device), _t(tr, cuda_device), _t(su, cuda_device), _t(sv, cuda_device), 4, 0)
    assert O.normwise_rel_err(y.float().cpu().numpy(), O.gemv_ref(x, tr, su, sv, 4, 0)) < TOL_F32_ACC


@pytest.mark.parametrize("dtype,tol", [(torch.float32, TOL_F32_ACC), (torch.bfloat16, TOL_BF16_OUT)])
def test_gemv_out_dtypes(cuda_device, dtype, tol):
    x, tr, su, sv = _case(11, 4, 384, 256, 3)
    y = ops.matmul(_t(x, cuda_device), _t(tr, cuda_device), _t(su, cuda_device), _t(sv, cuda_device), 3, 1,
                   out_dtype=dtype)
    assert y.dtype == dtype
    assert O.normwise_rel_err(y.float().cpu().numpy(), O.gemv_ref(x, tr, su, sv, 3, 1)) < tol


def test_gemv_strided_output_slice(cuda_device):
    """Write into a column slice of a wider output (fused qkv style)."""
    x, tr, su, sv = _case(12, 2, 256, 128, 4)
    wide = torch.full((2, 512), 7.0, dtype=torch.float16, device=cuda_device)
    ops.matmul(_t(x, cuda_device), _t(tr, cuda_device), _t(su, cuda_device), _t(sv, cuda_device), 4, 0,
               out=wide[:, 128:256])
    w = wide.float().cpu().numpy()
    assert np.all(w[:, :128] == 7.0) and np.all(w[:, 256:] == 7.0)
    assert O.normwise_rel_err(w[:, 128:256], O.gemv_ref(x, tr, su, sv, 4, 0)) < TOL_F32_ACC


def test_gemv_rows_above_16_are_chunked(cuda_device):
    x, tr, su, sv = _case(13, 37, 256, 256, 2)
    y = ops.matmul(_t(x, cuda_device), _t(tr, cuda_device), _t(su, cuda_device), _t(sv, cuda_device), 2, 0,
                   path="gemv")
    assert O.normwise_rel_err(y.float().cpu().numpy(), O.gemv_ref(x, tr, su, sv, 2, 0)) < TOL_F32_ACC


def test_gemv_state_reused_across_shapes(cuda_device):
    """The split-K state is left zeroed: alternate shapes on one stream."""
    cases = [_case(20, 1, 4096, 1024, 4), _case(21, 9, 1024, 4096, 3), _case(22, 2, 256, 128, 2)]
    refs = [O.gemv_ref(x, tr, su, sv, tr.shape[-1] // 16, 0) for x, tr, su, sv in cases]
    dev_cases = [[_t(a, cuda_device) for a in c] for c in cases]
    for _ in range(3):
        for (x, tr, su, sv), ref in zip(dev_cases, refs):
            y = ops.matmul(x, tr, su, sv, tr.shape[-1] // 16, 0)
            assert O.normwise_rel_err(y.float().cpu().numpy(), ref) < TOL_F32_ACC


def test_gemv_input_rotated_flag(cuda_device):
    x, tr, su, sv = _case(14, 3, 512, 256, 4)
    xh = O.input_transform(x, su)
    y = ops.matmul(_t(xh, cuda_device), _t(tr, cuda_device), None, _t(sv, cuda_device), 4, 0, input_rotated=True)
    assert O.normwise_rel_err(y.float().cpu().numpy(), O.gemv_ref(x, tr, su, sv, 4, 0)) < TOL_F32_ACC


def test_gemv_cuda_graph_replay(cuda_device):
    x, tr, su, sv = _case(15, 1, 1024, 512, 4)
    xd, trd, sud, svd = (_t(a, cuda_device) for a in (x, tr, su, sv))
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):
        for _ in range(3):
            ops.matmul(xd, trd, sud, svd, 4, 0)
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        y = ops.matmul(xd, trd, sud, svd, 4, 0)
    ref = O.gemv_ref(x, tr, su, sv, 4, 0)
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert O.normwise_rel_err(y.float().cpu().numpy(), ref) < TOL_F32_ACC
    x2 = np.random.default_rng(99).standard_normal((1, 1024)).astype(np.float16)
    xd.copy_(_t(x2, cuda_device))
    g.replay()
    torch.cuda.synchronize()
    assert O.normwise_rel_err(y.float().cpu().numpy(), O.gemv_ref(x2, tr, su, sv, 4, 0)) < TOL_F32_ACC


def test_reference_named_ops(cuda_device):
    x, tr, su, sv = _case(16, 4, 256, 256, 3)
    args = [_t(a, cuda_device) for a in (x, tr, su, sv)]
    y = ops.exl3_gemv(*args, 3, True)
    assert O.normwise_rel_err(y.float().cpu().numpy(), O.gemv_ref(x, tr, su, sv, 3, 1)) < TOL_F32_ACC
    y = ops.exl3_gemm(*args, 3, False)
    assert O.normwise_rel_err(y.float().cpu().numpy(), O.gemv_ref(x, tr, su, sv, 3, 2)) < TOL_F32_ACC
    with pytest.raises(RuntimeError):
        ops.exl3_gemv(_t(np.zeros((17, 256), np.float16), cuda_device), *args[1:], 3, True)


def test_gemv_rejects_bad_input(cuda_device):
    x, tr, su, sv = _case(17, 1, 256, 256, 4)
    xd, trd, sud, svd = (_t(a, cuda_device) for a in (x, tr, su, sv))
    with pytest.raises(RuntimeError):
        ops.matmul(xd.float(), trd, sud, svd, 4, 0)
    with pytest.raises(RuntimeError):
        ops.matmul(xd[:, :128], trd, sud, svd, 4, 0)
    with pytest.raises(RuntimeError):
        ops.matmul(xd, trd, sud, svd, 3, 0)
