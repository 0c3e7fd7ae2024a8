"""The workspace-free matmul entry point, called through the C ABI.

``exl3b200_gemv_noalloc`` exists for callers that cannot allocate device memory
(an allocator-less runtime that owns all device memory up front, or a thread that
must not enter the CUDA allocator): its scratch is a device array inside the
library.  This file is collected last so that a run stopping at the first failure
has already run every other test; it also passes on its own in a fresh process.
"""

import numpy as np
import pytest
import torch

import exl3_oracle as O
from exl3_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TOL = 2e-3  # the matmul tests' tolerance: normwise relative error, fp32 accumulate


_DTYPES = {0: torch.float16, 1: torch.bfloat16, 2: torch.float32}
TOL_BF16 = 4e-3  # bf16 outputs carry their own 2^-9 rounding


def _noalloc(L, x, tr, su, sv, K, cb, out, out_dtype=0):
    stream = torch.cuda.current_stream(x.device).cuda_stream
    return L.exl3b200_gemv_noalloc(x.data_ptr(), x.stride(0), x.size(0), x.size(1), tr.data_ptr(), tr.size(1) * 16,
                                   K, cb, su.data_ptr(), sv.data_ptr(), out.data_ptr(), out.stride(0), out_dtype,
                                   stream)


@pytest.mark.parametrize("K,cb,m,k,n,out_dtype", [(4, 0, 1, 4096, 4096, 0), (3, 1, 5, 1024, 768, 1),
                                                  (2, 2, 16, 512, 384, 2)])
def test_noalloc_matches_workspace_entry_twice(cuda_device, K, cb, m, k, n, out_dtype):
    """Two calls in a row: each agrees with the workspace entry point and with the
    oracle (fp32 matmul on the dequantised weights)."""
    L = _lib.lib()
    rng = np.random.default_rng(500 + K)
    tr_np, su_np, sv_np = O.random_trellis(rng, k, n, K), O.random_signs(rng, k), O.random_signs(rng, n)
    tr, su, sv = (torch.from_numpy(a).to(cuda_device) for a in (tr_np, su_np, sv_np))
    dtype = _DTYPES[out_dtype]
    tol = TOL_BF16 if dtype == torch.bfloat16 else TOL
    for call in range(2):  # the second call reuses the array the first one left behind
        x_np = rng.standard_normal((m, k)).astype(np.float16)
        x = torch.from_numpy(x_np).to(cuda_device)
        out = torch.empty((m, n), dtype=dtype, device=cuda_device)
        assert _noalloc(L, x, tr, su, sv, K, cb, out, out_dtype) == 0
        ref = ops.matmul(x, tr, su, sv, K, cb, out_dtype=dtype)
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert O.normwise_rel_err(got, ref.float().cpu().numpy()) < tol, call
        assert O.normwise_rel_err(got, O.gemv_ref(x_np, tr_np, su_np, sv_np, K, cb)) < tol, call


def test_noalloc_limits(cuda_device):
    L = _lib.lib()
    s_k = torch.ones(32768 + 128, dtype=torch.float16, device=cuda_device)
    tr_big_k = torch.zeros(((32768 + 128) // 16, 8, 64), dtype=torch.int16, device=cuda_device)
    x = torch.zeros((1, 32768 + 128), dtype=torch.float16, device=cuda_device)
    out = torch.empty((1, 128), dtype=torch.float16, device=cuda_device)
    assert _noalloc(L, x, tr_big_k, s_k, s_k[:128], 4, 0, out) == 1  # k beyond the limit: EXL3B200_EBADSHAPE
    tr = torch.zeros((8, 8, 64), dtype=torch.int16, device=cuda_device)
    s = torch.ones(128, dtype=torch.float16, device=cuda_device)
    x17 = torch.zeros((17, 128), dtype=torch.float16, device=cuda_device)
    out17 = torch.empty((17, 128), dtype=torch.float16, device=cuda_device)
    assert _noalloc(L, x17, tr, s, s, 4, 0, out17) == 1  # m beyond 16
