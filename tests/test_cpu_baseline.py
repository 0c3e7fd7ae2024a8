"""The pure-torch CPU baseline port (oracle/torch_lut.py) computes the same matmul as
the oracle: fp32 x @ W within the normwise 2e-3 of the matmul contract (it differs
from the oracle's reference only by not rounding W to fp16)."""

import numpy as np
import pytest
import torch

import exl3_oracle as O
from torch_lut import TorchLutLinear


@pytest.mark.parametrize("K,cb", [(4, 0), (3, 1), (2, 2)])
def test_torch_lut_matches_oracle(K, cb):
    rng = np.random.default_rng(60 + K)
    k, n = 256, 384
    tr, su, sv = O.random_trellis(rng, k, n, K), O.random_signs(rng, k), O.random_signs(rng, n)
    x = rng.standard_normal((3, k)).astype(np.float16)
    lin = TorchLutLinear(torch.from_numpy(tr), torch.from_numpy(su), torch.from_numpy(sv), K, cb, chunk_cols=128)
    assert O.normwise_rel_err(lin(torch.from_numpy(x)).numpy(), O.gemv_ref(x, tr, su, sv, K, cb)) < 2e-3
