"""GPU dequant (trellis -> fp16 W) against the oracle: bit-exact, both codebook roundings."""

import os

import numpy as np
import pytest
import torch

import exl3_oracle as O
from exl3_b200 import ops

pytestmark = pytest.mark.gpu


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("K", list(range(1, 9)))
@pytest.mark.parametrize("cb", [0, 1, 2])
@pytest.mark.parametrize("rounding", ["rn", "trunc"])
def test_dequant_bit_exact(cuda_device, K, cb, rounding):
    rng = np.random.default_rng(100 * K + 10 * cb + (rounding == "rn"))
    tr = O.random_trellis(rng, 256, 384, K)
    su = O.random_signs(rng, 256)
    sv = O.random_signs(rng, 384)
    got = ops.dequant(_t(tr, cuda_device), _t(su, cuda_device), _t(sv, cuda_device), K, cb, rounding)
    ref = O.dequant(tr, su, sv, K, cb, rounding)
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("K", [2, 3, 4, 8])
@pytest.mark.parametrize("cb", [1, 2])
def test_dequant_trellis_op_matches_reference_fixture(cuda_device, golden_dir, K, cb):
    """The reference-named op reproduces the reference's own dequant_trellis output."""
    path = os.path.join(golden_dir, "ref_dequant_trunc.npz")
    f = np.load(path)
    tag = f"{K}_{cb}"
    got = ops.dequant_trellis(_t(f[f"trellis_{tag}"], cuda_device), _t(f[f"suh_{tag}"], cuda_device),
                              _t(f[f"svh_{tag}"], cuda_device), K, cb == 1)
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint16), f[f"out_{tag}"])


def test_dequant_c1_shape_bit_exact(cuda_device):
    """Config 1 shape: 4096 x 4096, 4 bpw, 3INST, seed 0."""
    rng = np.random.default_rng(0)
    tr = O.random_trellis(rng, 4096, 4096, 4)
    su = O.random_signs(rng, 4096)
    sv = O.random_signs(rng, 4096)
    got = ops.dequant(_t(tr, cuda_device), _t(su, cuda_device), _t(sv, cuda_device), 4, 0, "rn")
    ref = O.dequant(tr, su, sv, 4, 0, "rn")
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint16), ref.view(np.uint16))


def test_dequant_rejects_bad_input(cuda_device):
    tr = torch.zeros((8, 8, 64), dtype=torch.int16, device=cuda_device)
    s = torch.ones(128, dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError):
        ops.dequant(tr, s, s, 5)  # last dim != 16*K
    with pytest.raises(RuntimeError):
        ops.dequant(tr[:7], s, s, 4)  # not whole Hadamard blocks
    with pytest.raises(RuntimeError):
        ops.dequant(tr.cpu(), s.cpu(), s.cpu(), 4)  # no CPU path
