"""Op surface: the drop-in module and the torch.ops registrations mirror the
reference's names and schemas (no GPU needed except where marked)."""

import inspect

import pytest
import torch

REFERENCE_OPS = ["dequant_trellis", "exl3_gemv", "exl3_gemm", "p2b_gemv_batched", "p2b_fused_moe",
                 "exl3_fat_gemm", "exl3_fat_gemm_scatter"]


def test_dropin_module_exports_reference_names():
    import sglang_exl3_c

    assert sglang_exl3_c.P2B_MOE_ABI_VERSION >= 2  # the reference's plugin refuses < 2 (exl3.py:892-894)
    for name in REFERENCE_OPS:
        assert callable(getattr(sglang_exl3_c, name)), name


def test_dropin_signatures_match_reference_binding():
    """Positional argument names of csrc/bindings.cpp:171-199."""
    import sglang_exl3_c as m

    expect = {
        "exl3_gemv": ["x", "trellis", "suh", "svh", "K", "mcg", "mmode"],
        "exl3_gemm": ["x", "trellis", "suh", "svh", "K", "mcg"],
        "p2b_gemv_batched": ["x", "trellis_ptrs", "suh_ptrs", "svh_ptrs", "expert_indices", "K", "mcg", "mmode"],
        "p2b_fused_moe": ["x", "out", "gate_trellis_ptrs", "gate_suh_ptrs", "gate_svh_ptrs", "up_trellis_ptrs",
                          "up_suh_ptrs", "up_svh_ptrs", "down_trellis_ptrs", "down_suh_ptrs", "down_svh_ptrs",
                          "expert_indices", "routing_weights", "K_gate", "K_up", "K_down", "mcg",
                          "intermediate_size", "swiglu_limit"],
        "exl3_fat_gemm": ["a", "packed", "out", "svh", "K", "mcg", "mul1"],
        "exl3_fat_gemm_scatter": ["a", "packed", "out", "svh", "token_idx", "route_weight", "K", "mcg", "mul1"],
    }
    for name, args in expect.items():
        params = list(inspect.signature(getattr(m, name)).parameters)
        assert params[:len(args)] == args, (name, params)
    assert inspect.signature(m.exl3_gemv).parameters["mmode"].default == 1
    assert inspect.signature(m.p2b_fused_moe).parameters["intermediate_size"].default == 2048


def test_torch_ops_registered_with_fake_kernels():
    from exl3_b200 import torch_ops

    assert torch_ops.register_custom_ops()
    assert torch_ops.register_custom_ops()  # idempotent
    for name in REFERENCE_OPS:
        assert hasattr(torch.ops.sglang_exl3, name), name
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty((3, 256), dtype=torch.float16)
        tr = torch.empty((16, 24, 64), dtype=torch.int16)
        su = torch.empty(256, dtype=torch.float16)
        sv = torch.empty(384, dtype=torch.float16)
        assert torch.ops.sglang_exl3.exl3_gemv(x, tr, su, sv, 4, True).shape == (3, 384)
        assert torch.ops.sglang_exl3.exl3_gemm(x, tr, su, sv, 4, True).shape == (3, 384)
        assert torch.ops.sglang_exl3.dequant_trellis(tr, su, sv, 4, True).shape == (256, 384)
        ptrs = torch.empty(8, dtype=torch.int64)
        ids = torch.empty(3, dtype=torch.int32)
        assert torch.ops.sglang_exl3.p2b_gemv_batched(x, ptrs, ptrs, ptrs, ids, 4, True, 384).shape == (3, 3, 384)


def test_codebook_mapping():
    from exl3_b200.ops import codebook_id, legacy_codebook

    assert codebook_id() == 0 and codebook_id(mcg=True) == 1 and codebook_id(mul1=True) == 2
    assert legacy_codebook(True) == 1 and legacy_codebook(False) == 2 and legacy_codebook(False, cb=0) == 0
    with pytest.raises(ValueError):
        codebook_id(mcg=True, mul1=True)
