"""The plugin-surface mirror end to end on the GPU against the oracle."""

import numpy as np
import pytest
import torch

import exl3_oracle as O
from exl3_b200 import layers as L

pytestmark = pytest.mark.gpu


class _Layer(torch.nn.Module):
    pass


def test_linear_method_qkv(cuda_device):
    rng = np.random.default_rng(5)
    K, k_in, outs = 4, 512, [512, 128, 128]
    layer = _Layer()
    m = L.EXL3LinearMethod(bits=K)
    m.create_weights(layer, k_in, outs, k_in, sum(outs), torch.bfloat16)
    ref_parts = []
    x = rng.standard_normal((3, k_in)).astype(np.float16)
    for i, n in enumerate(outs):
        tr, su, sv = O.random_trellis(rng, k_in, n, K), O.random_signs(rng, k_in), O.random_signs(rng, n)
        for suffix, val in (("trellis", tr), ("suh", su), ("svh", sv)):
            m._load_linear(getattr(layer, f"exl3_{i}_{suffix}"), torch.from_numpy(val), i)
        ref_parts.append(O.gemv_ref(x, tr, su, sv, K, 0))
    m.process_weights_after_loading(layer)
    y = m.apply(layer, torch.from_numpy(x).to(cuda_device).to(torch.bfloat16))
    assert y.dtype == torch.bfloat16 and y.shape == (3, sum(outs))
    # bf16 input and output roundings on top of the matmul
    assert O.normwise_rel_err(y.float().cpu().numpy(), np.concatenate(ref_parts, 1)) < 1e-2
    k, v = m.apply_kv_only(layer, torch.from_numpy(x).to(cuda_device))
    assert O.normwise_rel_err(k.float().cpu().numpy(), ref_parts[1]) < 1e-2


def test_moe_method_apply(cuda_device):
    rng = np.random.default_rng(6)
    E, H, I, K, T, topk = 5, 256, 256, 3, 6, 2
    layer = _Layer()
    m = L.EXL3MoEMethod(bits=K)
    m.create_weights(layer, E, H, I, torch.float16)
    layer.to(cuda_device)
    experts = []
    for e in range(E):
        ex = {}
        for which, (a, b), shard in (("gate", (H, I), "w1"), ("up", (H, I), "w3"), ("down", (I, H), "w2")):
            tr, su, sv = O.random_trellis(rng, a, b, K), O.random_signs(rng, a), O.random_signs(rng, b)
            for suffix, val in (("trellis", tr), ("suh", su), ("svh", sv)):
                pname = ("w2_" if shard == "w2" else "w13_") + suffix
                m._load_exl3(getattr(layer, pname), torch.from_numpy(val).to(cuda_device),
                             f"experts.{e}.{which}.{suffix}", shard, e)
            m._load_exl3(getattr(layer, ("w2_" if shard == "w2" else "w13_") + "mcg"),
                         torch.tensor(L.MCG_MARKER_SIGNED_INT32), f"experts.{e}.{which}.mcg", shard, e)
            ex[which] = (tr, su, sv, K, 1)
        experts.append(ex)
    m.process_weights_after_loading(layer)
    assert layer._exl3_cb == 1
    x = rng.standard_normal((T, H)).astype(np.float16)
    ids = rng.integers(0, E, size=(T, topk))
    w = rng.uniform(0.1, 1.0, size=(T, topk)).astype(np.float32)
    y = m.apply(layer, torch.from_numpy(x).to(cuda_device), torch.from_numpy(w).to(cuda_device),
                torch.from_numpy(ids).to(cuda_device))
    assert y.dtype == torch.float16
    assert O.normwise_rel_err(y.float().cpu().numpy(), O.moe_ref(x, experts, ids, w)) < 4e-3
