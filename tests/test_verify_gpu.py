"""Config-5 speculative-verify harness on a scaled-down model: the captured CUDA graph
reproduces an eager step, the logits are finite, and the five new positions of every
sequence are appended to the cache (the step is idempotent: it rewrites them)."""

import dataclasses

import pytest
import torch
from torch.nn.attention import SDPBackend, sdpa_kernel

from exl3_b200.verify import CONFIG5, VerifyModel

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a - b).norm() / b.norm()).item()


@pytest.mark.parametrize("batch", [1, 7])  # 5 and 35 rows: small-M and tensor-core attention projections
def test_verify_graph_matches_eager(cuda_device, batch):
    cfg = dataclasses.replace(CONFIG5, layers=2, hidden=1024, heads=8, kv_heads=2, experts=16, inter=512,
                              vocab=2048)
    ctx = 64
    m = VerifyModel(cfg, batch, ctx + cfg.rows_per_seq, cuda_device)
    m.fill_random_kv(ctx)
    m.tokens.random_(0, cfg.vocab, generator=torch.Generator(device=cuda_device).manual_seed(1))
    with sdpa_kernel(SDPBackend.MATH):  # one attention backend for eager and capture
        with torch.cuda.stream(m.stream):
            eager = m.step().clone()
            eager2 = m.step().clone()
        torch.cuda.synchronize()
        assert eager.shape == (batch * cfg.rows_per_seq, cfg.vocab) and torch.isfinite(eager).all()
        assert m.k_cache[:, :, :, ctx:ctx + cfg.rows_per_seq].abs().sum() > 0  # new positions written
        m.capture()
        m.replay()
        torch.cuda.synchronize()
    noise, err = _rel(eager2, eager), _rel(m.logits, eager)
    print(f"eager vs eager {noise:.2e}, graph vs eager {err:.2e}")
    assert err < max(1e-3, 10 * noise), (err, noise)  # routed-MoE fp32 atomics may add in another order
    m.close()
