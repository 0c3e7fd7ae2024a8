"""Fused decode sub-layers (exl3_b200.decode) against the unfused torch-glue step.

Both steps use the same EXL3 kernels for the matmuls; the fused one moves
RMSNorm, RoPE, the KV append, attention, SiLU*mul and the residual adds into the
matmul pipeline.  The unfused step rounds q to bf16, runs
scaled_dot_product_attention on bf16 and rounds its output to bf16; the fused one
keeps q and the softmax weights to ~16 bits (bf16 hi + lo pairs on the tensor
cores, fp32 sums) and the merged output in fp32, so the residual stream is held to a
relative error of 1e-2 (max abs difference over max abs value) and the KV
entries it appends to 2e-2 (bf16 rounding of slightly different fp32 values).
The shapes cover GQA groups of 1 to 16 query heads and contexts of one to
seventeen 64-position chunks (the chunk merge of the attention kernel).
"""

import pytest
import torch

from exl3_b200 import decode as D
from exl3_b200.harness import DecodeModel, DecoderConfig

pytestmark = pytest.mark.gpu

TOL_H = 1e-2
TOL_KV = 2e-2


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()


def _tame(m):
    """Scale every linear's output scales by 1/sqrt(k) so activations stay O(1)
    (random codes grow them by ~sqrt(k) per projection; fp16 would overflow)."""
    for L in m.layers:
        for lin in L["qkv"] + [L["o"]] + L["gu"] + [L["down"]]:
            lin[2].mul_(float(lin[0].size(0) * 16) ** -0.5)
    return m


def _pair(cfg, batch, max_ctx, ctx, dev, tokens):
    ms = []
    for fused in (False, True):
        m = _tame(DecodeModel(cfg, batch=batch, max_ctx=max_ctx, device=dev, fused=fused))
        m.fill_random_kv(ctx)
        m.tokens.copy_(tokens)
        ms.append(m)
    return ms


@pytest.mark.parametrize("heads,kv_heads,batch,ctx,max_ctx", [
    (4, 2, 1, 10, 160), (16, 2, 3, 70, 160), (8, 8, 2, 64, 160), (8, 1, 1, 127, 160),
    (16, 1, 1, 300, 320), (32, 4, 2, 1050, 1100), (8, 1, 1, 0, 64)])
def test_fused_step_matches_unfused(cuda_device, heads, kv_heads, batch, ctx, max_ctx):
    cfg = DecoderConfig(layers=2, hidden=512, heads=heads, kv_heads=kv_heads, head_dim=128, inter=1024, vocab=1024,
                        K=4, cb=0)
    tokens = torch.arange(batch, device=cuda_device) * 7 + 3
    ref, fus = _pair(cfg, batch, max_ctx, ctx, cuda_device, tokens)
    for step in range(2):
        pos = int(ref.pos.item())
        ref.step()
        fus.step()
        torch.cuda.synchronize()
        assert _rel(fus.h, ref.h) < TOL_H, step
        assert _rel(fus.last_logits, ref.last_logits) < TOL_H, step
        for li in range(cfg.layers):
            assert _rel(fus.k_cache[li][:, :, pos], ref.k_cache[li][:, :, pos]) < TOL_KV
            assert _rel(fus.v_cache[li][:, :, pos], ref.v_cache[li][:, :, pos]) < TOL_KV
        assert int(fus.pos.item()) == pos + 1


@pytest.mark.parametrize("cb", [1, 2])
def test_fused_step_codebooks(cuda_device, cb):
    cfg = DecoderConfig(layers=1, hidden=256, heads=2, kv_heads=1, head_dim=128, inter=512, vocab=256, K=3, cb=cb)
    ref, fus = _pair(cfg, 2, 64, 20, cuda_device, torch.tensor([1, 2], device=cuda_device))
    ref.step()
    fus.step()
    torch.cuda.synchronize()
    assert _rel(fus.h, ref.h) < TOL_H


def test_tensor_parallel_partial_path(cuda_device):
    """y-output + residual_add (the all-reduce path, here with one rank) equals the
    direct residual epilogue up to the summation order of the row sums of squares
    (atomics in a different kernel), which moves the next RMSNorm by ~1 fp16 ulp."""
    cfg = DecoderConfig(layers=1, hidden=512, heads=4, kv_heads=2, head_dim=128, inter=1024, vocab=256, K=4, cb=0)
    a = _tame(DecodeModel(cfg, batch=2, max_ctx=64, device=cuda_device, fused=True))
    a.fill_random_kv(12)
    h0 = torch.randn(2, 512, device=cuda_device)
    L = a.layers[0]
    outs = []
    for use_y in (False, True):
        a.fill_random_kv(12)
        h = h0.clone()
        ss = torch.zeros(2, 2, device=cuda_device)
        torch.sum(h * h, dim=-1, out=ss[0])
        y = torch.zeros_like(h) if use_y else None
        D.decode_attention(h, ss[0], ss[1], L["ln1"], cfg.eps, L["qkv"], L["o"], cfg.K, cfg.cb, a.k_cache[0],
                           a.v_cache[0], a.pos, a.inv_freq, y=y)
        if use_y:
            D.residual_add(h, y, ss[1])
        D.decode_mlp(h, ss[1], ss[0], L["ln2"], cfg.eps, L["gu"][0], L["gu"][1], L["down"], cfg.K, cfg.cb, y=y)
        if use_y:
            D.residual_add(h, y, ss[0])
        torch.cuda.synchronize()
        outs.append((h.clone(), ss[0].clone()))
    assert _rel(outs[1][0], outs[0][0]) < 2e-3
    torch.testing.assert_close(outs[0][1], outs[1][1], rtol=1e-3, atol=0)
    torch.testing.assert_close(outs[1][1], (outs[1][0] ** 2).sum(-1), rtol=1e-4, atol=0)


def test_fused_graph_replay(cuda_device):
    cfg = DecoderConfig(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, inter=1024, vocab=512, K=4, cb=0)
    m = _tame(DecodeModel(cfg, batch=2, max_ctx=96, device=cuda_device, fused=True))
    m.fill_random_kv(30)
    m.tokens.copy_(torch.tensor([4, 8], device=cuda_device))
    kv0 = (m.k_cache.clone(), m.v_cache.clone())
    eager = []
    for _ in range(3):
        m.step()
        eager.append(m.next_tokens.clone())
    m.k_cache.copy_(kv0[0])
    m.v_cache.copy_(kv0[1])
    m.pos.fill_(30)
    m.tokens.copy_(torch.tensor([4, 8], device=cuda_device))
    m.capture()
    m.pos.fill_(30)
    m.tokens.copy_(torch.tensor([4, 8], device=cuda_device))
    for i in range(3):
        m.decode(1)
        torch.cuda.synchronize()
        assert torch.equal(m.next_tokens, eager[i])
    m.release()


def test_decode_rejects_bad_state(cuda_device):
    cfg = DecoderConfig(layers=1, hidden=256, heads=2, kv_heads=1, head_dim=128, inter=512, vocab=256, K=4, cb=0)
    m = DecodeModel(cfg, batch=1, max_ctx=32, device=cuda_device, fused=True)
    L = m.layers[0]
    with pytest.raises(RuntimeError):
        D.decode_attention(m.h.half(), m.ss[0], m.ss[1], L["ln1"], cfg.eps, L["qkv"], L["o"], 4, 0, m.k_cache[0],
                           m.v_cache[0], m.pos, m.inv_freq)
    with pytest.raises(RuntimeError):
        D.decode_mlp(m.h, m.ss[0], m.ss[1], L["ln2"].float(), cfg.eps, L["gu"][0], L["gu"][1], L["down"], 4, 0)


def test_position_past_cache_sets_status(cuda_device):
    """A device-side position with no cache row (pos >= max_ctx) is not written:
    the sub-layer records EBADSHAPE in the sticky device status and the call
    returns without touching the cache."""
    from exl3_b200 import _lib, ops

    cfg = DecoderConfig(layers=1, hidden=256, heads=2, kv_heads=1, head_dim=128, inter=512, vocab=256, K=4, cb=0)
    m = DecodeModel(cfg, batch=1, max_ctx=64, device=cuda_device, fused=True)
    m.fill_random_kv(64)  # pos = 64 = max_ctx
    assert ops.device_status(cuda_device) == 0
    k0 = m.k_cache.clone()
    m.step()
    torch.cuda.synchronize()
    assert ops.device_status(cuda_device) == _lib.EBADSHAPE
    assert ops.device_status(cuda_device) == 0  # read-and-reset
    assert torch.equal(m.k_cache, k0)
