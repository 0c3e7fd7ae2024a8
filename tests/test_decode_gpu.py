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
seventeen 64-position chunks (the chunk merge of the attention kernel).  The fused
model runs whole layers with the RMSNorm folded into the residual epilogues by
default; the two sub-layer calls with input stages are checked as well, and the
fold against them.
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


def _pair(cfg, batch, max_ctx, ctx, dev, tokens, fold=True):
    ms = []
    for fused in (False, True):
        m = _tame(DecodeModel(cfg, batch=batch, max_ctx=max_ctx, device=dev, fused=fused, fold=fold))
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


@pytest.mark.parametrize("fold", [False])
@pytest.mark.parametrize("heads,kv_heads,batch,ctx,max_ctx", [(16, 2, 3, 70, 160), (8, 1, 1, 127, 160)])
def test_sub_layer_calls_match_unfused(cuda_device, heads, kv_heads, batch, ctx, max_ctx, fold):
    """The two sub-layer calls per layer (input stages as kernels) against the unfused step."""
    cfg = DecoderConfig(layers=2, hidden=512, heads=heads, kv_heads=kv_heads, head_dim=128, inter=1024, vocab=1024,
                        K=4, cb=0)
    tokens = torch.arange(batch, device=cuda_device) * 5 + 1
    ref, fus = _pair(cfg, batch, max_ctx, ctx, cuda_device, tokens, fold=fold)
    assert not fus.fold
    for step in range(2):
        ref.step()
        fus.step()
        torch.cuda.synchronize()
        assert _rel(fus.h, ref.h) < TOL_H, step
        assert _rel(fus.last_logits, ref.last_logits) < TOL_H, step


@pytest.mark.parametrize("K,cb,batch,layers", [(4, 0, 1, 3), (3, 1, 3, 2), (2, 2, 2, 2), (4, 0, 16, 2)])
def test_norm_fold_matches_sub_layer_calls(cuda_device, K, cb, batch, layers):
    """decode_layer (the RMSNorm folded into the residual epilogues: inputs pre-scaled by
    the row's old norm factor / 16, outputs of the consuming RoPE / SwiGLU epilogues
    scaled by the exact factor) against the two sub-layer calls with their input
    stages: the same linear maps with the fp16 rounding at other points.  Also the
    per-row sum of squares the layer leaves in ss[0], and the appended KV rows."""
    cfg = DecoderConfig(layers=layers, hidden=512, heads=8, kv_heads=2, head_dim=128, inter=1024, vocab=512, K=K,
                        cb=cb)
    tokens = torch.arange(batch, device=cuda_device) * 3 + 2
    ms = []
    for fold in (False, True):
        m = _tame(DecodeModel(cfg, batch=batch, max_ctx=160, device=cuda_device, fused=True, fold=fold))
        m.fill_random_kv(70)
        m.tokens.copy_(tokens)
        ms.append(m)
    a, b = ms
    assert b.fold and not a.fold
    for step in range(2):
        pos = int(a.pos.item())
        a.step()
        b.step()
        torch.cuda.synchronize()
        assert _rel(b.h, a.h) < 5e-3, step
        assert _rel(b.last_logits, a.last_logits) < TOL_H, step  # bf16 logits: one ulp is 2^-8
        torch.testing.assert_close(b.ss[0], (b.h.double() ** 2).sum(-1).float(), rtol=1e-4, atol=0)
        for li in range(cfg.layers):
            assert _rel(b.k_cache[li][:, :, pos], a.k_cache[li][:, :, pos]) < TOL_KV
            assert _rel(b.v_cache[li][:, :, pos], a.v_cache[li][:, :, pos]) < TOL_KV
        b.tokens.copy_(a.tokens)  # same inputs next step even if a near-tie flipped a greedy token


def test_norm_fold_row_growth(cuda_device):
    """Rows whose norm grows ~1000-fold across one sub-layer (a small residual stream
    meeting a large sub-layer output): the pre-scale keeps the folded fp16 inputs finite."""
    cfg = DecoderConfig(layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, inter=1024, vocab=256, K=4, cb=0)
    ms = []
    for fold in (False, True):
        m = _tame(DecodeModel(cfg, batch=2, max_ctx=64, device=cuda_device, fused=True, fold=fold))
        m.layers[0]["o"][2].mul_(1000.0)  # the first attention output dwarfs the embedding
        m.fill_random_kv(10)
        m.tokens.copy_(torch.tensor([1, 2], device=cuda_device))
        ms.append(m)
    for m in ms:
        m.step()
    torch.cuda.synchronize()
    assert torch.isfinite(ms[1].h).all() and torch.isfinite(ms[1].last_logits).all()
    assert _rel(ms[1].h, ms[0].h) < 5e-3
    assert _rel(ms[1].last_logits, ms[0].last_logits) < TOL_H


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
    for fold in (True, False):
        m = _tame(DecodeModel(cfg, batch=2, max_ctx=96, device=cuda_device, fused=True, fold=fold))
        m.fill_random_kv(30)
        _replay_matches_eager(m, torch.tensor([4, 8], device=cuda_device), 30, 3)


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


def _replay_matches_eager(m, tokens0, pos0, steps):
    """Eager steps, then the captured graph from the same state.  Each replay is fed the
    eager step's input tokens.  The fused step is not bitwise repeatable: the order of
    the fp32 atomic sums (split-K partials, the rows' sums of squares) moves values by
    ulps, and where that flips the bf16 rounding of an appended K/V entry (2^-8) the
    attention output follows - two eager runs of this model differ by ~1e-3 of the
    residual stream.  So the residual stream must agree to 5e-3, the bf16 logits to
    1e-2, and a greedy token may differ only at a near-tie."""
    rel = lambda a, b: ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()  # noqa: E731
    kv0 = (m.k_cache.clone(), m.v_cache.clone())
    m.pos.fill_(pos0)
    m.tokens.copy_(tokens0)
    eager = []
    for _ in range(steps):
        tin = m.tokens.clone()
        m.step()
        eager.append((tin, m.h.clone(), m.last_logits.float().clone(), m.next_tokens.clone()))
    m.k_cache.copy_(kv0[0])
    m.v_cache.copy_(kv0[1])
    m.pos.fill_(pos0)
    m.tokens.copy_(tokens0)
    m.capture()
    m.pos.fill_(pos0)
    for tin, h, logits, tok in eager:
        m.tokens.copy_(tin)
        m.decode(1)
        torch.cuda.synchronize()
        assert rel(m.h, h) < 5e-3
        assert rel(m.last_logits, logits) < 1e-2
        top = logits.max(-1).values
        picked = logits.gather(-1, m.next_tokens.view(-1, 1)).squeeze(-1)
        assert bool(torch.all((m.next_tokens == tok) | (top - picked <= 2.0 ** -7 * top.abs())))
    m.release()
