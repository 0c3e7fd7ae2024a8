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


def _torch_verify_step(m):
    """The same verify step in fp32 torch on the dequantised weights (no EXL3
    kernels): q/k/v, o and every expert as fp32 matmuls, the MoE as a loop over the
    routed experts with the SwiGLU activation rounded to fp16 where the kernels keep
    it.  Returns the logits and, per row, whether any layer's top-k choice was
    within 1e-3 of a tie (such rows may legitimately route differently)."""
    import torch.nn.functional as F
    from exl3_b200 import ops

    cfg = m.cfg
    B, S, R = m.batch, cfg.rows_per_seq, m.rows
    hd, nh, nkv = cfg.head_dim, cfg.heads, cfg.kv_heads
    qd, kvd = nh * hd, nkv * hd
    dev = m.device

    def W(lin, K):
        return ops.dequant(*lin, K, cfg.cb, "rn").float()

    positions = (m.pos + torch.arange(S, device=dev)).repeat(B)
    cols = torch.arange(m.max_ctx, device=dev)
    mask = cols[None, :] <= (m.pos + torch.arange(S, device=dev))[:, None]
    ang = positions.float()[:, None] * m.inv_freq[None, :]
    cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    k_cache, v_cache = m.k_cache.clone(), m.v_cache.clone()
    tie = torch.zeros(R, dtype=torch.bool, device=dev)
    h = m.embed[m.tokens.reshape(-1)].float()
    for li, L in enumerate(m.layers):
        xn = m._rms(h, L["ln1"]).float()
        q = m._rope((xn @ W(L["qkv"][0], cfg.K_attn)).view(R, nh, hd), cos, sin)
        k = m._rope((xn @ W(L["qkv"][1], cfg.K_attn)).view(R, nkv, hd), cos, sin)
        v = (xn @ W(L["qkv"][2], cfg.K_attn)).view(R, nkv, hd)
        idx = positions.view(B, S)[0]
        k_cache[li].index_copy_(2, idx, k.view(B, S, nkv, hd).transpose(1, 2).to(torch.bfloat16))
        v_cache[li].index_copy_(2, idx, v.view(B, S, nkv, hd).transpose(1, 2).to(torch.bfloat16))
        kk = k_cache[li].float().repeat_interleave(nh // nkv, dim=1)
        vv = v_cache[li].float().repeat_interleave(nh // nkv, dim=1)
        qh = q.view(B, S, nh, hd).transpose(1, 2)  # [B, nh, S, hd]
        att = F.scaled_dot_product_attention(qh, kk, vv, attn_mask=mask[None, None])
        att = att.transpose(1, 2).reshape(R, qd)
        h = h + att @ W(L["o"], cfg.K_attn)
        xn16 = m._rms(h, L["ln2"])
        logits = xn16.float() @ L["router"].t() + m.route_noise[li]
        p = torch.softmax(logits, dim=-1)
        top = torch.topk(p, cfg.topk + 1, dim=-1)
        tie |= (top.values[:, cfg.topk - 1] - top.values[:, cfg.topk]) < 1e-3
        w, ids = top.values[:, :cfg.topk], top.indices[:, :cfg.topk]
        w = w / w.sum(-1, keepdim=True)
        w13, w2, s13u, s13v, s2u, s2v = L["experts"]
        y = torch.zeros_like(h)
        for e in torch.unique(ids).tolist():
            ts, js = (ids == e).nonzero(as_tuple=True)
            xt = xn16[ts].float()
            g = xt @ ops.dequant(w13[e, 0], s13u[e, 0], s13v[e, 0], cfg.K_expert, cfg.cb, "rn").float()
            u = xt @ ops.dequant(w13[e, 1], s13u[e, 1], s13v[e, 1], cfg.K_expert, cfg.cb, "rn").float()
            a = (F.silu(g) * u).half().float()
            d = a @ ops.dequant(w2[e], s2u[e], s2v[e], cfg.K_expert, cfg.cb, "rn").float()
            y.index_add_(0, ts, w[ts, js, None] * d)
        h = h + y
    xf = m._rms(h, m.ln_f).to(torch.bfloat16)
    return (xf @ m.lm_head.t()).float(), tie


# Normwise tolerance of the verify step's logits against fp32 torch on the dequantised
# weights: the step keeps fp16 normed inputs and projection outputs and a bf16 KV cache
# and attention, as the plugin path does.
TOL_LOGITS = 1e-2


# batch 1, 3 and 7 run the fused attention sub-layer (rows_per_seq = 5; batch 7 in three
# calls of 3, 3 and 1 sequences), batch 9 and the fused=False case the torch-glue path
@pytest.mark.parametrize("batch,fused", [(1, None), (3, None), (7, None), (1, False), (9, None)])
def test_verify_step_matches_fp32_torch(cuda_device, batch, fused):
    torch.backends.cuda.matmul.allow_tf32 = False
    cfg = dataclasses.replace(CONFIG5, layers=2, hidden=1024, heads=8, kv_heads=2, experts=16, inter=512,
                              vocab=2048)
    ctx = 64
    m = VerifyModel(cfg, batch, ctx + cfg.rows_per_seq, cuda_device, fused=fused)
    assert m.fused == (batch <= 8 and fused is None)
    m.fill_random_kv(ctx)
    m.tokens.random_(0, cfg.vocab, generator=torch.Generator(device=cuda_device).manual_seed(2))
    ref, tie = _torch_verify_step(m)
    with torch.cuda.stream(m.stream):
        got = m.step()
    torch.cuda.synchronize()
    keep = ~tie
    assert int(keep.sum()) >= (m.rows + 1) // 2, "too many near-tied routes to compare"
    err = _rel(got[keep], ref[keep])
    print(f"verify step vs fp32 torch: {err:.2e} over {int(keep.sum())} of {m.rows} rows")
    assert err < TOL_LOGITS
    m.close()


# appended cache entries: bf16 of the same fp32 projections, within two bf16 ulps
TOL_KV = 2e-2


# 61: the 5 new positions straddle a 64-position chunk; batch 4: two calls of 3 and 1 sequences
@pytest.mark.parametrize("batch,ctx", [(2, 64), (3, 61), (4, 64)])
def test_verify_fused_attention_matches_unfused(cuda_device, batch, ctx):
    """The fused path (decode attention with 5 rows per sequence at positions
    ctx..ctx+4, causal among them) against the unfused torch-glue step on the same
    model: appended K/V, the step's logits, and a CUDA graph of the fused step."""
    cfg = dataclasses.replace(CONFIG5, layers=2, hidden=1024, heads=8, kv_heads=2, experts=16, inter=512,
                              vocab=2048)
    models = [VerifyModel(cfg, batch, ctx + 8, cuda_device, fused=f) for f in (True, False)]
    gen = torch.Generator(device=cuda_device).manual_seed(3)
    toks = torch.randint(0, cfg.vocab, (batch, cfg.rows_per_seq), device=cuda_device, generator=gen)
    outs = []
    for m in models:
        m.fill_random_kv(ctx)
        m.tokens.copy_(toks)
        with torch.cuda.stream(m.stream):
            outs.append(m.step().clone())
    torch.cuda.synchronize()
    fz, uf = models
    new = slice(ctx, ctx + cfg.rows_per_seq)
    for c in ("k_cache", "v_cache"):  # layer 0: the same inputs on both paths
        a, b = getattr(fz, c)[0, :, :, new].float(), getattr(uf, c)[0, :, :, new].float()
        assert a.abs().sum() > 0
        assert _rel(a, b) < TOL_KV, c
    assert torch.equal(fz.k_cache[:, :, :, :ctx], uf.k_cache[:, :, :, :ctx])  # older positions untouched
    # per row: a row whose top-k routing is within rounding of a tie may pick another
    # expert on one path; at most one such row is allowed
    row_err = (outs[0] - outs[1]).norm(dim=-1) / outs[1].norm(dim=-1)
    print(f"fused vs unfused verify logits per row: {row_err.tolist()}")
    assert int((row_err >= TOL_LOGITS).sum()) <= 1
    with torch.cuda.stream(fz.stream):
        again = fz.step().clone()
    fz.capture()
    fz.replay()
    torch.cuda.synchronize()
    noise, err = _rel(again, outs[0]), _rel(fz.logits, outs[0])
    print(f"fused eager vs eager {noise:.2e}, graph vs eager {err:.2e}")
    assert err < max(1e-3, 10 * noise)  # routed-MoE fp32 atomics may add in another order
    for m in models:
        m.close()
