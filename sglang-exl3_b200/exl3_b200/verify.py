"""Speculative-verify harness for the config-5 MoE model.

A random-initialised MoE decoder (48 layers, hidden 4096, 32 query / 4 KV heads of
128, 128 routed experts top-8 with intermediate 1536, vocab 151936): the experts
are EXL3 3 bpw and the attention projections EXL3 4 bpw (3INST), run by this
backend; embeddings, lm_head and the KV cache are bf16, the router fp32.  One verify step
takes ``draft`` proposed tokens plus the last accepted one for each of ``batch``
sequences (5 rows per sequence), runs them through every layer at positions
ctx .. ctx+4 (each row attends to the cache and to the new rows before it), and
returns the logits of all rows; the caller compares them with the draft.  The
step is captured in one CUDA graph.

Up to batch 8 the attention sub-layer is the fused decode sub-layer (one call per
chunk of up to 3 sequences, 16 rows)
(``decode.decode_attention`` with ``rows_per_seq = 5``: RMSNorm, q/k/v, RoPE and the
append of the 5 new positions, cluster attention causal among the new rows, o and the
residual, in 6 PDL-chained kernels on an fp32 residual stream); the MoE sub-layer
reads the row sums of squares it leaves.  Otherwise (and with ``fused=False``):

Per layer: RMSNorm -> q/k/v (one grouped EXL3 launch for 5*batch rows) -> RoPE ->
KV append -> attention (``scaled_dot_product_attention`` over the bf16 cache with
an explicit causal mask; the query heads of a KV head folded into the query
length, so the cache is read once per KV head) -> o (EXL3) -> residual -> RMSNorm
-> router (fp32, plus a fixed N(0, 1) term per row, below) ->
softmax, top-8, renormalised -> routed MoE (``moe.moe_forward``: the small-M or
the tensor-core pipeline by rows per expert) -> residual.  Under a process group
the experts are split over the ranks (expert parallelism over NVLink peer memory,
``ep.PeerExpertParallelMoE``: each row goes once to every rank owning one of its
experts, the weighted results come back); attention and the dense parts are
replicated, every rank verifying the same sequences.

The prompt is not run: the KV cache holds random values for ``ctx`` positions.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from . import decode as _dec
from . import moe as _moe
from . import ops
from .ep import PeerExpertParallelMoE
from .harness import _random_linear


@dataclass
class VerifyConfig:
    layers: int = 48
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    experts: int = 128
    topk: int = 8
    inter: int = 1536
    vocab: int = 151936
    rope_theta: float = 1e6
    K_attn: int = 4
    K_expert: int = 3
    cb: int = 0  # 3INST
    eps: float = 1e-6
    rows_per_seq: int = 5  # 4 draft tokens + 1


CONFIG5 = VerifyConfig()


class VerifyModel:
    def __init__(self, cfg: VerifyConfig, batch: int, max_ctx: int, device: torch.device, world: int = 1,
                 rank: int = 0, group=None, seed: int = 4, fused: Optional[bool] = None):
        if cfg.experts % world:
            raise ValueError(f"{cfg.experts} experts do not split over {world} ranks")
        self.cfg, self.batch, self.max_ctx, self.device = cfg, batch, max_ctx, device
        self.world, self.rank = world, rank
        H, hd, K = cfg.hidden, cfg.head_dim, cfg.K_attn
        qd, kvd = cfg.heads * hd, cfg.kv_heads * hd
        self.rows = batch * cfg.rows_per_seq
        # the fused attention sub-layer takes up to 16 rows per call: whole sequences of
        # rows_per_seq rows, so larger batches run it over chunks of sequences
        self.seq_chunk = 16 // cfg.rows_per_seq
        fusable = self.seq_chunk >= 1 and cfg.head_dim == 128 and cfg.heads // cfg.kv_heads <= 16
        if fused and not fusable:
            raise ValueError("the fused attention sub-layer takes up to 16 rows and head_dim 128")
        # measured on one B200 (8 layers, context 8192, ms per step unfused / fused):
        # batch 4 9.52 / 7.40, batch 8 11.06 / 10.08, batch 16 12.65 / 14.29 (the
        # attention codes then stream once per chunk of 3 sequences)
        self.fused = (fusable and batch <= 8) if fused is None else bool(fused)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)  # dense parts are the same on every rank
        egen = torch.Generator(device=device)
        egen.manual_seed(seed + 1000 * (rank + 1))
        el = cfg.experts // world
        I, KE = cfg.inter, cfg.K_expert
        self.layers = []
        for _ in range(cfg.layers):
            w13 = torch.randint(-32768, 32768, (el, 2, H // 16, I // 16, 16 * KE), dtype=torch.int16, device=device,
                                generator=egen)
            w2 = torch.randint(-32768, 32768, (el, I // 16, H // 16, 16 * KE), dtype=torch.int16, device=device,
                               generator=egen)

            def signs(*shape):
                return ((torch.randint(0, 2, shape, device=device, generator=egen) * 2 - 1).half()
                        * (torch.rand(shape, device=device, generator=egen) + 0.5).half())

            s13u, s13v, s2u, s2v = signs(el, 2, H), signs(el, 2, I), signs(el, I), signs(el, H)
            # random codes decode to weights of order 1: scale each projection's output by
            # 1/sqrt(k) so activations stay of order 1 (and the fp16 SwiGLU intermediate
            # finite) through 48 layers, as in a trained model
            s13v.mul_(H ** -0.5)
            s2v.mul_(I ** -0.5)

            def ptrs(t):
                return torch.tensor([int(t[e].data_ptr()) for e in range(el)], dtype=torch.int64, device=device)

            tables = {"gate_trellis": ptrs(w13[:, 0]), "gate_suh": ptrs(s13u[:, 0]), "gate_svh": ptrs(s13v[:, 0]),
                      "up_trellis": ptrs(w13[:, 1]), "up_suh": ptrs(s13u[:, 1]), "up_svh": ptrs(s13v[:, 1]),
                      "down_trellis": ptrs(w2), "down_suh": ptrs(s2u), "down_svh": ptrs(s2v)}
            qkv = [_random_linear(gen, H, qd, K, device), _random_linear(gen, H, kvd, K, device),
                   _random_linear(gen, H, kvd, K, device)]
            o = _random_linear(gen, qd, H, K, device)
            for lin, k_in in ((qkv[0], H), (qkv[1], H), (qkv[2], H), (o, qd)):
                lin[2].mul_(k_in ** -0.5)
            self.layers.append({
                "qkv": qkv,
                "o": o,
                # fp32 router: bf16 logits tie often at the top-k boundary, and which tied
                # expert wins then depends on the order of fp32 atomics upstream
                "router": torch.randn(cfg.experts, H, generator=gen, device=device) * 0.02,
                "experts": (w13, w2, s13u, s13v, s2u, s2v), "tables": tables,
                "ln1": torch.ones(H, dtype=torch.bfloat16, device=device),
                "ln2": torch.ones(H, dtype=torch.bfloat16, device=device),
            })
        self.embed = (torch.randn(cfg.vocab, H, generator=gen, device=device) * 0.02).to(torch.bfloat16)
        self.lm_head = (torch.randn(cfg.vocab, H, generator=gen, device=device) * 0.02).to(torch.bfloat16)
        self.ln_f = torch.ones(H, dtype=torch.bfloat16, device=device)
        self.k_cache = torch.zeros((cfg.layers, batch, cfg.kv_heads, max_ctx, hd), dtype=torch.bfloat16,
                                   device=device)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd))
        self.tokens = torch.zeros((batch, cfg.rows_per_seq), dtype=torch.long, device=device)
        self.pos = torch.zeros((), dtype=torch.long, device=device)  # first new position (= cached tokens)
        self.logits: Optional[torch.Tensor] = None
        self.h = torch.empty((self.rows, H), dtype=torch.float32, device=device)  # fused: residual stream
        self.ss = torch.zeros((2, self.rows), dtype=torch.float32, device=device)  # fused: row sums of h^2
        self.qkv = torch.empty((self.rows, qd + 2 * kvd), dtype=torch.float16, device=device)
        self.o = torch.empty((self.rows, H), dtype=torch.float16, device=device)
        self.ep = (PeerExpertParallelMoE(cfg.experts, self.rows, cfg.topk, H, group=group)
                   if world > 1 else None)
        # The random-init model's hidden states collapse onto a few routes (a handful of
        # experts per layer whatever the batch).  A fixed N(0, 1) term per (layer, row)
        # in the router logits spreads the routing the way a trained router does (the
        # config's "router logits ~N(0, 1)"), so a step touches as many experts as a
        # real verify step would.
        self.route_noise = torch.randn((cfg.layers, self.rows, cfg.experts), generator=gen, device=device)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.stream = torch.cuda.Stream(device)
        self.record: Optional[list] = None  # eager steps: distinct experts routed per layer

    def fill_random_kv(self, ctx: int) -> None:
        g = torch.Generator(device=self.device)
        g.manual_seed(5)
        for li in range(self.cfg.layers):
            self.k_cache[li, :, :, :ctx].normal_(generator=g)
            self.v_cache[li, :, :, :ctx].normal_(generator=g)
        self.pos.fill_(ctx)

    def _rms(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.eps) * w.float()).to(torch.float16)

    @staticmethod
    def _rope(t: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        t1, t2 = t[..., : t.size(-1) // 2], t[..., t.size(-1) // 2:]
        return torch.cat([t1 * cos - t2 * sin, t2 * cos + t1 * sin], dim=-1)

    def _local_moe(self, L, x16: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        return _moe.moe_forward(x16, ids, w, L["tables"], cfg.K_expert, cfg.K_expert, cfg.K_expert, cfg.cb,
                                cfg.inter)

    def _moe_sublayer(self, li, L, xn: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        logits = xn.float() @ L["router"].t() + self.route_noise[li]
        w, ids = torch.topk(torch.softmax(logits, dim=-1), cfg.topk, dim=-1)
        w = w / w.sum(-1, keepdim=True)
        if self.record is not None:
            self.record.append(int(torch.unique(ids).numel()))
        if self.ep is None:
            return self._local_moe(L, xn, ids.to(torch.int32), w)
        return self.ep(xn, ids, w, L["tables"], cfg.K_expert, cfg.K_expert, cfg.K_expert, cfg.cb, cfg.inter)

    def _step_fused(self) -> torch.Tensor:
        cfg = self.cfg
        h, ss = self.h, self.ss
        h.copy_(self.embed[self.tokens.reshape(-1)].float())
        torch.sum(h * h, dim=-1, out=ss[0])
        S, C = cfg.rows_per_seq, self.seq_chunk
        for li, L in enumerate(self.layers):
            for s0 in range(0, self.batch, C):
                s1 = min(self.batch, s0 + C)
                r0, r1 = s0 * S, s1 * S
                _dec.decode_attention(h[r0:r1], ss[0, r0:r1], ss[1, r0:r1], L["ln1"], cfg.eps, L["qkv"], L["o"],
                                      cfg.K_attn, cfg.cb, self.k_cache[li, s0:s1], self.v_cache[li, s0:s1],
                                      self.pos, self.inv_freq, rows_per_seq=S)
            # RMSNorm from the row sums of squares the attention sub-layer accumulated
            xn = (h * torch.rsqrt(ss[1, :, None] / cfg.hidden + cfg.eps) * L["ln2"].float()).to(torch.float16)
            h.add_(self._moe_sublayer(li, L, xn))
            torch.sum(h * h, dim=-1, out=ss[0])
        xf = self._rms(h, self.ln_f).to(torch.bfloat16)
        return (xf @ self.lm_head.t()).float()

    def step(self) -> torch.Tensor:
        """One verify step over the rows in ``self.tokens``; logits [batch*5, vocab] fp32."""
        if self.fused:
            return self._step_fused()
        cfg = self.cfg
        B, S, R = self.batch, cfg.rows_per_seq, self.rows
        hd, nh, nkv = cfg.head_dim, cfg.heads, cfg.kv_heads
        qd, kvd = nh * hd, nkv * hd
        positions = (self.pos + torch.arange(S, device=self.device)).repeat(B)  # [R]
        kv_len = self.max_ctx
        # row j of a sequence sees cache positions < pos + j + 1
        cols = torch.arange(kv_len, device=self.device)
        mask = cols[None, :] <= (self.pos + torch.arange(S, device=self.device))[:, None]  # [S, kv_len]
        mask_g = mask.repeat(cfg.heads // cfg.kv_heads, 1)  # [G * S, kv_len], row g * S + j
        ang = positions.float()[:, None] * self.inv_freq[None, :]  # [R, hd/2], the same for every layer
        cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
        h = self.embed[self.tokens.reshape(-1)].float()  # [R, H]
        for li, L in enumerate(self.layers):
            xn = self._rms(h, L["ln1"])
            outs = [self.qkv[:, :qd], self.qkv[:, qd:qd + kvd], self.qkv[:, qd + kvd:]]
            ops.matmul_multi(xn, L["qkv"], cfg.K_attn, cfg.cb, outs=outs)
            q = self._rope(self.qkv[:, :qd].float().view(R, nh, hd), cos, sin)
            k = self._rope(self.qkv[:, qd:qd + kvd].float().view(R, nkv, hd), cos, sin)
            v = self.qkv[:, qd + kvd:].float().view(R, nkv, hd)
            # append the 5 new positions of every sequence
            idx = positions.view(B, S)[0]  # same positions for every sequence
            self.k_cache[li].index_copy_(2, idx, k.view(B, S, nkv, hd).transpose(1, 2).to(torch.bfloat16))
            self.v_cache[li].index_copy_(2, idx, v.view(B, S, nkv, hd).transpose(1, 2).to(torch.bfloat16))
            # grouped-query attention without expanding the cache: the G query heads of a
            # kv head are folded into the query length (G * S rows per kv head)
            G = nh // nkv
            qh = q.view(B, S, nkv, G, hd).permute(0, 2, 3, 1, 4).reshape(B, nkv, G * S, hd).to(torch.bfloat16)
            att = F.scaled_dot_product_attention(qh, self.k_cache[li], self.v_cache[li], attn_mask=mask_g)
            att = att.view(B, nkv, G, S, hd).permute(0, 3, 1, 2, 4).reshape(R, qd).to(torch.float16)
            ops.matmul(att, *L["o"], cfg.K_attn, cfg.cb, out=self.o)
            h = h + self.o.float()
            xn = self._rms(h, L["ln2"])
            h = h + self._moe_sublayer(li, L, xn)
        xf = self._rms(h, self.ln_f).to(torch.bfloat16)
        return (xf @ self.lm_head.t()).float()

    def capture(self) -> None:
        s = self.stream
        s.wait_stream(torch.cuda.current_stream(self.device))
        pos0 = int(self.pos.item())
        with torch.cuda.stream(s):
            for _ in range(2):  # workspaces of this stream
                self.pos.fill_(pos0)
                self.logits = self.step()
            self.pos.fill_(pos0)
            torch.cuda.synchronize(self.device)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=s):
                self.logits = self.step()
        torch.cuda.current_stream(self.device).wait_stream(s)

    def replay(self, n: int = 1) -> None:
        with torch.cuda.stream(self.stream):
            for _ in range(n):
                self.graph.replay()

    def close(self) -> None:
        """Every rank, before the process group goes away (the peer buffers)."""
        self.graph = None
        if self.ep is not None:
            self.ep.close()
            self.ep = None
