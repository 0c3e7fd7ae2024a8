"""Decode harness for the Llama-70B-shaped benchmark model (config 4).

A random-initialised Llama-architecture decoder whose every linear is an EXL3
4-bpw 3INST layer run by this backend.  Embeddings, lm_head and the KV cache are
bf16.  Two step implementations:

* fused (default for batch <= 16): per layer the two fused sub-layers of
  ``exl3_b200.decode`` - RMSNorm in the matmul input stage, RoPE + KV append in
  the q/k/v epilogue, split-K attention, residual add in the o / down epilogues,
  SwiGLU in the gate/up epilogue - about a dozen kernels per layer;
* unfused: one grouped launch for q/k/v, one for o, one for gate/up, one for
  down, with RMSNorm, RoPE, KV append, SiLU*mul and attention
  (``scaled_dot_product_attention``) in plain torch.  Under
tensor parallelism (one process per GPU) q/k/v/gate/up are column shards, o/down
row shards followed by an NCCL all-reduce, and lm_head is sharded by vocabulary
with an all-gather of the logits.  A decode step (one token per sequence) is
captured in one CUDA graph.

The prompt is not run through the model: the KV cache is filled with random
values for ``ctx`` positions, which costs a decode step exactly as a real
prompt of that length would.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import ctypes

import torch
import torch.nn.functional as F

from . import _lib, ops


@dataclass
class DecoderConfig:
    layers: int = 80
    hidden: int = 8192
    heads: int = 64
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 28672
    vocab: int = 128256
    rope_theta: float = 5e5
    K: int = 4
    cb: int = 0  # 3INST
    eps: float = 1e-5


LLAMA_70B = DecoderConfig()


def _random_linear(gen: torch.Generator, k_in: int, n_out: int, K: int, device) -> tuple:
    tr = torch.randint(-32768, 32768, (k_in // 16, n_out // 16, 16 * K), dtype=torch.int16, device=device,
                       generator=gen)
    su = ((torch.randint(0, 2, (k_in,), device=device, generator=gen) * 2 - 1).half()
          * (torch.rand(k_in, device=device, generator=gen) + 0.5).half())
    sv = ((torch.randint(0, 2, (n_out,), device=device, generator=gen) * 2 - 1).half()
          * (torch.rand(n_out, device=device, generator=gen) + 0.5).half())
    return tr, su, sv


def exl3_weight_bytes(cfg: DecoderConfig, world: int = 1) -> int:
    """Trellis bytes one rank streams per decode step."""
    H, I, qd, kvd = cfg.hidden, cfg.inter, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    per_layer = (H * qd + 2 * H * kvd + qd * H + 3 * H * I) // world
    return cfg.layers * per_layer * cfg.K // 8


class DecodeModel:
    def __init__(self, cfg: DecoderConfig, batch: int, max_ctx: int, device: torch.device, world: int = 1,
                 rank: int = 0, group=None, seed: int = 3, fused: Optional[bool] = None, peer: bool = True,
                 fold: bool = True):
        if cfg.heads % world or cfg.kv_heads % world or cfg.inter % (128 * world) or cfg.vocab % world:
            raise ValueError(f"config does not shard over tp={world}")
        self.cfg, self.batch, self.max_ctx, self.device = cfg, batch, max_ctx, device
        self.world, self.rank, self.group = world, rank, group
        H, hd = cfg.hidden, cfg.head_dim
        self.hq, self.hkv = cfg.heads // world, cfg.kv_heads // world
        self.q_out, self.kv_out, self.i_loc = self.hq * hd, self.hkv * hd, cfg.inter // world
        gen = torch.Generator(device=device)
        gen.manual_seed(seed + 1000 * rank)
        K = cfg.K
        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append({
                "qkv": [_random_linear(gen, H, self.q_out, K, device), _random_linear(gen, H, self.kv_out, K, device),
                        _random_linear(gen, H, self.kv_out, K, device)],
                "o": _random_linear(gen, self.q_out, H, K, device),
                "gu": [_random_linear(gen, H, self.i_loc, K, device), _random_linear(gen, H, self.i_loc, K, device)],
                "down": _random_linear(gen, self.i_loc, H, K, device),
                "ln1": torch.ones(H, dtype=torch.bfloat16, device=device),
                "ln2": torch.ones(H, dtype=torch.bfloat16, device=device),
            })
        self.embed = (torch.randn(cfg.vocab, H, generator=gen, device=device) * 0.02).to(torch.bfloat16)
        self.v_loc = cfg.vocab // world
        self.lm_head = (torch.randn(self.v_loc, H, generator=gen, device=device) * 0.02).to(torch.bfloat16)
        self.ln_f = torch.ones(H, dtype=torch.bfloat16, device=device)
        # KV cache: [layer][B, kv_heads_local, max_ctx, head_dim] bf16
        # zero-filled: the unfused step attends over the whole cache with a mask, and a
        # masked position holding NaN garbage would still poison the softmax sum
        self.k_cache = torch.zeros((cfg.layers, batch, self.hkv, max_ctx, hd), dtype=torch.bfloat16, device=device)
        self.v_cache = torch.zeros_like(self.k_cache)
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd))
        self.inv_freq = inv
        # static step buffers
        self.tokens = torch.zeros(batch, dtype=torch.long, device=device)
        self.pos = torch.zeros((), dtype=torch.long, device=device)
        self.next_tokens = torch.zeros(batch, dtype=torch.long, device=device)
        self.qkv = torch.empty((batch, self.q_out + 2 * self.kv_out), dtype=torch.float16, device=device)
        self.gu = torch.empty((batch, 2 * self.i_loc), dtype=torch.float16, device=device)
        self.o = torch.empty((batch, H), dtype=torch.float16, device=device)
        self.down = torch.empty((batch, H), dtype=torch.float16, device=device)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.ctx = 0
        self.fused = (batch <= 16) if fused is None else bool(fused)
        if self.fused and batch > 16:
            raise ValueError("the fused decode layer takes at most 16 sequences")
        self.h = torch.zeros((batch, H), dtype=torch.float32, device=device)       # residual stream
        self.ss = torch.zeros((2, batch), dtype=torch.float32, device=device)      # per-row sum of squares
        self.y = torch.zeros((batch, H), dtype=torch.float32, device=device)       # TP partial outputs
        self.peers = None
        if self.fused and world > 1 and peer:
            from .decode import PeerExchange

            self.peers = PeerExchange(batch, H, group)  # partial sums over NVLink, no NCCL in the layers
        # whole layers with the RMSNorm input stages folded into the residual epilogues
        # (single GPU, or the peer exchange: the all-reduce form has no residual epilogue)
        self.fold = bool(fold) and self.fused and (world == 1 or self.peers is not None)
        self.layer_descs = []
        if self.fold:
            from .decode import LayerDesc

            self.layer_descs = [LayerDesc(L["ln1"], L["qkv"], L["o"], L["ln2"], L["gu"][0], L["gu"][1], L["down"])
                                for L in self.layers]

    def fill_random_kv(self, ctx: int, seed: int = 11):
        g = torch.Generator(device=self.device)
        g.manual_seed(seed + self.rank)
        for lay in range(self.cfg.layers):
            self.k_cache[lay, :, :, :ctx].normal_(generator=g)
            self.v_cache[lay, :, :, :ctx].normal_(generator=g)
        self.ctx = ctx
        self.pos.fill_(ctx)

    def _rms(self, h: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        hf = h.float()
        return (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + self.cfg.eps) * w.float()).to(torch.float16)

    def _rope(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        # x [B, heads, hd]; rotate-half convention
        ang = pos.float() * self.inv_freq
        cos, sin = torch.cos(ang), torch.sin(ang)
        x1, x2 = x[..., : x.shape[-1] // 2].float(), x[..., x.shape[-1] // 2:].float()
        return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)

    def _allreduce(self, t: torch.Tensor):
        if self.world > 1:
            torch.distributed.all_reduce(t, group=self.group)

    def step(self):
        """One decode step for the batch: reads self.tokens and self.pos, writes
        self.next_tokens (greedy) and appends to the KV cache."""
        if self.fused:
            return self._step_fused()
        return self._step_unfused()

    def _step_fused(self):
        from . import decode as D

        cfg = self.cfg
        h, ss = self.h, self.ss
        h.copy_(self.embed[self.tokens].float())
        torch.sum(h * h, dim=-1, out=ss[0])
        pe = self.peers
        if self.fold:
            descs = self.layer_descs
            for li, desc in enumerate(descs):
                D.decode_layer(h, ss[0], ss[1], cfg.eps, desc, descs[li + 1] if li + 1 < len(descs) else None, li > 0,
                               cfg.K, cfg.cb, self.k_cache[li], self.v_cache[li], self.pos, self.inv_freq, peers=pe)
            self._finish(h)
            return
        y = self.y if (self.world > 1 and pe is None) else None
        for li, L in enumerate(self.layers):
            D.decode_attention(h, ss[0], ss[1], L["ln1"], cfg.eps, L["qkv"], L["o"], cfg.K, cfg.cb,
                               self.k_cache[li], self.v_cache[li], self.pos, self.inv_freq, y=y, peers=pe)
            if y is not None:
                self._allreduce(y)
                D.residual_add(h, y, ss[1])
            D.decode_mlp(h, ss[1], ss[0], L["ln2"], cfg.eps, L["gu"][0], L["gu"][1], L["down"], cfg.K, cfg.cb, y=y,
                         peers=pe)
            if y is not None:
                self._allreduce(y)
                D.residual_add(h, y, ss[0])
        self._finish(h)

    def _finish(self, h: torch.Tensor):
        hf = self._rms(h, self.ln_f).to(torch.bfloat16)
        logits = hf @ self.lm_head.t()
        if self.world > 1:
            parts = [torch.empty_like(logits) for _ in range(self.world)]
            torch.distributed.all_gather(parts, logits, group=self.group)
            logits = torch.cat(parts, dim=-1)
        self.last_logits = logits
        self.next_tokens.copy_(logits.argmax(-1))
        self.tokens.copy_(self.next_tokens)
        self.pos.add_(1)

    def _step_unfused(self):
        cfg = self.cfg
        B, hd = self.batch, cfg.head_dim
        h = self.embed[self.tokens].float()
        pos = self.pos
        # causal mask over the fixed-size cache: positions <= pos are visible
        vis = (torch.arange(self.max_ctx, device=self.device) <= pos).view(1, 1, 1, self.max_ctx)
        for li, L in enumerate(self.layers):
            x = self._rms(h, L["ln1"])
            q, k, v = self.qkv[:, :self.q_out], self.qkv[:, self.q_out:self.q_out + self.kv_out], self.qkv[:, self.q_out + self.kv_out:]
            ops.matmul_multi(x, L["qkv"], cfg.K, cfg.cb, outs=[q, k, v])
            qh = self._rope(q.view(B, self.hq, hd), pos).to(torch.bfloat16)
            kh = self._rope(k.view(B, self.hkv, hd), pos).to(torch.bfloat16)
            self.k_cache[li].index_copy_(2, pos.view(1), kh.unsqueeze(2))
            self.v_cache[li].index_copy_(2, pos.view(1), v.view(B, self.hkv, hd).to(torch.bfloat16).unsqueeze(2))
            attn = F.scaled_dot_product_attention(qh.unsqueeze(2), self.k_cache[li], self.v_cache[li], attn_mask=vis,
                                                  enable_gqa=True)
            ops.matmul(attn.reshape(B, self.q_out).to(torch.float16), *L["o"], cfg.K, cfg.cb, out=self.o)
            self._allreduce(self.o)
            h = h + self.o.float()
            x = self._rms(h, L["ln2"])
            g, u = self.gu[:, :self.i_loc], self.gu[:, self.i_loc:]
            ops.matmul_multi(x, L["gu"], cfg.K, cfg.cb, outs=[g, u])
            act = (F.silu(g.float()) * u.float()).to(torch.float16)
            ops.matmul(act, *L["down"], cfg.K, cfg.cb, out=self.down)
            self._allreduce(self.down)
            h = h + self.down.float()
        self.h.copy_(h)
        self._finish(h)

    def capture(self, stream: Optional[torch.cuda.Stream] = None):
        """Warm up on a side stream and capture one decode step in a CUDA graph."""
        s = stream or torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        pos0 = int(self.pos.item())
        tok0 = self.tokens.clone()
        with torch.cuda.stream(s):
            for _ in range(2):
                self.step()
            self.pos.fill_(pos0)
            self.tokens.copy_(tok0)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self.step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.pos.fill_(pos0)
        self.tokens.copy_(tok0)
        self.graph = g
        self.stream = s
        return g

    def release(self):
        self.graph = None

    def close(self):
        """Release the graph and the peer buffers (every rank, before the process
        group is destroyed)."""
        self.release()
        if self.peers is not None:
            self.peers.close()
            self.peers = None

    def _pinned(self, n: int):
        """Pinned host buffers of a generate call (kept across calls: allocating page-locked
        memory costs far more than a decode step)."""
        buf = getattr(self, "_host_bufs", None)
        if buf is None or buf[1].size(1) < n:
            buf = (torch.empty(self.batch, dtype=torch.long).pin_memory(),
                   torch.empty((self.batch, n), dtype=torch.long).pin_memory())
            self._host_bufs = buf
        return buf

    def generate(self, prompt_tokens: torch.Tensor, n: int) -> torch.Tensor:
        """Public API: greedy-decode n tokens after ``prompt_tokens`` (host [B] last
        prompt tokens); returns the host [B, n] tokens.  Each step copies its input
        tokens from pinned host memory (the previous step's output as the host received
        it) and its output tokens back, then waits for them, as a serving loop does."""
        if self.graph is None:
            raise RuntimeError("call capture() first")
        host_in, host_out = self._pinned(n)
        status = self._status_host()
        host_in.copy_(prompt_tokens.to(torch.long))
        L = _lib.lib()
        with torch.cuda.stream(self.stream):
            for i in range(n):
                if i > 0:
                    host_in.copy_(host_out[:, i - 1])
                self.tokens.copy_(host_in, non_blocking=True)
                self.graph.replay()
                host_out[:, i].copy_(self.next_tokens, non_blocking=True)
                # the library's sticky device status rides along with the tokens: a
                # device wait that gave up (peer exchange, tensor-core pipeline) is an error
                L.exl3b200_device_status(ctypes.c_void_p(status.data_ptr()), 0, self.stream.cuda_stream)
                self.stream.synchronize()
                if int(status[0]) != 0:
                    raise RuntimeError(f"decode step {i}: device status {_lib.status_string(int(status[0]))}")
        return host_out[:, :n].clone()

    def _status_host(self) -> torch.Tensor:
        buf = getattr(self, "_status_buf", None)
        if buf is None:
            buf = torch.zeros(1, dtype=torch.int32).pin_memory()
            self._status_buf = buf
        return buf

    def decode(self, n: int):
        """Run n captured decode steps (feeding back the greedy tokens)."""
        if self.graph is None:
            raise RuntimeError("call capture() first")
        with torch.cuda.stream(self.stream):
            for _ in range(n):
                self.graph.replay()
