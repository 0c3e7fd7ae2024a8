"""Pure-torch CPU restatement of the EXL3 matmul: 65536-entry codebook table, window
gather, transforms, ``torch.mm`` on all host cores.

TEST INFRASTRUCTURE ONLY (a CPU baseline): only ``bench.py``'s CPU-baseline leg and
``tests/`` use it; the product path never imports it.

It follows the pattern of the reference's own pure-torch decode
(``src/sglang_exl3/ple_ngram.py:22-51``: build the codebook as a table over every
16-bit state, compute each weight's state from the packed stream, gather), applied
to the matmul's trellis format:

* codebook: the 3INST / MCG / mul1 tables of ``exl3_oracle.codebook_bits`` (device
  round-to-nearest semantics, ``csrc/quant/codebook.cuh:56-123``);
* windows: element t of a tile reads the 16 bits ending at stream bit (t+1)K-1 of
  the tile's cyclic MSB-first stream (``csrc/exl3_dequant.cuh:110-135``), here as
  int64 tensor arithmetic over column chunks;
* fragment swizzle (``csrc/bindings.cpp:51-75``) and the natural-order 128-point
  Hadamard transform as an fp32 matmul with the +-1 matrix, scale 1/sqrt(128),
  suh / svh (``csrc/bindings.cpp:79-98``);
* ``y = x @ W`` in fp32 (``torch.mm``).

The weight matrix is decoded in chunks of output columns, so memory stays bounded
for the 8192 x 28672 projections of the benchmark.
"""

from __future__ import annotations

import numpy as np
import torch

import exl3_oracle as O


def codebook_table(cb: int) -> torch.Tensor:
    """fp32 value of every 16-bit state (round-to-nearest fp16 codebook)."""
    return torch.from_numpy(O.codebook_values(cb).astype(np.float32))


def hadamard128() -> torch.Tensor:
    """Natural (Sylvester) order +-1 matrix of order 128, fp32."""
    h = torch.ones(1, 1)
    while h.size(0) < 128:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h


def _window_index(K: int):
    t = torch.arange(256, dtype=torch.int64)
    b0 = ((t + 257) * K - 16) % (256 * K)
    i1u = (b0 + 15) // 32
    i0 = (b0 // 32) % (8 * K)
    i1 = i1u % (8 * K)
    shift = (i1u + 1) * 32 - (b0 + 16)
    return i0, i1, shift


def _swizzle():
    t = torch.arange(256)
    lane, j = t // 8, t % 8
    k = 2 * (lane % 4) + (j & 1) + 8 * ((j >> 1) & 1)
    n = lane // 4 + 8 * (j >> 2)
    return k * 16 + n  # position of element t inside the row-major 16 x 16 tile


class TorchLutLinear:
    """One EXL3 linear decoded on the CPU with torch ops (``trellis`` int16
    ``[k/16, n/16, 16K]``, ``suh`` / ``svh`` fp16)."""

    def __init__(self, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int, cb: int,
                 chunk_cols: int = 2048):
        self.tr = trellis
        self.su = suh.float()
        self.sv = svh.float()
        self.K, self.cb = K, cb
        self.lut = codebook_table(cb)
        self.h128 = hadamard128() * float(O.HAD_SCALE)
        self.i0, self.i1, self.shift = _window_index(K)
        self.swz = _swizzle()
        self.chunk_tiles = max(8, chunk_cols // 16)

    def weight_chunk(self, nt0: int, nt1: int) -> torch.Tensor:
        """fp32 W[:, 16 nt0 : 16 nt1]."""
        w16 = self.tr[:, nt0:nt1].to(torch.int64) & 0xFFFF             # int16 words as unsigned
        words = w16[..., 0::2] | (w16[..., 1::2] << 16)               # [kt, nt, 8K] uint32 in int64
        merged = (words[..., self.i0] << 32) | words[..., self.i1]     # [kt, nt, 256]
        states = (merged >> self.shift) & 0xFFFF
        vals = self.lut[states]                                        # [kt, nt, 256] fp32
        kt, nt = vals.shape[0], vals.shape[1]
        tile = torch.empty_like(vals)
        tile[..., self.swz] = vals                                     # row-major 16 x 16 tiles
        m = tile.view(kt, nt, 16, 16).permute(0, 2, 1, 3).reshape(kt * 16, nt * 16)
        m = (m.view(kt * 16, nt // 8, 128) @ self.h128).view(kt * 16, nt * 16)           # rows (over n)
        m = (self.h128.t() @ m.view(kt // 8, 128, nt * 16)).view(kt * 16, nt * 16)       # columns (over k)
        return m * self.su[:, None] * self.sv[16 * nt0:16 * nt1][None, :]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        nt = self.tr.size(1)
        xf = x.float()
        out = torch.empty(x.size(0), nt * 16, dtype=torch.float32)
        for c0 in range(0, nt, self.chunk_tiles):
            c1 = min(nt, c0 + self.chunk_tiles)
            out[:, 16 * c0:16 * c1] = xf @ self.weight_chunk(c0, c1)
        return out
