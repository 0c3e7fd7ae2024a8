"""CPU oracle for the EXL3 trellis-decode matmul path.

TEST INFRASTRUCTURE ONLY.  This module is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it.
The product path (``sglang-exl3_b200``) never imports, links or calls it and
fails loudly when its CUDA library is missing.

It restates, in NumPy, the arithmetic of the reference (vcruz305/sglang-exl3)
for every step of the path, each function citing the reference lines it
follows:

* codebooks (3INST cb0, MCG cb1, mul1 cb2) with the device kernels'
  round-to-nearest fp16 semantics (``csrc/quant/codebook.cuh:26-123``), and
  with the reference CPU helpers' truncating semantics
  (``csrc/exl3_dequant.cuh:41-93``) so the restatement can be pinned
  bit-for-bit against the compiled reference ``dequant_cpu``;
* the trellis bit windows: element ``t`` of a 16x16 tile reads the 16 bits
  ending at stream bit ``(t+1)*K - 1`` of the tile's cyclic MSB-first stream of
  uint32 words (``csrc/exl3_dequant.cuh:110-135``, ``csrc/quant/exl3_dq.cuh:15-31``);
* the tensor-core fragment swizzle from the 256 decoded values to a row-major
  16x16 tile (``csrc/bindings.cpp:37-77``);
* the natural-order 128-point Walsh-Hadamard transform with the scale
  1/sqrt(128) and the suh / svh sign scales (``csrc/bindings.cpp:79-98``,
  ``csrc/quant/hadamard_inner.cuh:93-147``).

Pinning (see ``tests/test_oracle.py``): the truncating mode equals the output
of the reference's own ``dequant_trellis`` (compiled from
``csrc/bindings.cpp`` by ``oracle/build_ref.py``) bit for bit; the
round-to-nearest mul1 table equals the reference's pure-torch
``ple_ngram.mul1_codebook`` (``src/sglang_exl3/ple_ngram.py:22-29``) on all
65536 codes; and the round-to-nearest tables of all three codebooks equal the
reference's device functions run on a B200 (fixtures in ``tests/golden``).
"""

from __future__ import annotations

import numpy as np

INST3_MULT = 89226354
INST3_ADD = 64248484
MCG_MULT = 0xCBAC1FED
MUL1_MULT = 0x83DCD12D
MUL1_INV_BITS = 0x1EEE  # fp16 0.00677 (csrc/quant/codebook.cuh:38)
MUL1_BIAS_BITS = 0xC931  # fp16 -10.39 (csrc/quant/codebook.cuh:39)
HAD_SCALE = np.float32(0.08838834764831845)  # 1/sqrt(128) as float32

ROUNDING = ("rn", "trunc")


def _f16(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16)


def _lop3_6a(x: np.ndarray) -> np.ndarray:
    # lop3.b32 d, x, 0x8fff8fff, 0x3b603b60, 0x6a  ==  (x & b) ^ c
    return (x & np.uint64(0x8FFF8FFF)) ^ np.uint64(0x3B603B60)


def trunc_half_bits(v: np.ndarray) -> np.ndarray:
    """float32 -> fp16 bits by truncation, as ``float_to_half_bits``
    (``csrc/exl3_dequant.cuh:41-55``), including its subnormal branch."""
    v = np.asarray(v, dtype=np.float32)
    raw = v.view(np.uint32).astype(np.int64)
    sign = (raw >> 16) & 0x8000
    exp = ((raw >> 23) & 0xFF) - 127
    mant = raw & 0x7FFFFF
    normal = sign | ((exp + 15) << 10) | (mant >> 13)
    sub_shift = np.clip(-exp - 1, 0, 63)
    sub = sign | (((mant | 0x800000) >> sub_shift) >> 13)
    out = np.where(exp > 15, sign | 0x7C00,
                   np.where(exp < -14, np.where(exp < -24, sign, sub), normal))
    return out.astype(np.uint16)


def codebook_bits(cb: int, rounding: str = "rn") -> np.ndarray:
    """fp16 bit pattern of every codebook entry, indexed by the 16-bit window.

    ``rounding="rn"`` follows the device decode (``__hadd`` / ``__hfma`` round to
    nearest, ``csrc/quant/codebook.cuh:56-90``); ``"trunc"`` follows the CPU
    helpers of ``csrc/exl3_dequant.cuh:57-93``.
    """
    if cb not in (0, 1, 2):
        raise ValueError(f"codebook must be 0, 1 or 2, got {cb}")
    if rounding not in ROUNDING:
        raise ValueError(f"rounding must be one of {ROUNDING}")
    w = np.arange(65536, dtype=np.uint64)
    m32 = np.uint64(0xFFFFFFFF)
    if cb in (0, 1):
        if cb == 0:
            x = (w * np.uint64(INST3_MULT) + np.uint64(INST3_ADD)) & m32
        else:
            x = (w * np.uint64(MCG_MULT)) & m32
        x = _lop3_6a(x)
        lo = _f16((x & np.uint64(0xFFFF)).astype(np.uint16))
        hi = _f16((x >> np.uint64(16)).astype(np.uint16))
        if rounding == "rn":
            # both halves have exponents 12..15, so the float64 sum is exact and
            # the conversion is the single rounding of __hadd
            return (lo.astype(np.float64) + hi.astype(np.float64)).astype(np.float16).view(np.uint16)
        s = lo.astype(np.float32) + hi.astype(np.float32)
        return trunc_half_bits(s)
    x = (w * np.uint64(MUL1_MULT)) & m32
    bsum = (x & 0xFF) + ((x >> 8) & 0xFF) + ((x >> 16) & 0xFF) + ((x >> 24) & 0xFF)
    h = _f16((0x6400 + bsum).astype(np.uint16))
    k_inv = _f16(np.uint16(MUL1_INV_BITS))
    k_bias = _f16(np.uint16(MUL1_BIAS_BITS))
    if rounding == "rn":
        # exact in float64, then one rounding: the semantics of __hfma
        v = h.astype(np.float64) * np.float64(k_inv) + np.float64(k_bias)
        return v.astype(np.float16).view(np.uint16)
    p = h.astype(np.float32) * np.float32(k_inv)
    return trunc_half_bits(p + np.float32(k_bias))


def codebook_values(cb: int, rounding: str = "rn") -> np.ndarray:
    return _f16(codebook_bits(cb, rounding))


def tile_windows(trellis: np.ndarray, K: int) -> np.ndarray:
    """16-bit windows of every element of every tile: ``[..., 16K] -> [..., 256]``.

    The tile's int16 words pair into little-endian uint32 words; the stream is
    read MSB first; element t takes bits ``[(t+257)K-16, (t+257)K)`` modulo the
    tile's ``256K`` bits (``csrc/exl3_dequant.cuh:110-135``).
    """
    tw = np.asarray(trellis).view(np.uint16)
    if tw.shape[-1] != 16 * K:
        raise ValueError(f"last dim {tw.shape[-1]} != 16*K ({16 * K})")
    lo = tw[..., 0::2].astype(np.uint64)
    hi = tw[..., 1::2].astype(np.uint64)
    words = lo | (hi << np.uint64(16))
    n32 = 8 * K
    t = np.arange(256, dtype=np.int64)
    b0 = ((t + 257) * K - 16) % (256 * K)
    i1u = (b0 + 15) // 32
    i0 = (b0 // 32) % n32
    i1 = i1u % n32
    shift = ((i1u + 1) * 32 - (b0 + 16)).astype(np.uint64)
    merged = (words[..., i0] << np.uint64(32)) | words[..., i1]
    return ((merged >> shift) & np.uint64(0xFFFF)).astype(np.uint16)


def _swizzle_index():
    """(k, n) inside a 16x16 tile of decoded element t (``csrc/bindings.cpp:51-75``):
    lane L = t // 8, j = t % 8, k = 2(L%4) + (j&1) + 8((j>>1)&1), n = L//4 + 8(j>>2)."""
    t = np.arange(256)
    lane, j = t // 8, t % 8
    k = 2 * (lane % 4) + (j & 1) + 8 * ((j >> 1) & 1)
    n = lane // 4 + 8 * (j >> 2)
    return k, n


_SWZ_K, _SWZ_N = _swizzle_index()


def tiles_to_matrix(vals: np.ndarray) -> np.ndarray:
    """``[Kt, Nt, 256]`` per-tile values in decode order -> ``[Kt*16, Nt*16]``."""
    Kt, Nt, _ = vals.shape
    out = np.empty((Kt, 16, Nt, 16), dtype=vals.dtype)
    out[:, _SWZ_K, :, _SWZ_N] = vals.transpose(2, 0, 1)
    return out.reshape(Kt * 16, Nt * 16)


def decode_raw(trellis: np.ndarray, K: int, cb: int, rounding: str = "rn") -> np.ndarray:
    """Decoded codebook values before the Hadamard transforms, fp16 ``[K_in, N_out]``."""
    lut = codebook_bits(cb, rounding)
    win = tile_windows(trellis, K)
    return tiles_to_matrix(_f16(lut[win]))


def fwht128(v: np.ndarray, axis: int = -1) -> np.ndarray:
    """Unnormalised natural-order Walsh-Hadamard transform over blocks of 128,
    float32, butterfly strides 1, 2, ..., 64 in the order of
    ``csrc/exl3_dequant.cuh:137-148`` (the warp form of
    ``csrc/quant/hadamard_inner.cuh:17-44,93-147`` adds in the same order)."""
    v = np.moveaxis(np.asarray(v, dtype=np.float32), axis, -1)
    lead = v.shape[:-1]
    n = v.shape[-1]
    if n % 128:
        raise ValueError("length must be a multiple of 128")
    v = v.reshape(*lead, n // 128, 128)
    s = 1
    while s < 128:
        w = v.reshape(*lead, n // 128, 128 // (2 * s), 2, s)
        a = w[..., 0, :]
        b = w[..., 1, :]
        v = np.stack([a + b, a - b], axis=-2).reshape(*lead, n // 128, 128)
        s *= 2
    return np.moveaxis(v.reshape(*lead, n), -1, axis)


def dequant(trellis: np.ndarray, suh: np.ndarray, svh: np.ndarray, K: int, cb: int,
            rounding: str = "rn") -> np.ndarray:
    """Full fp16 weight ``W[k, n]`` with ``y = x @ W`` (``csrc/bindings.cpp:15-100``).

    Row transform (over n) then column transform (over k), each scaled by
    1/sqrt(128) in float32, then ``* suh[k] * svh[n]`` and one fp16 rounding."""
    Kt, Nt, _ = trellis.shape
    if (Kt * 16) % 128 or (Nt * 16) % 128:
        raise ValueError("trellis dimensions must reconstruct whole 128-element Hadamard blocks")
    m = decode_raw(trellis, K, cb, rounding).astype(np.float32)
    m = fwht128(m, axis=1) * HAD_SCALE
    m = fwht128(m, axis=0)
    su = np.asarray(suh, dtype=np.float16).astype(np.float32)[: Kt * 16]
    sv = np.asarray(svh, dtype=np.float16).astype(np.float32)[: Nt * 16]
    m = ((m * HAD_SCALE) * su[:, None]) * sv[None, :]
    return m.astype(np.float16)


def input_transform(x: np.ndarray, suh: np.ndarray) -> np.ndarray:
    """fp16 ``H128(x * suh) / sqrt(128)`` with the device roundings of
    ``had_hf_r_128_inner<true,false>`` (``csrc/quant/hadamard_inner.cuh:93-147``):
    fp16 product, float32 transform and scale, one fp16 rounding."""
    xs = (np.asarray(x, dtype=np.float16).astype(np.float32)
          * np.asarray(suh, dtype=np.float16).astype(np.float32)).astype(np.float16)
    h = fwht128(xs.astype(np.float32), axis=-1) * HAD_SCALE
    return h.astype(np.float16)


def output_transform(acc: np.ndarray, svh: np.ndarray) -> np.ndarray:
    """float32 ``H128(acc) / sqrt(128) * svh`` over blocks of 128 output columns."""
    h = fwht128(np.asarray(acc, dtype=np.float32), axis=-1) * HAD_SCALE
    return h * np.asarray(svh, dtype=np.float16).astype(np.float32)


def gemv_ref(x: np.ndarray, trellis: np.ndarray, suh: np.ndarray, svh: np.ndarray,
             K: int, cb: int) -> np.ndarray:
    """The parity reference of the matmul ops: fp32 ``x @ W`` on the
    round-to-nearest dequantised weights."""
    w = dequant(trellis, suh, svh, K, cb, "rn").astype(np.float32)
    return np.asarray(x, dtype=np.float16).astype(np.float32) @ w


def fat_gemm_ref(a: np.ndarray, trellis: np.ndarray, svh: np.ndarray, K: int, cb: int) -> np.ndarray:
    """``exl3_fat_gemm``: the input is already rotated, output float32
    ``H128(a @ W_raw) / sqrt(128) * svh`` (``csrc/exl3_fat_gemm.cu:33-63,139-197``)."""
    raw = decode_raw(trellis, K, cb, "rn").astype(np.float32)
    acc = np.asarray(a, dtype=np.float16).astype(np.float32) @ raw
    return output_transform(acc, svh)


def silu(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, dtype=np.float64)
    return v / (1.0 + np.exp(-v))


def swiglu(gate: np.ndarray, up: np.ndarray, limit: float = 0.0) -> np.ndarray:
    """SwiGLU with the optional input clip of ``p2b_moe.cu:304-313``
    (``limit`` 0 or infinite disables it): ``silu(min(g, L)) * clamp(u, -L, L)``."""
    g = np.asarray(gate, dtype=np.float64)
    u = np.asarray(up, dtype=np.float64)
    if limit and np.isfinite(limit) and limit > 0:
        g = np.minimum(g, limit)
        u = np.clip(u, -limit, limit)
    return silu(g) * u


def linear_device_ref(x: np.ndarray, trellis: np.ndarray, suh: np.ndarray, svh: np.ndarray, K: int,
                      cb: int) -> np.ndarray:
    """``x @ W`` with the device pipeline's roundings: fp16 rotated input
    (``input_transform``), float64 product with the raw decoded tile matrix, then the
    output transform.  Differs from ``gemv_ref`` only in where fp16 roundings sit."""
    xh = input_transform(x, suh).astype(np.float64)
    raw = decode_raw(trellis, K, cb, "rn").astype(np.float64)
    return output_transform(xh @ raw, svh)


def moe_ref(x: np.ndarray, experts: list, ids: np.ndarray, weights: np.ndarray,
            limit: float = 0.0) -> np.ndarray:
    """Routed SwiGLU MoE for rows of ``x``: ``sum_j w[t,j] * down_e(swiglu(gate_e x, up_e x))``
    (``p2b_moe.cu:202-379``, ``exl3.py:960-1110``).  ``experts[e]`` is a dict with
    ``gate``/``up``/``down`` each ``(trellis, suh, svh, K, cb)``.  Ids outside
    ``[0, len(experts))`` contribute nothing (``exl3.py:494-509``).  The fp16
    intermediates sit where the reference keeps them: rotated inputs, the SwiGLU
    activation, and the rotated down-projection input."""
    x = np.asarray(x, dtype=np.float16)
    T = x.shape[0]
    out = np.zeros((T, x.shape[1]), dtype=np.float64)
    ids = np.asarray(ids)
    for e in range(len(experts)):
        ts, js = np.nonzero(ids == e)  # every (token, slot) routed to expert e; rows are independent
        if ts.size == 0:
            continue
        xt = x[ts]
        g = linear_device_ref(xt, *experts[e]["gate"])
        u = linear_device_ref(xt, *experts[e]["up"])
        a = swiglu(g, u, limit).astype(np.float16)
        d = linear_device_ref(a, *experts[e]["down"]).astype(np.float64)
        np.add.at(out, ts, np.asarray(weights, dtype=np.float64)[ts, js][:, None] * d)
    return out.astype(np.float32)


def normwise_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max |got - ref| / max |ref| — the error measure the parity tests bound."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = float(np.max(np.abs(ref)))
    if denom == 0.0:
        return float(np.max(np.abs(got)))
    return float(np.max(np.abs(got - ref)) / denom)


def random_trellis(rng: np.random.Generator, k_in: int, n_out: int, K: int) -> np.ndarray:
    """Uniform random int16 codes ``[k_in/16, n_out/16, 16K]``."""
    return rng.integers(-32768, 32768, size=(k_in // 16, n_out // 16, 16 * K), dtype=np.int64).astype(np.int16)


def random_signs(rng: np.random.Generator, n: int) -> np.ndarray:
    """fp16 +-1 signs times U(0.5, 1.5), the suh/svh distribution of the benchmark configs."""
    s = np.where(rng.integers(0, 2, size=n) == 0, -1.0, 1.0)
    return (s * rng.uniform(0.5, 1.5, size=n)).astype(np.float16)
