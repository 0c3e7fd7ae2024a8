"""The CPU oracle, pinned against the reference's own outputs (no GPU needed)."""

import os

import numpy as np
import pytest

import exl3_oracle as O


def _load(golden_dir, name):
    path = os.path.join(golden_dir, name)
    if not os.path.exists(path):
        pytest.skip(f"fixture {name} not generated")
    return np.load(path)


@pytest.mark.parametrize("K", [2, 3, 4, 8])
@pytest.mark.parametrize("cb", [1, 2])
def test_trunc_mode_matches_reference_dequant_bit_exact(golden_dir, K, cb):
    f = _load(golden_dir, "ref_dequant_trunc.npz")
    tag = f"{K}_{cb}"
    got = O.dequant(f[f"trellis_{tag}"], f[f"suh_{tag}"], f[f"svh_{tag}"], K, cb, "trunc")
    np.testing.assert_array_equal(got.view(np.uint16), f[f"out_{tag}"])


def test_mul1_rn_table_matches_reference_torch_lut(golden_dir):
    f = _load(golden_dir, "ref_mul1_lut.npz")
    np.testing.assert_array_equal(O.codebook_bits(2, "rn"), f["lut"])


def test_reference_cpu_gemv_fixture(golden_dir):
    """The reference's CPU exl3_gemv (trunc dequant + fp32 mm) against the oracle."""
    f = _load(golden_dir, "ref_cpu_gemv.npz")
    w = O.dequant(f["trellis"], f["suh"], f["svh"], 4, 1, "trunc").astype(np.float32)
    y = (f["x"].astype(np.float32) @ w).astype(np.float16)
    # both are one fp16 rounding of a float32 dot product; summation order may differ
    assert O.normwise_rel_err(f["y"], y) < 2e-3


@pytest.mark.parametrize("cb", [0, 1, 2])
def test_rn_tables_match_reference_device_decode(golden_dir, cb):
    f = _load(golden_dir, "ref_device_decode.npz")
    np.testing.assert_array_equal(O.codebook_bits(cb, "rn"), f[f"table_{cb}"])


@pytest.mark.parametrize("K", range(1, 9))
@pytest.mark.parametrize("cb", [0, 1, 2])
def test_windows_match_reference_device_extraction(golden_dir, K, cb):
    """dq_dispatch<K, cb> on a B200 (64 random tiles) equals window + table lookup."""
    f = _load(golden_dir, "ref_device_decode.npz")
    tiles = f[f"tiles_{K}"]
    lut = O.codebook_bits(cb, "rn")
    np.testing.assert_array_equal(lut[O.tile_windows(tiles, K)], f[f"decoded_{K}_{cb}"])


def test_truncation_differs_from_rounding():
    """The reference's two decodes disagree on a large share of the codebook."""
    for cb, lo in ((0, 10000), (1, 10000), (2, 20000)):
        assert int(np.sum(O.codebook_bits(cb, "rn") != O.codebook_bits(cb, "trunc"))) > lo


def test_swizzle_is_a_permutation():
    k, n = O._swizzle_index()
    assert len(set(zip(k.tolist(), n.tolist()))) == 256
    vals = np.arange(256, dtype=np.float32).reshape(1, 1, 256)
    m = O.tiles_to_matrix(vals)
    assert sorted(m.ravel().tolist()) == list(range(256))
    # lane 0 holds t = 0..7 at rows {0,1,8,9}, columns {0,8}
    assert m[0, 0] == 0 and m[1, 0] == 1 and m[8, 0] == 2 and m[9, 0] == 3 and m[0, 8] == 4


def test_fwht_is_involution_up_to_128():
    rng = np.random.default_rng(0)
    v = rng.standard_normal((3, 256)).astype(np.float32)
    h = O.fwht128(O.fwht128(v)) / 128.0
    np.testing.assert_allclose(h, v, rtol=1e-5, atol=1e-5)


def test_fwht_matches_hadamard_matrix():
    from scipy.linalg import hadamard

    H = hadamard(128).astype(np.float64)
    rng = np.random.default_rng(1)
    v = rng.standard_normal((2, 128)).astype(np.float32)
    np.testing.assert_allclose(O.fwht128(v), v.astype(np.float64) @ H, rtol=1e-5, atol=1e-4)


def test_window_of_known_stream():
    """K = 4, a tile whose stream is all zero except one nibble."""
    tr = np.zeros((1, 1, 64), dtype=np.int16)
    words = np.zeros(32, dtype=np.uint32)
    words[1] = 0xF0000000  # stream bits 32..35 (MSB first)
    tr[0, 0, 0::2] = (words & 0xFFFF).astype(np.uint16).view(np.int16)
    tr[0, 0, 1::2] = (words >> 16).astype(np.uint16).view(np.int16)
    w = O.tile_windows(tr, 4)[0, 0]
    # element t reads stream bits [4t - 12, 4t + 4): t = 8 ends at bit 35
    assert w[8] == 0x000F and w[9] == 0x00F0 and w[10] == 0x0F00 and w[11] == 0xF000 and w[12] == 0
    assert int(np.count_nonzero(w)) == 4


def test_dequant_scales_linearly_in_svh():
    rng = np.random.default_rng(2)
    tr = O.random_trellis(rng, 128, 128, 3)
    su = O.random_signs(rng, 128)
    sv = np.ones(128, dtype=np.float16)
    a = O.dequant(tr, su, sv, 3, 0).astype(np.float32)
    b = O.dequant(tr, su, -sv, 3, 0).astype(np.float32)
    np.testing.assert_array_equal(a, -b)


def test_moe_ref_ignores_invalid_ids():
    rng = np.random.default_rng(3)

    def lin(k, n):
        return (O.random_trellis(rng, k, n, 2), O.random_signs(rng, k), O.random_signs(rng, n), 2, 0)

    experts = [{"gate": lin(128, 128), "up": lin(128, 128), "down": lin(128, 128)} for _ in range(2)]
    x = rng.standard_normal((2, 128)).astype(np.float16)
    ids = np.array([[0, 1], [1, 5]])
    w = np.array([[0.5, 0.5], [1.0, 0.3]], dtype=np.float32)
    out = O.moe_ref(x, experts, ids, w)
    ids2 = np.array([[0, 1], [1, -1]])
    np.testing.assert_allclose(out, O.moe_ref(x, experts, ids2, w), rtol=0, atol=0)


def test_windows_match_bit_string_definition():
    """Random tiles, K = 1..8: the vectorised extraction equals a literal reading of the
    format - little-endian uint32 words, a cyclic MSB-first bit stream, element t the
    16 bits ending at stream bit (t + 1) * K - 1 (mod 256 K)."""
    from hypothesis import given, settings, strategies as st

    @settings(max_examples=40, deadline=None)
    @given(K=st.integers(1, 8), seed=st.integers(0, 2**31 - 1))
    def check(K, seed):
        rng = np.random.default_rng(seed)
        tile = rng.integers(-32768, 32768, size=16 * K).astype(np.int16)
        u16 = tile.view(np.uint16).astype(np.uint32)
        words = u16[0::2] | (u16[1::2] << 16)
        bits = "".join(format(int(w), "032b") for w in words)  # MSB first, word by word
        n = len(bits)
        got = O.tile_windows(tile.reshape(1, 1, -1), K)[0, 0]
        for t in range(256):
            end = ((t + 1) * K - 1) % n
            window = "".join(bits[(end - 15 + i) % n] for i in range(16))
            assert got[t] == int(window, 2), (K, t)

    check()
