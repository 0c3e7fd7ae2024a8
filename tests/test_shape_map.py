"""The kernel-shape map (exl3b200_select_shape; CPU: no kernel runs).  Pins the
selections to the crossovers measured on a B200: small-M with one 8-row group up to 8
rows, two groups up to 16, the tensor-core kernel from 17 rows (from 33 for matrices of
at most 2^24 weights; for every K); routed MoE on the tensor-core pipeline from 12 rows
per expert."""

import ctypes

import pytest

from exl3_b200 import _lib, ops

SHAPES_C4 = [(8192, 8192), (8192, 1024), (8192, 28672), (28672, 8192), (8192, 3584), (3584, 8192)]
SHAPES_C2 = [(5120, 51200), (25600, 5120)]


SHAPES_SMALL = [(2048, 2048), (1024, 2048), (4096, 1536), (2048, 8192)]  # config 3/5 experts, shared expert


@pytest.mark.parametrize("K", [2, 3, 4])
@pytest.mark.parametrize("k,n", SHAPES_C4 + SHAPES_C2 + SHAPES_SMALL)
def test_dense_selection(K, k, n):
    sel = [ops.select_shape(m, k, n, K, 0) for m in range(1, 65)]
    tc_from = 33 if k * n <= 1 << 24 else 17  # matrices of at most 2^24 weights: two 16-row chunks to 32 rows
    assert sel[:8] == [_lib.SHAPE_GV8] * 8
    assert sel[8:tc_from - 1] == [_lib.SHAPE_GV16] * (tc_from - 9)
    assert sel[tc_from - 1:] == [_lib.SHAPE_TC] * (65 - tc_from)
    assert ops.select_shape(2048, k, n, K, 1) == _lib.SHAPE_TC


@pytest.mark.parametrize("tokens,topk,experts,want", [
    (1, 8, 288, _lib.SHAPE_MOE_SMALL),     # decode
    (64, 8, 288, _lib.SHAPE_MOE_SMALL),    # config 3, T = 64: 1.8 rows per expert
    (512, 8, 288, _lib.SHAPE_MOE_TC),      # config 3, T = 512: 14 rows
    (80, 8, 128, _lib.SHAPE_MOE_SMALL),    # config 5, batch 16: 5 rows
    (160, 8, 128, _lib.SHAPE_MOE_SMALL),   # config 5, batch 32: 10 rows
    (320, 8, 128, _lib.SHAPE_MOE_TC),      # config 5, batch 64: 20 rows
    (12, 1, 1, _lib.SHAPE_MOE_TC),
    (11, 1, 1, _lib.SHAPE_MOE_SMALL),
])
def test_moe_selection(tokens, topk, experts, want):
    assert _lib.lib().exl3b200_select_shape(tokens, 2048, 1024, 3, 0, experts, topk) == want


def test_compat_and_info():
    L = _lib.lib()
    assert L.exl3b200_num_shapes() == 6
    assert L.exl3b200_shape_compat(_lib.SHAPE_GV8, 8, 256, 256, 4) == 1
    assert L.exl3b200_shape_compat(_lib.SHAPE_GV8, 9, 256, 256, 4) == 0
    assert L.exl3b200_shape_compat(_lib.SHAPE_GV16, 16, 256, 256, 3) == 1
    assert L.exl3b200_shape_compat(_lib.SHAPE_TC, 5000, 256, 384, 2) == 1
    assert L.exl3b200_shape_compat(_lib.SHAPE_TC, 5000, 200, 384, 2) == 0
    assert L.exl3b200_shape_compat(_lib.SHAPE_TC, 5000, 256, 384, 5) == 0
    assert L.exl3b200_shape_compat(7, 1, 256, 256, 4) == 0
    d = _lib.ShapeDesc()
    assert L.exl3b200_shape_info(_lib.SHAPE_TC, ctypes.byref(d)) == 0
    assert d.tile_rows == 256 and d.tile_cols == 256 and b"tcgen05" in d.name
    assert L.exl3b200_shape_info(0, ctypes.byref(d)) == _lib.EBADARG
    assert L.exl3b200_select_shape(1, 256, 256, 5, 0, 0, 0) == 0  # K outside 2..4: no shape
