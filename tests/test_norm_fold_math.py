"""The algebra of the decode layers' norm fold, on the CPU oracle.

A residual epilogue does not know the row's new RMS norm when it writes the next
sub-layer's input, so it writes fp16(h * w * c) with c = rsqrt(ss_old/hidden + eps) / 16
(the row's factor before the add, with a power-of-two headroom), and the consuming
epilogue multiplies the matmul's output by rsqrt(ss_new/hidden + eps) / c
(csrc/exl3_epilogue.cuh: fold_out, fold_factor).  The matmul is linear in its input,
so this equals normalising first, up to where the fp16 roundings fall; the headroom
keeps the folded input finite unless a row's norm grows by more than the documented
limit across one sub-layer.
"""

import numpy as np

import exl3_oracle as O

EPS = 1e-5
HEADROOM = 1.0 / 16


def _rs(h):
    return 1.0 / np.sqrt((h.astype(np.float64) ** 2).mean(-1, keepdims=True) + EPS)


def _linear(rng, k, n):
    return O.random_trellis(rng, k, n, 4), O.random_signs(rng, k), O.random_signs(rng, n)


def _fold_vs_norm(h_old, h_new, w, lin):
    tr, su, sv = lin
    x_norm = (h_new * _rs(h_new) * w).astype(np.float16)
    y_ref = O.gemv_ref(x_norm, tr, su, sv, 4, 0)
    c = _rs(h_old) * HEADROOM
    x_fold = (h_new * c * w).astype(np.float16)
    y_fold = O.gemv_ref(x_fold, tr, su, sv, 4, 0) * (_rs(h_new) / c)
    return x_fold, y_fold, y_ref


def test_fold_equals_normalised_input():
    rng = np.random.default_rng(7)
    k, n = 256, 128
    lin = _linear(rng, k, n)
    w = rng.uniform(0.5, 1.5, k).astype(np.float32)
    for growth in (0.05, 1.0, 30.0, 1000.0):
        h_old = rng.standard_normal((3, k)).astype(np.float32) * 0.02
        h_new = h_old + rng.standard_normal((3, k)).astype(np.float32) * 0.02 * growth
        x_fold, y_fold, y_ref = _fold_vs_norm(h_old, h_new, w, lin)
        assert np.isfinite(x_fold.astype(np.float32)).all()
        assert O.normwise_rel_err(y_fold, y_ref) < 2e-3, growth


def test_headroom_limit():
    """With the whole row's energy in one element, the folded input overflows fp16 once
    the norm grows by more than 65504 * 16 / sqrt(hidden) / |w| across the add (about
    1.2e4 at hidden 8192 and w = 1); below that it stays finite."""
    k = 8192
    w = np.ones(k, dtype=np.float32)
    h_old = np.full((1, k), 0.02, dtype=np.float32)
    limit = 65504.0 * 16 / np.sqrt(k)
    for growth, finite in ((0.9 * limit, True), (1.1 * limit, False)):
        h_new = np.zeros((1, k), dtype=np.float32)
        h_new[0, 0] = 0.02 * np.sqrt(k) * growth  # RMS = 0.02 * growth, all in one element
        c = _rs(h_old) * HEADROOM
        with np.errstate(over="ignore"):
            x_fold = (h_new * c * w).astype(np.float16)
        assert bool(np.isfinite(x_fold.astype(np.float32)).all()) == finite, growth
