"""The C-ABI library loads and exports every symbol include/*.h declares (no GPU calls)."""

import glob
import os
import re

import pytest

from exl3_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        names |= set(re.findall(r"EXL3B200_API\s+[\w\s\*]+?\b(exl3b200_\w+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    names = _declared_symbols()
    assert {"exl3b200_dequant", "exl3b200_gemv", "exl3b200_abi_version"} <= names


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in sorted(_declared_symbols()):
        assert hasattr(L, name), name


def test_ctypes_signatures_cover_header():
    assert set(_lib.SIGNATURES) == _declared_symbols()


def test_abi_version_and_status_strings():
    L = _lib.lib()
    assert L.exl3b200_abi_version() == 1
    assert _lib.status_string(0) == "ok"
    assert "workspace" in _lib.status_string(6)
    assert _lib.status_string(1234) == "unknown status"


def test_argument_validation_without_gpu():
    """Validation happens before any CUDA call, so these run on a CPU-only host."""
    L = _lib.lib()
    assert L.exl3b200_dequant(None, 8, 8, 4, 0, None, None, None, 0, None) == 7  # null
    fake = 256  # never dereferenced: rejected before use
    assert L.exl3b200_dequant(fake, 8, 8, 9, 0, fake, fake, fake, 0, None) == 2  # K
    assert L.exl3b200_dequant(fake, 8, 8, 4, 3, fake, fake, fake, 0, None) == 3  # codebook
    assert L.exl3b200_dequant(fake, 7, 8, 4, 0, fake, fake, fake, 0, None) == 1  # shape
    assert L.exl3b200_dequant(fake, 8, 8, 4, 0, fake, fake, fake, 2, None) == 8  # rounding
    args = dict(x=fake, xs=128, m=1, k=128, tr=fake, n=128, K=4, cb=0, suh=fake, svh=fake, out=fake,
                os=128, dt=0, fl=0, st=fake, stn=1 << 20, sc=fake, scn=1 << 20, stream=None)

    def gemv(**kw):
        a = dict(args)
        a.update(kw)
        return L.exl3b200_gemv(*a.values())

    assert gemv(m=17) == 1
    assert gemv(K=5) == 2
    assert gemv(cb=7) == 3
    assert gemv(k=100) == 1
    assert gemv(dt=3) == 8
    assert gemv(stn=16) == 6
    assert gemv(x=None) == 7
    assert L.exl3b200_gemv_state_size(4096) > 0
    assert L.exl3b200_gemv_state_size(100) == 0
    assert L.exl3b200_gemv_scratch_size(1, 4096) >= 8192


def test_missing_library_fails_loudly(monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libexl3b200.so")
    with pytest.raises(_lib.Exl3LibraryError):
        _lib.lib()


def test_tensor_core_moe_and_combine_validation_without_gpu():
    """exl3b200_moe_tc / exl3b200_gemm_combine reject bad arguments before any CUDA call."""
    import ctypes

    L = _lib.lib()
    f = 256  # never dereferenced
    assert L.exl3b200_moe_tc_scratch_size(64, 8, 128, 4096, 1536) > 0
    assert L.exl3b200_moe_tc_scratch_size(16384, 8, 128, 4096, 1536) == 0  # 131072 pairs > 65536
    assert L.exl3b200_moe_tc_scratch_size(64, 8, 4096, 4096, 1536) == 0    # > 2048 experts
    assert L.exl3b200_moe_tc_scratch_size(64, 8, 128, 4000, 1536) == 0     # hidden % 128
    tabs = [f] * 9
    ok = L.exl3b200_moe_tc_scratch_size(4, 2, 8, 256, 256)

    def moe(**kw):
        a = dict(x=f, xs=256, T=4, H=256, I=256, ids=f, w=f, topk=2, E=8, Kg=3, Ku=3, Kd=3, cb=0, out=4096,
                 os=256, mt=4, sc=4096, scb=ok)
        a.update(kw)
        return L.exl3b200_moe_tc(a["x"], a["xs"], a["T"], a["H"], a["I"], a["ids"], a["w"], a["topk"], a["E"],
                                 *tabs, a["Kg"], a["Ku"], a["Kd"], a["cb"], ctypes.c_float(0.0), a["out"], a["os"], 0,
                                 a["mt"], a["sc"], a["scb"], None)

    assert moe(x=None) == _lib.ENULL
    assert moe(T=5) == _lib.EBADSHAPE        # tokens > max_tokens
    assert moe(H=200) == _lib.EBADSHAPE
    assert moe(Kd=5) == _lib.EBADBITS
    assert moe(cb=3) == _lib.EBADCODEBOOK
    assert moe(out=4100) == _lib.EUNALIGNED  # fp32 rows need 16-byte alignment
    assert moe(os=258) == _lib.EUNALIGNED
    assert moe(scb=ok - 1) == _lib.EWORKSPACE

    assert L.exl3b200_gemm_combine_scratch_size(300, 256, 384) > 0
    assert L.exl3b200_gemm_combine_scratch_size(0, 256, 384) == 0
    g = dict(x=f, xs=256, m=40, k=256, tr=f, n=384, K=4, cb=1, suh=f, svh=f, out=4096, os=384, flags=0, sc=4096,
             scb=L.exl3b200_gemm_combine_scratch_size(40, 256, 384))

    def comb(**kw):
        a = dict(g)
        a.update(kw)
        return L.exl3b200_gemm_combine(a["x"], a["xs"], a["m"], a["k"], a["tr"], a["n"], a["K"], a["cb"], a["suh"],
                                       a["svh"], a["out"], a["os"], None, None, a["flags"], a["sc"], a["scb"], None)

    assert comb(suh=None) == _lib.ENULL                     # suh needed unless the input is rotated
    assert comb(n=300) == _lib.EBADSHAPE
    assert comb(K=1) == _lib.EBADBITS
    assert comb(svh=f + 8) == _lib.EUNALIGNED
    assert comb(scb=0) == _lib.EWORKSPACE


def test_decode_layer_validation_without_gpu():
    """Whole-layer decode entry point: workspace sizes and the argument checks that run
    before any CUDA call (fake device pointers, never dereferenced)."""
    import ctypes

    L = _lib.lib()
    st, sc = ctypes.c_size_t(), ctypes.c_size_t()
    ast, asc, mst, msc = (ctypes.c_size_t() for _ in range(4))
    assert L.exl3b200_decode_layer_workspace(2, 512, 8, 2, 1024, 96, ctypes.byref(st), ctypes.byref(sc)) == 0
    assert L.exl3b200_decode_attention_workspace(2, 512, 8, 2, 96, ctypes.byref(ast), ctypes.byref(asc)) == 0
    assert L.exl3b200_decode_mlp_workspace(2, 512, 1024, ctypes.byref(mst), ctypes.byref(msc)) == 0
    # one state and one scratch hold both sub-layers' (no aliasing) and the per-row pre-scale
    assert st.value == ast.value + mst.value
    assert sc.value == asc.value + msc.value + 256
    for bad in ((17, 512, 8, 2, 1024, 96), (2, 500, 8, 2, 1024, 96), (2, 512, 8, 3, 1024, 96),
                (2, 512, 34, 2, 1024, 96), (2, 512, 8, 2, 1000, 96), (2, 512, 8, 2, 1024, 0)):
        assert L.exl3b200_decode_layer_workspace(*bad, ctypes.byref(st), ctypes.byref(sc)) == 1, bad
    assert L.exl3b200_decode_layer_workspace(2, 512, 8, 2, 1024, 96, None, None) == 7

    fake = 1 << 20  # 256-byte aligned, never dereferenced

    def lin(k, n):
        return _lib.Linear(fake, fake, fake, k, n)

    lins = [lin(512, 1024), lin(512, 256), lin(512, 256), lin(1024, 512), lin(512, 1024), lin(512, 1024),
            lin(1024, 512)]
    q, k, v, o, g, u, d = (ctypes.addressof(x) for x in lins)
    layer = _lib.DecodeLayer(fake, q, k, v, o, fake, g, u, d)
    L.exl3b200_decode_layer_workspace(2, 512, 8, 2, 1024, 96, ctypes.byref(st), ctypes.byref(sc))

    def step(layer_p, next_p=None, state_n=None, scratch_n=None, ss_a=fake, rows=2):
        return L.exl3b200_decode_layer_step(
            rows, 1, 512, 8, 2, 1024, 4, 0, fake, 512, ss_a, fake, 1e-5, layer_p, next_p, 0, fake, fake, 96, fake,
            fake, 0.0, None, fake, st.value if state_n is None else state_n, fake,
            sc.value if scratch_n is None else scratch_n, None)

    assert step(None) == 7                                     # no layer
    assert step(ctypes.byref(layer), ss_a=None) == 7           # no sum-of-squares buffer
    assert step(ctypes.byref(layer), scratch_n=sc.value - 1) == 6  # workspace too small
    assert step(ctypes.byref(layer), rows=17) == 1             # more rows than the small-M kernels take
    wrong_gate = _lib.DecodeLayer(fake, q, k, v, o, fake, ctypes.addressof(lins[3]), u, d)
    assert step(ctypes.byref(wrong_gate)) == 1                 # gate is not hidden -> inter
    no_norm = _lib.DecodeLayer(0, q, k, v, o, fake, g, u, d)
    assert step(ctypes.byref(layer), ctypes.byref(no_norm)) == 7  # next layer without its norm weight
    wrong_q = _lib.DecodeLayer(fake, ctypes.addressof(lins[3]), k, v, o, fake, g, u, d)
    assert step(ctypes.byref(layer), ctypes.byref(wrong_q)) == 1  # next layer's q shape

