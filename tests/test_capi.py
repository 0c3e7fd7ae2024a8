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
