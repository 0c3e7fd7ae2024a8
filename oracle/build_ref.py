"""Build the reference's own code, in place, into ``oracle/_ref/`` (test infrastructure).

Two artefacts, each compiled from the read-only reference sources where they lie
(never copied into this repository):

* ``sglang_exl3_ref*.so`` - the reference's pybind module ``csrc/bindings.cpp``
  built with g++ against the image's torch headers, with ``oracle/ref_stub.cpp``
  standing in for the six CUDA entry points.  Its ``dequant_trellis`` and the
  CPU branch of ``exl3_gemv`` (``csrc/bindings.cpp:15-147``) are the
  reference's CPU path: the bit-exact pin of the oracle's truncating mode and
  the timed CPU baseline.
* ``ref_codebook_dump`` - ``oracle/ref_codebook_dump.cu`` built with nvcc for
  sm_100a against ``csrc/quant/codebook.cuh`` / ``csrc/quant/exl3_dq.cuh``.
  Run on a B200 it dumps the reference device decode (tables and window
  extraction for K=1..8); ``tests/golden/make_fixtures.py`` turns the dump into
  a committed fixture.

Usage: ``python oracle/build_ref.py --reference /path/to/reference`` (or with the
environment variable ``EXL3_REFERENCE_DIR`` set).  Needs the reference tree, so it
only runs in the build container; the GPU box uses the prebuilt files.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
REF_ENV = "EXL3_REFERENCE_DIR"  # where the reference tree lies, when it is present


def reference_dir(arg=None):
    """The reference tree named by the argument or by ``EXL3_REFERENCE_DIR``, else None."""
    return arg or os.environ.get(REF_ENV) or None


def ref_module_path() -> str:
    return os.path.join(OUT, "sglang_exl3_ref" + sysconfig.get_config_var("EXT_SUFFIX"))


def dump_binary_path() -> str:
    return os.path.join(OUT, "ref_codebook_dump")


def _run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_cpu_module(ref: str) -> str:
    import torch
    import torch.utils.cpp_extension as ce

    out = ref_module_path()
    src = os.path.join(ref, "csrc", "bindings.cpp")
    stub = os.path.join(HERE, "ref_stub.cpp")
    if os.path.exists(out) and os.path.getmtime(out) > max(os.path.getmtime(src), os.path.getmtime(stub)):
        return out
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=sglang_exl3_ref", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-I{os.path.join(ref, 'csrc')}", f"-I{sysconfig.get_paths()['include']}"]
    cmd += [f"-I{p}" for p in ce.include_paths()]
    cmd += [src, stub, "-o", out]
    for p in ce.library_paths():
        cmd += [f"-L{p}", f"-Wl,-rpath,{p}"]
    cmd += ["-ltorch", "-ltorch_cpu", "-lc10", "-ltorch_python"]
    _run(cmd)
    return out


def build_dump_binary(ref: str) -> str:
    out = dump_binary_path()
    src = os.path.join(HERE, "ref_codebook_dump.cu")
    if os.path.exists(out) and os.path.getmtime(out) > os.path.getmtime(src):
        return out
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-w",
           f"-I{os.path.join(ref, 'csrc')}", src, "-o", out]
    _run(cmd)
    return out


def build(ref=None) -> bool:
    """Build both artefacts; returns False (and builds nothing) without the reference tree."""
    ref = reference_dir(ref)
    if not ref or not os.path.isdir(os.path.join(ref, "csrc")):
        return False
    os.makedirs(OUT, exist_ok=True)
    build_cpu_module(ref)
    build_dump_binary(ref)
    return True


def load_ref_module():
    """Import the compiled reference CPU module from ``oracle/_ref`` (or return None)."""
    import importlib.util

    path = ref_module_path()
    if not os.path.exists(path):
        return None
    import torch  # noqa: F401  (the module links against torch)

    spec = importlib.util.spec_from_file_location("sglang_exl3_ref", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help=f"reference tree (default: ${REF_ENV})")
    args = ap.parse_args()
    if not build(args.reference):
        print(f"reference tree not found at {args.reference}; nothing built", file=sys.stderr)
        sys.exit(1)
    print("built", ref_module_path(), dump_binary_path())
