"""Generate the golden fixtures in ``tests/golden`` from the reference itself.

Run in the build container, where the reference tree is present:

    python oracle/build_ref.py --reference R   # compiles the reference into oracle/_ref
    python tests/golden/make_fixtures.py --reference R   # CPU fixtures
    python tests/golden/make_fixtures.py --device-dump <dump file>
                                               # the file oracle/_ref/ref_codebook_dump wrote on a B200

Fixtures (inputs are seeded; outputs come from the reference's own code):

* ``ref_dequant_trunc.npz`` - the reference's ``dequant_trellis``
  (``csrc/bindings.cpp:15-132``, compiled by ``oracle/build_ref.py``) on seeded
  trellis/suh/svh for K in {2, 3, 4, 8} x {MCG, mul1}.
* ``ref_mul1_lut.npz`` - the reference's pure-torch ``mul1_codebook``
  (``src/sglang_exl3/ple_ngram.py:22-29``), all 65536 entries.
* ``ref_cpu_gemv.npz`` - the reference's CPU ``exl3_gemv`` (dequant + at::mm,
  ``csrc/bindings.cpp:134-147``) on a seeded small case.
* ``ref_device_decode.npz`` - the reference's device decode functions
  (``decode_3inst<cb>``, ``dq_dispatch<K, cb>``) run on a B200 by
  ``oracle/_ref/ref_codebook_dump``: the three codebook tables and the first 16 of the
  dump's 64 tiles per K in 1..8.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import exl3_oracle as O  # noqa: E402
from build_ref import load_ref_module, reference_dir  # noqa: E402


def make_dequant(ref) -> None:
    import torch

    rng = np.random.default_rng(1234)
    arrays = {}
    for K in (2, 3, 4, 8):
        for cb in (1, 2):
            k_in, n_out = 128, 128
            tr = O.random_trellis(rng, k_in, n_out, K)
            su = O.random_signs(rng, k_in)
            sv = O.random_signs(rng, n_out)
            out = ref.dequant_trellis(torch.from_numpy(tr), torch.from_numpy(su), torch.from_numpy(sv),
                                      K, cb == 1).numpy()
            tag = f"{K}_{cb}"
            arrays[f"trellis_{tag}"] = tr
            arrays[f"suh_{tag}"] = su
            arrays[f"svh_{tag}"] = sv
            arrays[f"out_{tag}"] = out.view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "ref_dequant_trunc.npz"), **arrays)


def make_mul1_lut(ref_dir: str) -> None:
    spec = importlib.util.spec_from_file_location("ref_ple_ngram",
                                                  os.path.join(ref_dir, "src/sglang_exl3/ple_ngram.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    lut = mod.mul1_codebook("cpu").numpy().view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "ref_mul1_lut.npz"), lut=lut)


def make_cpu_gemv(ref) -> None:
    import torch

    rng = np.random.default_rng(99)
    K = 4
    tr = O.random_trellis(rng, 256, 256, K)
    su = O.random_signs(rng, 256)
    sv = O.random_signs(rng, 256)
    x = rng.standard_normal((3, 256)).astype(np.float16)
    y = ref.exl3_gemv(torch.from_numpy(x), torch.from_numpy(tr), torch.from_numpy(su), torch.from_numpy(sv),
                      K, True, 1).numpy()
    np.savez_compressed(os.path.join(HERE, "ref_cpu_gemv.npz"), x=x, trellis=tr, suh=su, svh=sv, y=y)


def convert_device_dump(path: str) -> None:
    raw = open(path, "rb").read()
    if raw[:8] != b"EXL3CBD1":
        raise SystemExit(f"{path}: not a ref_codebook_dump output")
    off = 8
    arrays = {}
    for cb in range(3):
        arrays[f"table_{cb}"] = np.frombuffer(raw, dtype=np.uint16, count=65536, offset=off).copy()
        off += 65536 * 2
    ntiles = int(np.frombuffer(raw, dtype=np.uint32, count=1, offset=off)[0])
    off += 4
    for K in range(1, 9):
        nw = ntiles * 16 * K
        arrays[f"tiles_{K}"] = np.frombuffer(raw, dtype=np.uint16, count=nw, offset=off).reshape(ntiles, 16 * K).copy()
        off += nw * 2
        for cb in range(3):
            arrays[f"decoded_{K}_{cb}"] = np.frombuffer(raw, dtype=np.uint16, count=ntiles * 256, offset=off).reshape(ntiles, 256).copy()
            off += ntiles * 256 * 2
    if off != len(raw):
        raise SystemExit(f"{path}: {len(raw) - off} trailing bytes")
    # keep the full tables and the first 16 tiles per K (the dump holds 64)
    for key in list(arrays):
        if key.startswith(("tiles_", "decoded_")):
            arrays[key] = arrays[key][:16]
    np.savez_compressed(os.path.join(HERE, "ref_device_decode.npz"), **arrays)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--device-dump", default=None, help="raw output of oracle/_ref/ref_codebook_dump")
    ap.add_argument("--reference", default=None, help="reference tree (default: $EXL3_REFERENCE_DIR)")
    args = ap.parse_args()
    if args.device_dump:
        convert_device_dump(args.device_dump)
    else:
        ref = load_ref_module()
        if ref is None:
            raise SystemExit("oracle/_ref not built: run python oracle/build_ref.py first")
        ref_dir = reference_dir(args.reference)
        if not ref_dir:
            raise SystemExit("name the reference tree: --reference or EXL3_REFERENCE_DIR")
        make_dequant(ref)
        make_mul1_lut(ref_dir)
        make_cpu_gemv(ref)
    print("fixtures written to", HERE)
