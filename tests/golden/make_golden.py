"""Generate the committed golden fixtures for the quantized GEMV parity tests.

Run with the reference tree named (--ref, or the KS_REFERENCE_DIR
environment variable) and its C library built by `make -C oracle ref`:

    python tests/golden/make_golden.py --ref /path/to/reference

Writes two files next to this script:

* reference_smoke.json -- the reference's own golden bundles for the
  quantized path (tests/golden/generated/{dot_i8,matvec_i8,dot_w4a8,
  matvec_w4a8,matmul_i8,rms_norm_f32}_smoke in the reference), copied as
  numbers after their sha256 is checked against each bundle's manifest, with
  the case parameters from the manifest (zero points, scales, group size,
  strides, compare policy).
* ref_seeded.npz / ref_seeded.json -- larger seeded cases whose expected
  outputs come from running the reference's C implementation
  (oracle/_ref/libks_ref_generic.so, compiled unmodified from the reference's
  lib/kernelsmith/*.c).  Inputs follow the reference generator convention,
  default_rng(seed + idx * 1009), and are stored too, so the fixtures do not
  depend on the numpy version that reads them.

GPU hosts never read the reference tree: tests use only these files.
"""

from __future__ import annotations

import argparse
import os
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "oracle"))

import oracle as O  # noqa: E402

SMOKE_CASES = ["dot_i8", "matvec_i8", "dot_w4a8", "matvec_w4a8", "matmul_i8", "rms_norm_f32"]

# name, kind, rows, cols, group, packed/weight stride (None = dense),
# scale stride (None = dense), sx, zx, zw, seed
SEEDED = [
    ("w4a8_fast_g32", "w4a8", 64, 256, 32, None, None, 0.02, 0, 0, 20261201),
    ("w4a8_fast_g128_zp", "w4a8", 20, 1024, 128, None, None, 0.05, -5, 1, 20261202),
    ("w4a8_fast_strided", "w4a8", 48, 512, 64, 272, 12, 0.03, 2, 0, 20261203),
    ("w4a8_generic_g10", "w4a8", 37, 130, 10, 80, 16, 0.125, 3, -2, 20261204),
    ("w4a8_generic_oddcols", "w4a8", 9, 77, 7, 39, 11, 0.25, 0, 0, 20261205),
    ("i8_fast", "i8", 64, 512, 0, None, None, 0.0, 0, 0, 20261211),
    ("i8_fast_zp", "i8", 40, 1024, 0, None, None, 0.0, 7, -9, 20261212),
    ("i8_generic_strided", "i8", 33, 100, 0, 112, None, 0.0, -3, 2, 20261213),
    ("i8_generic_odd", "i8", 17, 61, 0, 67, None, 0.0, -128, 127, 20261214),
]


def sha256(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def smoke_bundles(ref: Path) -> dict:
    out = {}
    for case in SMOKE_CASES:
        d = ref / "tests" / "golden" / "generated" / f"{case}_smoke"
        manifest = json.loads((d / "manifest.json").read_text())
        arrays = {}
        for t in manifest["tensors"]:
            f = d / t["filename"]
            if sha256(f) != t["sha256"]:
                raise SystemExit(f"sha256 mismatch for {f}")
            a = np.load(f)
            arrays[t["name"]] = {
                "role": t["role"],
                "dtype": str(a.dtype),
                "shape": list(a.shape),
                "layout": t.get("layout", {}),
                "data": a.ravel().tolist(),
            }
        out[case] = {
            "kernel": manifest["kernel"],
            "compare": manifest["compare"],
            "quantization_policy": manifest.get("quantization_policy", {}),
            "source": f"tests/golden/generated/{case}_smoke (reference), sha256-checked",
            "tensors": arrays,
        }
    return out


def seeded_cases() -> tuple[dict, dict]:
    ref = O.RefLib("generic")
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}
    for name, kind, rows, cols, group, wstride, sstride, sx, zx, zw, seed in SEEDED:
        x = O.rng(seed, 0).integers(-128, 128, size=cols, dtype=np.int8)
        if kind == "w4a8":
            prb = (cols + 1) // 2
            groups = -(-cols // group)
            wstride = wstride or prb
            sstride = sstride or groups
            w4 = O.rng(seed, 1).integers(-8, 8, size=(rows, cols), dtype=np.int8)
            packed = np.zeros((rows, wstride), np.uint8)
            packed[:, :prb] = O.pack_int4(w4)
            packed[:, prb:] = O.rng(seed, 3).integers(0, 256, size=(rows, wstride - prb), dtype=np.uint8)
            scales = O.rng(seed, 2).uniform(1e-3, 1e-2, size=(rows, sstride)).astype(np.float32)
            rc, y = ref.matvec_w4a8(x, packed, wstride, scales, sstride, rows, cols, group, sx, zx, zw)
            assert rc == 0, (name, rc)
            arrays[f"{name}.x"] = x
            arrays[f"{name}.w"] = packed
            arrays[f"{name}.s"] = scales
            arrays[f"{name}.y"] = y
        else:
            wstride = wstride or cols
            w = O.rng(seed, 1).integers(-128, 128, size=(rows, wstride), dtype=np.int8)
            rc, y = ref.matvec_i8(x, w, rows, cols, wstride, zx, zw)
            assert rc == 0, (name, rc)
            arrays[f"{name}.x"] = x
            arrays[f"{name}.w"] = w
            arrays[f"{name}.y"] = y
        meta[name] = dict(kind=kind, rows=rows, cols=cols, group=group, wstride=wstride,
                          sstride=sstride, sx=sx, zx=zx, zw=zw, seed=seed,
                          expected_from="reference C (lib/kernelsmith/ks_quantized.c, generic profile)")
    return arrays, meta


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("KS_REFERENCE_DIR"),
                    help="the reference tree (default: $KS_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("name the reference tree with --ref or KS_REFERENCE_DIR")
    ref = Path(args.ref)
    smoke = smoke_bundles(ref)
    (HERE / "reference_smoke.json").write_text(json.dumps(smoke, indent=1, sort_keys=True) + "\n")
    arrays, meta = seeded_cases()
    np.savez_compressed(HERE / "ref_seeded.npz", **arrays)
    (HERE / "ref_seeded.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(smoke)} smoke bundles and {len(meta)} seeded cases")


if __name__ == "__main__":
    main()
