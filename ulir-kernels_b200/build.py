"""Build libkernelsmith for B200 (sm_100a) in-tree.

Produces, under ulir-kernels_b200/lib/:
  libkernelsmith.so   shared drop-in (exports only the ks_* C ABI)
  libkernelsmith.a    static drop-in, for link-time replacement of the
                      reference's libkernelsmith.a (link with -lcudart_static
                      -lstdc++ -ldl -lrt -lpthread)

Usage: python ulir-kernels_b200/build.py [--force] [--ptxas-v]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
OBJ = PKG / "lib" / "obj"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-Wall",
    f"-I{ROOT / 'include'}",
    f"-I{PKG / 'target'}",
    f"-I{CSRC}",
]

SOURCES = sorted(CSRC.glob("*.cu"))
HEADERS = (
    sorted(CSRC.glob("*.cuh"))
    + sorted(CSRC.glob("*.h"))
    + sorted((ROOT / "include").rglob("*.h"))
    + sorted((PKG / "target").glob("*.h"))
)


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the B200 library cannot be built")
    return cand


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, ptxas_v: bool, force: bool) -> tuple[Path, str]:
    obj = OBJ / (src.stem + ".o")
    if not force and not _stale(obj, [src, *HEADERS, Path(__file__)]):
        return obj, ""
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stdout + res.stderr


def build(force: bool = False, ptxas_v: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link the libraries."""
    OBJ.mkdir(parents=True, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_v, force), SOURCES))
    objs = [o for o, _ in results]
    if verbose or ptxas_v:
        for _, log in results:
            if log:
                print(log, file=sys.stderr)
    so = LIB / "libkernelsmith.so"
    if force or _stale(so, objs):
        vscript = OBJ / "exports.map"
        vscript.write_text("{\n  global: ks_*;\n  local: *;\n};\n")
        cmd = [
            nvcc(),
            *ARCH,
            "-shared",
            "-cudart",
            "static",
            "-o",
            str(so),
            *map(str, objs),
            "-Xlinker",
            f"--version-script={vscript}",
            "-Xlinker",
            "-Bsymbolic",
        ]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    ar = LIB / "libkernelsmith.a"
    if force or _stale(ar, objs):
        if ar.exists():
            ar.unlink()
        subprocess.run(["ar", "rcs", str(ar), *map(str, objs)], check=True)
    return so


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    args = ap.parse_args()
    so = build(force=args.force, ptxas_v=args.ptxas_v, verbose=True)
    print(so)


if __name__ == "__main__":
    main()
