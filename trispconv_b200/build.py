"""Builds libtrispconv_b200.so in-tree with nvcc for sm_100a.

Usage: ``python -m trispconv_b200.build`` (or ``__graft_entry__.build()``).
The shared library is written next to this file so that it travels with the
source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libtrispconv_b200.so"
BUILD_DIR = ROOT / "_build"

GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found: the trispconv_b200 CUDA library cannot be built")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compiles every csrc/*.cu for sm_100a and links libtrispconv_b200.so."""
    srcs = sources()
    deps = srcs + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))
    if LIB.exists() and not force:
        lib_mtime = LIB.stat().st_mtime
        if all(p.stat().st_mtime <= lib_mtime for p in deps):
            return LIB
    BUILD_DIR.mkdir(exist_ok=True)
    nvcc = _nvcc()

    def compile_one(src: Path):
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [nvcc, *GENCODE, *NVCC_FLAGS, "-I", str(ROOT / "include"), "-I", str(CSRC),
               "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        (BUILD_DIR / (src.stem + ".ptxas.txt")).write_text(res.stdout + res.stderr)
        return src, obj, res

    from concurrent.futures import ThreadPoolExecutor

    workers = max(1, min(len(srcs), os.cpu_count() or 1))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        results = list(pool.map(compile_one, srcs))
    objs = []
    for src, obj, res in results:
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError(f"nvcc failed on {src.name}")
        if verbose:
            sys.stdout.write(res.stdout + res.stderr)
        objs.append(obj)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *GENCODE, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("linking libtrispconv_b200.so failed")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(path)
