"""Builds libb200fo.so (the sm_100a kernels and their C ABI) in-tree with nvcc.

Usage: ``python -m icpp_tuning_b200.build [--force] [-j N]``.  The library lands next to
this file so it travels with the source tree; nothing is installed elsewhere.
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
CSRC = PKG / "csrc"
ROOT = PKG.parent
INCLUDE = ROOT / "include"
LIB = PKG / "libb200fo.so"
OBJ = PKG / "_build"

# (source, object name, extra flags)
SOURCES = [
    ("fo_api.cu", "fo_api", []),
    ("fo_family_gemm.cu", "fo_family_gemm", ["-DFO_PAIR=0"]),
    ("fo_family_gemm.cu", "fo_family_gemm_pair", ["-DFO_PAIR=1"]),
    ("fo_family_ln.cu", "fo_family_ln", []),
    ("fo_family_conv.cu", "fo_family_conv", []),
    ("fo_family_direct.cu", "fo_family_direct", []),
    ("fo_noalloc.cu", "fo_noalloc", []),
]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def _deps() -> list[Path]:
    return [CSRC / s for s, _, _ in SOURCES] + list(CSRC.glob("*.cuh")) + [INCLUDE / "b200fo.h"]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def _compile(item, verbose: bool) -> Path:
    src, name, extra = item
    obj = OBJ / (name + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", str(CSRC / src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    OBJ.mkdir(exist_ok=True)
    jobs = jobs or min(len(SOURCES), os.cpu_count() or 1)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.verbose))


if __name__ == "__main__":
    main()
