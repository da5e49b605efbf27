"""Build libsmooth_attn_b200.so (all CUDA sources, sm_100a) in-tree.

    python smooth-attn_b200/build.py [-j N] [--force] [--debug]

Each ``csrc/*.cu`` is compiled with ``nvcc -gencode arch=compute_100a,code=sm_100a``
to an object under ``smooth-attn_b200/_build/`` (rebuilt when the source or
any header is newer), then linked with the static CUDA runtime into
``smooth-attn_b200/smooth_attn/libsmooth_attn_b200.so``.

``--debug`` builds the same sources with ``-DSA_DEBUG_CHECKS`` (device-side
index checks that count failures instead of trapping; see ``csrc/sa_common.cuh``)
into ``_build_debug/`` and ``smooth_attn/libsmooth_attn_b200_debug.so``, which
``smooth_attn`` loads when the environment sets ``SA_DEBUG_LIB=1``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
CSRC = PKG_ROOT / "csrc"
BUILD = PKG_ROOT / "_build"
REPO = PKG_ROOT.parent
INCLUDE = REPO / "include"
LIB = PKG_ROOT / "smooth_attn" / "libsmooth_attn_b200.so"
BUILD_DEBUG = PKG_ROOT / "_build_debug"
LIB_DEBUG = PKG_ROOT / "smooth_attn" / "libsmooth_attn_b200_debug.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _deps_mtime():
    files = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((f.stat().st_mtime for f in files), default=0.0)


def build(jobs: int = 8, force: bool = False, verbose: bool = False, debug: bool = False) -> Path:
    bdir, lib = (BUILD_DEBUG, LIB_DEBUG) if debug else (BUILD, LIB)
    flags = FLAGS + (["-DSA_DEBUG_CHECKS"] if debug else [])
    bdir.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    hdr = _deps_mtime()
    nv = nvcc()

    def compile_one(src: Path):
        obj = bdir / (src.stem + ".o")
        if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr):
            return obj
        cmd = [nv, *ARCH, *flags, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        return obj

    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(compile_one, sources))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not lib.exists() or lib.stat().st_mtime < newest:
        tmp = lib.with_suffix(".so.tmp")
        cmd = [nv, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=os.cpu_count() or 4)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--debug", action="store_true", help="the library with device-side index checks")
    a = ap.parse_args()
    print(build(a.j, a.force, a.v, a.debug))
    sys.exit(0)
