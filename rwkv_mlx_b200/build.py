"""Build the sm_100a C-ABI library ``rwkv_mlx_b200/_lib/librwkv_b200.so`` with nvcc.

``python -m rwkv_mlx_b200.build`` (or ``__graft_entry__.build()``).  Every ``.cu``
under ``csrc/`` is compiled for ``-gencode arch=compute_100a,code=sm_100a`` into
an object under ``_build/`` and linked into one shared library with the CUDA
runtime linked statically, so the library carries no dependency on the
torch-bundled runtime.  Rebuilds only what changed (sources or headers newer
than the object).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "_lib" / "librwkv_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def cflags(debug: bool = False):
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}", f"-I{CSRC}"]
    if debug:
        f += ["-DRWKV_DEBUG_CHECKS"]
    return f


def _headers():
    return list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))


def _compile(src: Path, debug: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    newest = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest:
        return obj
    cmd = [nvcc()] + cflags(debug) + ["-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr}")
    return obj


def build(verbose: bool = False, debug: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, debug), srcs))
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-Xcompiler", "-fPIC",
                                 "-o", str(tmp)] + [str(o) for o in objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(verbose=True, debug="--debug" in sys.argv)
