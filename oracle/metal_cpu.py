"""Compile and run an ``mx.fast.metal_kernel`` body on the CPU (test infrastructure).

Only tests, the fixture generator and ``oracle/build_ref.py`` use this.  Given a
kernel body written for ``mx.fast.metal_kernel`` (the MLX API the reference uses
at ``rwkv_mlx/kernels/wkv7_metal.py:223-247``), its input/output names and the
dtypes, it writes a C++ translation unit that wraps the body with the
``oracle/metal_shim.hpp`` stand-ins, compiles it with g++ and launches it with
one std::thread per Metal thread of a threadgroup.

The kernel signature follows what ``mx.fast.metal_kernel`` generates: each input
is ``const device <dtype>* name`` and each output ``device <dtype>* name``, in the
order given, and the template parameter ``T`` is a typedef.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

_CTYPE = {
    np.dtype(np.float32): "float",
    np.dtype(np.float16): "half",
    np.dtype(np.uint32): "uint",
    np.dtype(np.int32): "int",
}


def _ctype(dt) -> str:
    dt = np.dtype(dt)
    if dt not in _CTYPE:
        raise TypeError(f"metal_cpu: unsupported dtype {dt}")
    return _CTYPE[dt]


def generate_tu(source: str, in_names, in_dtypes, out_names, out_dtypes, template_T=None) -> str:
    params = [f"const {_ctype(d)}* __restrict {n}" for n, d in zip(in_names, in_dtypes)]
    params += [f"{_ctype(d)}* __restrict {n}" for n, d in zip(out_names, out_dtypes)]
    unpack = [f"(const {_ctype(d)}*)ins[{i}]" for i, d in enumerate(in_dtypes)]
    unpack += [f"({_ctype(d)}*)outs[{i}]" for i, d in enumerate(out_dtypes)]
    tdef = f"typedef {_ctype(template_T)} T;\n" if template_T is not None else ""
    return (
        '#include "metal_shim.hpp"\n'
        f"{tdef}"
        f"static void kernel_body({', '.join(params)}) {{\n{source}\n}}\n"
        'extern "C" void mtl_launch(void** ins, void** outs, unsigned gx, unsigned gy, '
        "unsigned gz, unsigned tx, unsigned ty, unsigned tz) {\n"
        "  mtl_dispatch(gx, gy, gz, tx, ty, tz, [=]() { kernel_body("
        + ", ".join(unpack)
        + "); });\n}\n"
    )


def compile_tu(tu: str, out_dir: Path, stem: str) -> Path:
    out_dir.mkdir(parents=True, exist_ok=True)
    h = hashlib.sha256(tu.encode()).hexdigest()[:12]
    so = out_dir / f"{stem}_{h}.so"
    if so.exists():
        return so
    src = out_dir / f"{stem}_{h}.cpp"
    src.write_text(tu)
    cmd = ["g++", "-std=c++20", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-pthread",
           f"-I{HERE}", str(src), "-o", str(so) + ".tmp"]
    subprocess.run(cmd, check=True, capture_output=True)
    os.replace(str(so) + ".tmp", so)
    return so


class CpuMetalKernel:
    """A compiled kernel body; call with numpy arrays like mx.fast.metal_kernel."""

    def __init__(self, so_path: Path):
        self._lib = ctypes.CDLL(str(so_path))
        self._fn = self._lib.mtl_launch
        self._fn.restype = None
        self._fn.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)] + [ctypes.c_uint] * 6

    def launch(self, inputs, outputs, grid, threadgroup):
        ins = [np.ascontiguousarray(x) for x in inputs]
        for o in outputs:
            assert o.flags["C_CONTIGUOUS"]
        in_ptrs = (ctypes.c_void_p * max(1, len(ins)))(*[x.ctypes.data for x in ins])
        out_ptrs = (ctypes.c_void_p * max(1, len(outputs)))(*[o.ctypes.data for o in outputs])
        g = tuple(grid) + (1,) * (3 - len(grid))
        t = tuple(threadgroup) + (1,) * (3 - len(threadgroup))
        self._fn(in_ptrs, out_ptrs, *g, *t)
        return outputs


def build_kernel(source, in_names, in_dtypes, out_names, out_dtypes, template_T, out_dir, stem):
    tu = generate_tu(source, in_names, in_dtypes, out_names, out_dtypes, template_T)
    return compile_tu(tu, Path(out_dir), stem)
