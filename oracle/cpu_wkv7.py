"""ctypes front-ends for the two CPU WKV-7 implementations (test infrastructure).

* ``port_*`` : ``oracle/wkv7_metal_port.c`` -- our C restatement of the reference
  Metal kernels (``wkv7_metal.py:28-91``, ``:102-214``), OpenMP over (b, h).
* ``ref_*``  : the reference's own kernel bodies compiled for the CPU by
  ``oracle/build_ref.py`` into ``oracle/_ref/`` and launched the way
  ``wkv7_metal_forward`` / ``wkv7_metal_backward`` launch them
  (``wkv7_metal.py:250-279``, ``:282-319``): grid B*H*N threads, threadgroups of N.

Both take numpy arrays shaped (B, T, H, N) and return numpy arrays.
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
CHUNK = 16
N = 64

_port = None


def _load_port():
    global _port
    if _port is None:
        so = HERE / "libwkv7_port.so"
        if not so.exists():
            raise FileNotFoundError(f"{so} missing: run `make -C oracle`")
        lib = ctypes.CDLL(str(so))
        fp = ctypes.POINTER(ctypes.c_float)
        lib.wkv7_port_forward.argtypes = [fp] * 9 + [ctypes.c_int] * 3
        lib.wkv7_port_backward.argtypes = [fp] * 15 + [ctypes.c_int] * 3
        _port = lib
    return _port


def _f32(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def _p(x):
    return None if x is None else x.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def port_forward(r, w, k, v, a, b, want_states=True):
    """Returns (y, s, sa) like ``wkv7_metal_forward`` (s flat, per-16 snapshots)."""
    lib = _load_port()
    r, w, k, v, a, b = map(_f32, (r, w, k, v, a, b))
    B, T, H, n = r.shape
    assert n == N
    y = np.empty_like(r)
    s = np.empty(B * H * (T // CHUNK) * N * N, np.float32) if want_states else None
    sa = np.empty_like(r) if want_states else None
    lib.wkv7_port_forward(_p(r), _p(w), _p(k), _p(v), _p(a), _p(b), _p(y), _p(s), _p(sa), B, T, H)
    return y, s, sa


def port_backward(r, w, k, v, a, b, dy, s, sa):
    lib = _load_port()
    r, w, k, v, a, b, dy, s, sa = map(_f32, (r, w, k, v, a, b, dy, s, sa))
    B, T, H, n = r.shape
    outs = [np.empty_like(r) for _ in range(6)]
    lib.wkv7_port_backward(*[_p(x) for x in (r, w, k, v, a, b, dy, s, sa)], *[_p(o) for o in outs], B, T, H)
    return tuple(outs)


_ref = {}


def ref_available() -> bool:
    return (HERE / "_ref" / "manifest.json").exists()


def _ref_kernel(name):
    if name not in _ref:
        from oracle.metal_cpu import CpuMetalKernel

        man = json.loads((HERE / "_ref" / "manifest.json").read_text())
        _ref[name] = CpuMetalKernel(HERE / "_ref" / man["kernels"][name])
    return _ref[name]


def ref_forward(r, w, k, v, a, b):
    """The reference's forward body; dtype of r selects f32 or f16 (its template T)."""
    dt = np.dtype(r.dtype)
    tag = {np.dtype(np.float32): "f32", np.dtype(np.float16): "f16"}[dt]
    xs = [np.ascontiguousarray(x, dtype=dt) for x in (r, w, k, v, a, b)]
    B, T, H, n = xs[0].shape
    y = np.empty((B, T, H, n), dt)
    s = np.zeros(B * H * (T // CHUNK) * n * n, np.float32)
    sa = np.empty((B, T, H, n), np.float32)
    Hs, Ts = np.array([H], np.uint32), np.array([T], np.uint32)
    _ref_kernel(f"fwd_{tag}").launch(xs + [Hs, Ts], [y, s, sa], (B * H * n, 1, 1), (n, 1, 1))
    return y, s, sa


def ref_backward(r, w, k, v, a, b, dy, s, sa):
    dt = np.dtype(r.dtype)
    tag = {np.dtype(np.float32): "f32", np.dtype(np.float16): "f16"}[dt]
    xs = [np.ascontiguousarray(x, dtype=dt) for x in (r, w, k, v, a, b, dy)]
    B, T, H, n = xs[0].shape
    outs = [np.empty((B, T, H, n), dt) for _ in range(6)]
    Hs, Ts = np.array([H], np.uint32), np.array([T], np.uint32)
    _ref_kernel(f"bwd_{tag}").launch(
        xs + [_f32(s), _f32(sa), Hs, Ts], outs, (B * H * n, 1, 1), (n, 1, 1)
    )
    return tuple(outs)
