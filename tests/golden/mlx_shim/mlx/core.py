"""mlx.core stand-in (numpy).  Fixture generation only."""

import sys
from pathlib import Path

import numpy as np

float32 = np.float32
float16 = np.float16
uint32 = np.uint32
int32 = np.int32


def array(x, dtype=None):
    a = np.array(x)
    if dtype is not None:
        a = a.astype(dtype)
    elif a.dtype == np.float64:
        a = a.astype(np.float32)  # MLX's default float type
    elif a.dtype == np.int64:
        a = a.astype(np.int32)
    return a


def zeros(shape, dtype=np.float32):
    return np.zeros(shape, dtype)


def zeros_like(x):
    return np.zeros_like(x)


def full(shape, val, dtype=None):
    return np.full(shape, val, dtype or np.float32)


def concatenate(xs, axis=0):
    return np.concatenate(xs, axis=axis)


def stack(xs, axis=0):
    return np.stack(xs, axis=axis)


sqrt, tanh, exp, log, maximum, where = np.sqrt, np.tanh, np.exp, np.log, np.maximum, np.where


def sigmoid(x):
    return (1.0 / (1.0 + np.exp(-x))).astype(x.dtype)


def softmax(x, axis=-1):
    m = x.max(axis=axis, keepdims=True)
    e = np.exp(x - m)
    return (e / e.sum(axis=axis, keepdims=True)).astype(x.dtype)


def argpartition(a, kth, axis=-1):
    return np.argpartition(a, kth, axis=axis).astype(np.uint32)


def take_along_axis(a, idx, axis):
    return np.take_along_axis(a, idx.astype(np.int64), axis=axis)


def save_safetensors(path, arrays):
    from safetensors.numpy import save_file

    save_file({k: np.ascontiguousarray(v) for k, v in arrays.items()}, str(path))


def load(path):
    from safetensors.numpy import load_file

    return load_file(str(path))


def stop_gradient(x):
    return x


def eval(*args, **kwargs):
    return None


class _Random:
    _rng = np.random.default_rng(0)

    def normal(self, shape=(), dtype=np.float32, loc=0.0, scale=1.0):
        return (self._rng.standard_normal(shape) * scale + loc).astype(dtype)

    def uniform(self, low=0.0, high=1.0, shape=(), dtype=np.float32):
        return self._rng.uniform(low, high, shape).astype(dtype)


random = _Random()


class custom_function:
    """mx.custom_function: forward call only (the VJP is recorded, not used)."""

    def __init__(self, fn):
        self.fn = fn
        self.vjp_fn = None

    def __call__(self, *args):
        return self.fn(*args)

    def vjp(self, fn):
        self.vjp_fn = fn
        return fn


class _Fast:
    def metal_kernel(self, name, input_names, output_names, source, **_):
        return _CpuMetalKernel(name, input_names, output_names, source)


fast = _Fast()


class _CpuMetalKernel:
    """Runs the Metal kernel body on the CPU via oracle/metal_cpu.py."""

    def __init__(self, name, input_names, output_names, source):
        self.name, self.inn, self.outn, self.src = name, input_names, output_names, source

    def __call__(self, inputs, template, grid, threadgroup, output_shapes, output_dtypes, **_):
        root = Path(__file__).resolve().parents[4]
        sys.path.insert(0, str(root))
        from oracle.metal_cpu import CpuMetalKernel, build_kernel

        T = dict(template)["T"]
        ins = [np.ascontiguousarray(x) for x in inputs]
        so = build_kernel(self.src, self.inn, [x.dtype for x in ins], self.outn, list(output_dtypes), T,
                          root / "_build" / "metal_cpu", self.name)
        outs = [np.zeros(s, d) for s, d in zip(output_shapes, output_dtypes)]
        CpuMetalKernel(so).launch(ins, outs, grid, threadgroup)
        return outs
