"""Deterministic random parameters for the golden-vector models.

Given the reference's parameter names and shapes (stored in the fixture), draws the
same values the fixture generator used, so the fixture stores names, shapes and a
SHA-256 of the values instead of the values themselves."""

import hashlib

import numpy as np


def random_params(spec, seed):
    """spec: list of (name, shape) in generation order -> {name: float32 array}."""
    rng = np.random.default_rng(seed)
    out = {}
    for n, shape in spec:
        shape = tuple(int(s) for s in shape)
        last = n.split(".")[-1]
        owner = n.split(".")[-2] if "." in n else ""
        if n.endswith("emb.weight"):
            x = rng.standard_normal(shape)
        elif last == "w0":
            x = rng.uniform(-5.0, -0.5, shape)
        elif "ln" in owner and last == "weight":
            x = 1.0 + 0.1 * rng.standard_normal(shape)
        elif last == "bias":
            x = 0.1 * rng.standard_normal(shape)
        elif last in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g"):
            x = rng.uniform(0, 1, shape)
        elif last == "k_a":
            x = 1.0 + 0.05 * rng.standard_normal(shape)
        elif len(shape) >= 2:
            x = rng.standard_normal(shape) / np.sqrt(shape[-1] if len(shape) == 2 else shape[-2])
        else:
            x = 0.3 * rng.standard_normal(shape)
        if last in ("lora_A", "lora_B"):
            x = x * 0.5
        out[n] = x.astype(np.float32)
    return out


def params_sha256(params):
    h = hashlib.sha256()
    for n in sorted(params):
        h.update(n.encode())
        h.update(np.ascontiguousarray(params[n], np.float32).tobytes())
    return np.frombuffer(h.digest(), np.uint8)


def spec_arrays(spec):
    names = np.array([n for n, _ in spec])
    shapes = np.zeros((len(spec), 4), np.int64)
    for i, (_, s) in enumerate(spec):
        shapes[i, : len(s)] = s
        shapes[i, len(s):] = -1
    return names, shapes


def spec_from_arrays(names, shapes):
    return [(str(n), tuple(int(x) for x in s if x >= 0)) for n, s in zip(names, shapes)]


RESHAPE_1D = {"x_r", "x_w", "x_k", "x_v", "x_a", "x_g", "w0", "a0", "v0", "k_k", "k_a"}


def pth_state_dict(spec, seed):
    """A PyTorch-layout RWKV-7 state dict for the model spec: the values of
    random_params(spec, seed), mixing vectors and biases of shape (1, 1, C) stored
    1-D, and layer 0 without att.v0 / v1 / v2 (the layout convert.py reads)."""
    import torch

    P = random_params(spec, seed)
    sd = {}
    for n, v in P.items():
        if n in ("blocks.0.att.v0", "blocks.0.att.v1", "blocks.0.att.v2"):
            continue
        if n.split(".")[-1] in RESHAPE_1D and v.ndim == 3:
            v = v.reshape(-1)
        sd[n] = torch.tensor(v)
    return sd
