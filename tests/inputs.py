"""Seeded synthetic inputs with the shapes and distributions of the benchmark configs.

WKV-7 op (config 1): r, k, v ~ N(0,1); w ~ U(-6, -0.5) (decay = exp(-exp(w)));
kk = L2-normalised N(0,1) per head; a = -kk; b = kk * sigmoid(N(0,1)); dy ~ N(0,1).
Drawn with numpy's PCG64 in the order r, w, k, v, kk, iclr, dy.
"""

import numpy as np


def wkv_inputs(B, T, H, seed=0, N=64, w_lo=-6.0, w_hi=-0.5):
    rng = np.random.default_rng(seed)
    shp = (B, T, H, N)
    r = rng.standard_normal(shp)
    w = rng.uniform(w_lo, w_hi, shp)
    k = rng.standard_normal(shp)
    v = rng.standard_normal(shp)
    kk = rng.standard_normal(shp)
    kk = kk / np.linalg.norm(kk, axis=-1, keepdims=True)
    iclr = 1.0 / (1.0 + np.exp(-rng.standard_normal(shp)))
    dy = rng.standard_normal(shp)
    a = -kk
    b = kk * iclr
    return {"r": r, "w": w, "k": k, "v": v, "a": a, "b": b, "dy": dy}


def rel_rms(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.sqrt(np.mean(ref ** 2))
    return float(np.sqrt(np.mean((x - ref) ** 2)) / max(den, 1e-30))


def router_x(ntok, C, seed):
    """Router inputs of BASELINE configs[3]: x ~ N(0, 1) as fp16, (ntok, C)."""
    return np.random.default_rng(seed).standard_normal((ntok, C)).astype(np.float16)
