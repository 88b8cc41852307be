"""CPU oracle for the WKV-7 recurrence (test infrastructure, never the product).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this module, and only as the checker.

What it restates
----------------
The reference computes WKV-7 with a Metal kernel
(``rwkv_mlx/kernels/wkv7_metal.py:47-91`` forward, ``:116-214`` backward) and the
RNN-mode state update in ``rwkv_mlx/model.py:475-483``.  Per (batch, head) the
state ``S`` is an ``N x N`` fp32 matrix whose row ``i`` is the value index and
column ``j`` the key index.  One time step, in matrix form:

    decay = exp(-exp(w_t))                  (wkv7_metal.py:57)
    sa    = S @ a_t                         (wkv7_metal.py:63-66)
    S     = S * decay[None, :] + sa b_t^T + v_t k_t^T   (wkv7_metal.py:71-74)
    y_t   = S @ r_t                         (wkv7_metal.py:74, after the update)

``model.py:480-483`` is the same update written with ``state @ (a b^T)``; the decay
there is passed directly (``exp(-0.606531*sigmoid(.))``) instead of as log-log ``w``.

This module evaluates that recurrence in float64 with numpy, step by step, and
its exact reverse-mode derivative (stored states, no division by the decay).  The
reference's own backward reconstructs earlier states by dividing by the decay
(``wkv7_metal.py:174-178``), which is an approximation; the exact float64
derivative here is the target the CUDA backward is checked against, and the gap
to the reference's algorithm is measured separately with ``oracle/wkv7_metal_port.c``.

Pinning: ``tests/test_oracle_pins.py`` checks this module against golden vectors
produced by running the reference's own Metal kernel bodies (compiled as C++ on
the CPU by ``oracle/build_ref.py``) and the reference's own ``model.py`` /
``moe.py`` Python (``tests/golden/make_golden.py``).

Layout: every per-token tensor is ``(B, T, H, N)`` (the reference reshapes
``(B, T, C)`` to this at ``wkv7_metal.py:257-262``).  States are ``(B, H, N, N)``.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "wkv7_forward_exact",
    "wkv7_backward_exact",
    "wkv7_step_exact",
    "checkpoints_from_states",
]


def _as64(x):
    return np.asarray(x, dtype=np.float64)


def wkv7_forward_exact(r, w, k, v, a, b, s0=None, w_is_decay=False, keep_states=False):
    """Sequential float64 WKV-7 forward.

    Args: ``r, w, k, v, a, b`` of shape (B, T, H, N). ``w`` is the log-log decay
    (decay = exp(-exp(w))) unless ``w_is_decay``. ``s0`` optional (B, H, N, N).

    Returns ``(y, sa, sT, states)``: y and sa (B, T, H, N); sT (B, H, N, N);
    states (B, H, T+1, N, N) when ``keep_states`` (states[:, :, t] is the state
    *before* step t, states[:, :, T] the final one), else None.
    """
    r, w, k, v, a, b = map(_as64, (r, w, k, v, a, b))
    B, T, H, N = r.shape
    decay = w if w_is_decay else np.exp(-np.exp(w))
    S = np.zeros((B, H, N, N)) if s0 is None else _as64(s0).copy()
    y = np.zeros((B, T, H, N))
    sa = np.zeros((B, T, H, N))
    states = np.zeros((B, H, T + 1, N, N)) if keep_states else None
    for t in range(T):
        if keep_states:
            states[:, :, t] = S
        at = a[:, t]  # (B, H, N)
        u = np.einsum("bhij,bhj->bhi", S, at)
        S = (S * decay[:, t][:, :, None, :]
             + u[..., :, None] * b[:, t][:, :, None, :]
             + v[:, t][..., :, None] * k[:, t][:, :, None, :])
        sa[:, t] = u
        y[:, t] = np.einsum("bhij,bhj->bhi", S, r[:, t])
    if keep_states:
        states[:, :, T] = S
    return y, sa, S, states


def wkv7_backward_exact(r, w, k, v, a, b, dy, s0=None, dsT=None):
    """Exact float64 reverse-mode derivative of :func:`wkv7_forward_exact`.

    Returns ``(dr, dw, dk, dv, da, db, ds0)``. ``dw`` is with respect to the
    log-log ``w`` input, i.e. includes d decay / d w = decay * (-exp(w)) as the
    reference does at ``wkv7_metal.py:192-193``.
    """
    r, w, k, v, a, b, dy = map(_as64, (r, w, k, v, a, b, dy))
    B, T, H, N = r.shape
    decay = np.exp(-np.exp(w))
    _, sa, _, states = wkv7_forward_exact(r, w, k, v, a, b, s0=s0, keep_states=True)
    G = np.zeros((B, H, N, N)) if dsT is None else _as64(dsT).copy()
    out = {n: np.zeros((B, T, H, N)) for n in ("dr", "dw", "dk", "dv", "da", "db")}
    for t in range(T - 1, -1, -1):
        S_prev = states[:, :, t]
        S_t = states[:, :, t + 1]
        G = G + dy[:, t][..., :, None] * r[:, t][:, :, None, :]
        out["dr"][:, t] = np.einsum("bhij,bhi->bhj", S_t, dy[:, t])
        out["dv"][:, t] = np.einsum("bhij,bhj->bhi", G, k[:, t])
        out["dk"][:, t] = np.einsum("bhij,bhi->bhj", G, v[:, t])
        du = np.einsum("bhij,bhj->bhi", G, b[:, t])
        out["db"][:, t] = np.einsum("bhij,bhi->bhj", G, sa[:, t])
        dD = np.einsum("bhij,bhij->bhj", S_prev, G)
        out["dw"][:, t] = dD * decay[:, t] * (-np.exp(w[:, t]))
        out["da"][:, t] = np.einsum("bhij,bhi->bhj", S_prev, du)
        G = G * decay[:, t][:, :, None, :] + du[..., :, None] * a[:, t][:, :, None, :]
    return (out["dr"], out["dw"], out["dk"], out["dv"], out["da"], out["db"], G)


def wkv7_step_exact(S, r, w, k, v, a, b, w_is_decay=True):
    """One RNN-mode step for a batch of sequences (``model.py:480-483``).

    ``S`` (Bs, H, N, N); vectors (Bs, H, N). Returns ``(y, S_new)`` in float64.
    """
    S, r, w, k, v, a, b = map(_as64, (S, r, w, k, v, a, b))
    decay = w if w_is_decay else np.exp(-np.exp(w))
    u = np.einsum("bhij,bhj->bhi", S, a)
    S = S * decay[:, :, None, :] + u[..., :, None] * b[:, :, None, :] + v[..., :, None] * k[:, :, None, :]
    y = np.einsum("bhij,bhj->bhi", S, r)
    return y, S


def checkpoints_from_states(states, ckpt_len):
    """States after steps ckpt_len, 2*ckpt_len, ... as (B, H, T//ckpt_len, N, N).

    Matches the snapshot rule of ``wkv7_metal.py:80-89``: a snapshot is written after
    step t whenever (t + 1) % ckpt_len == 0.
    """
    T = states.shape[2] - 1
    idx = [c * ckpt_len for c in range(1, T // ckpt_len + 1)]
    return states[:, :, idx]
