"""CPU oracle for the LoRA-MoE ChannelMix path (test infrastructure, never the product).

Restates rwkv_mlx/moe.py in numpy (float64 unless stated):
  * ``router``          : Router.__call__            (moe.py:51-86)
  * ``topk_from_logits``: the top-k of moe.py:66-68 with the order pinned to
                          (logit descending, expert id ascending); argpartition
                          itself leaves slot order and ties unspecified
  * ``lora_moe``        : LoRAMoE_CMix.__call__ delta (moe.py:129-147), dense over
                          experts exactly as the reference loops
  * ``orthogonal_loss`` : LoRAMoE_CMix.orthogonal_loss (moe.py:149-163)
  * ``full_moe``        : MoE_CMix.__call__ output (moe.py:226-242), dense over the
                          E full experts exactly as the reference loops
  * ``full_moe_step``   : one RNN-mode token through the same experts (the
                          reference's forward_rnn has no MoE branch; this applies
                          _channel_mixing_rnn, model.py:498-506, per expert)
  * ``cmix``            : RWKV_CMix_x070.__call__ (model.py:259-263), the frozen base

Pinned against the reference's own moe.py / model.py code by
``tests/test_oracle_pins.py`` (golden vectors from ``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import numpy as np


def gate_logits(x, gate_w, bias=None):
    """fp32 logits = x.astype(f32) @ W^T (moe.py:56), computed in float64."""
    lg = np.asarray(x, np.float32).astype(np.float64) @ np.asarray(gate_w, np.float32).astype(np.float64).T
    if bias is not None:
        lg = lg + np.asarray(bias, np.float32).astype(np.float64)
    return lg


def topk_from_logits(logits, k):
    """Indices (..., k): logit descending, ties to the lower expert id."""
    lg = np.asarray(logits)
    E = lg.shape[-1]
    flat = lg.reshape(-1, E)
    ids = np.broadcast_to(np.arange(E), flat.shape)
    order = np.lexsort((ids, -flat), axis=-1)  # primary: -logit, secondary: id
    return order[:, :k].reshape(lg.shape[:-1] + (k,))


def router(x, gate_w, top_k, bias=None, logits=None):
    """Returns (inds, scores, aux, z) like moe.py:86 (inds int64, scores float64).

    ``logits`` may be supplied (e.g. the GPU's fp32 logits) so that routing is
    compared on identical inputs."""
    lg = gate_logits(x, gate_w, bias) if logits is None else np.asarray(logits, np.float64)
    E = lg.shape[-1]
    lse = np.log(np.exp(lg).sum(-1))                       # moe.py:61
    z = float((lse ** 2).mean())                           # moe.py:62
    inds = topk_from_logits(lg, top_k)                     # moe.py:66-68
    sel = np.take_along_axis(lg, inds, -1)                 # moe.py:69
    sc = np.exp(sel - sel.max(-1, keepdims=True))
    scores = sc / sc.sum(-1, keepdims=True)                # moe.py:70
    probs = np.exp(lg - lg.max(-1, keepdims=True))
    probs = probs / probs.sum(-1, keepdims=True)           # moe.py:76
    p_e = probs.reshape(-1, E).mean(0)                     # moe.py:77-78
    flat = inds.reshape(-1, top_k)
    f_e = np.array([(flat == e).astype(np.float64).mean() for e in range(E)])  # moe.py:80-82
    aux = float(E * (f_e * p_e).sum())                     # moe.py:84
    return inds, scores, aux, z, f_e


def lora_moe_delta(x, A, B, inds, scores):
    """sum_e w_e * ((x @ A_e) @ B_e), w_e = sum_slots where(inds == e, scores, 0)."""
    x = np.asarray(x, np.float64)
    out = np.zeros(x.shape[:-1] + (B.shape[-1],))
    for e in range(A.shape[0]):
        adapter = (x @ np.asarray(A[e], np.float64)) @ np.asarray(B[e], np.float64)
        w_e = np.where(inds == e, scores, 0.0).sum(-1, keepdims=True)
        out = out + w_e * adapter
    return out


def orthogonal_loss(A):
    A = np.asarray(A, np.float64)
    tot = 0.0
    for i in range(A.shape[0]):
        for j in range(i + 1, A.shape[0]):
            cross = A[i].T @ A[j]
            tot += float((cross * cross).sum())
    return tot


def time_shift(x):
    """(B, T, C): prepend a zero row, drop the last (model.py:67-75)."""
    out = np.zeros_like(x)
    out[:, 1:] = x[:, :-1]
    return out


def cmix(x, x_k, key_w, value_w):
    """RWKV_CMix_x070 (model.py:259-263); key_w (F, C), value_w (C, F)."""
    x = np.asarray(x, np.float64)
    xx = time_shift(x) - x
    kin = x + xx * np.asarray(x_k, np.float64).reshape(1, 1, -1)
    k = np.maximum(kin @ np.asarray(key_w, np.float64).T, 0.0) ** 2
    return k @ np.asarray(value_w, np.float64).T


def full_moe(x, x_k, key, val, inds, scores):
    """MoE_CMix output (moe.py:226-242) for x (B, T, C): per expert e,
    k_e = x + (shift(x) - x) * x_k[e]; out_e = relu(k_e @ key[e]^T)^2 @ val[e]^T;
    out = sum_e w_e * out_e with w_e = sum_slots where(inds == e, scores, 0).
    x_k (E, 1, 1, C), key (E, D, C), val (E, C, D); inds / scores (B, T, k)."""
    x = np.asarray(x, np.float64)
    xx = time_shift(x) - x
    out = np.zeros_like(x)
    for e in range(key.shape[0]):
        ke = x + xx * np.asarray(x_k[e], np.float64).reshape(1, 1, -1)
        ke = np.maximum(ke @ np.asarray(key[e], np.float64).T, 0.0) ** 2
        oe = ke @ np.asarray(val[e], np.float64).T
        w_e = np.where(inds == e, scores, 0.0).sum(-1, keepdims=True)
        out = out + w_e * oe
    return out


def full_moe_step(x, x_prev, x_k, key, val, inds, scores):
    """One token per row: x, x_prev (n, C); inds / scores (n, k)."""
    x = np.asarray(x, np.float64)
    d = np.asarray(x_prev, np.float64) - x
    out = np.zeros_like(x)
    for e in range(key.shape[0]):
        ke = x + d * np.asarray(x_k[e], np.float64).reshape(1, -1)
        oe = np.maximum(ke @ np.asarray(key[e], np.float64).T, 0.0) ** 2 @ np.asarray(val[e], np.float64).T
        out = out + np.where(inds == e, scores, 0.0).sum(-1, keepdims=True) * oe
    return out
