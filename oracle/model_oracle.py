"""CPU restatement of the RWKV-v7 model forward (test infrastructure + CPU baseline).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs
may use this.  It restates rwkv_mlx/model.py with torch CPU tensors:

  * ``forward``      : RWKV.__call__ (model.py:346-375) -> (logits, aux_loss), with
                       Block (:312-327), RWKV_Tmix_x070 (:182-240), RWKV_CMix_x070
                       (:259-263), LoRAMoE_CMix (moe.py:129-147) and MoE_CMix
                       (moe.py:226-242)
  * ``forward_rnn``  : RWKV.forward_rnn (model.py:377-421) with _time_mixing_rnn
                       (:441-495) and _channel_mixing_rnn (:498-506)

Weights are a dict keyed by the reference's parameter names (e.g.
``blocks.3.att.w1``, ``blocks.3.ffn.key.weight``).  The WKV-7 recurrence is the C
restatement of the reference Metal kernel (``oracle/wkv7_metal_port.c``, fp32), the
reference's own kernel body compiled for the CPU (``wkv="ref"``, ``oracle/_ref``) or
the float64 oracle (``wkv="exact"``).  ``ln_x`` uses MLX's GroupNorm grouping
(channels c = g mod H form group g) unless ``groupnorm="per_head"``.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import cpu_wkv7, moe_oracle, wkv7_oracle


def _lin(x, w):
    return x @ w.T


def _ln(x, w, b, eps=1e-5):
    m = x.mean(-1, keepdim=True)
    v = ((x - m) ** 2).mean(-1, keepdim=True)
    return (x - m) / torch.sqrt(v + eps) * w + b


def _groupnorm(x2d, G, w, b, eps, mode):
    n, C = x2d.shape
    xg = x2d.view(n, C // G, G) if mode == "mlx" else x2d.view(n, G, C // G)
    ax = 1 if mode == "mlx" else 2
    m = xg.mean(ax, keepdim=True)
    v = ((xg - m) ** 2).mean(ax, keepdim=True)
    y = ((xg - m) / torch.sqrt(v + eps)).reshape(n, C)
    return y * w + b


def _shift(x):
    out = torch.zeros_like(x)
    out[:, 1:] = x[:, :-1]
    return out


def _wkv(r, w, k, v, a, b, H, mode):
    B, T, C = r.shape
    sh = (B, T, H, C // H)
    args = [t.reshape(sh).numpy() for t in (r, w, k, v, a, b)]
    if mode == "exact":
        y = wkv7_oracle.wkv7_forward_exact(*args)[0]
    elif mode == "ref":  # the reference's own Metal kernel body, compiled for the CPU
        y = cpu_wkv7.ref_forward(*[x.astype(np.float32) for x in args])[0]
    else:
        y = cpu_wkv7.port_forward(*args, want_states=False)[0]
    return torch.from_numpy(np.ascontiguousarray(y)).to(r.dtype).reshape(B, T, C)


def _tmix(p, pre, x, v_first, layer_id, H, N, wkv, gn):
    B, T, C = x.shape
    g_ = lambda n: p[pre + n]
    xx = _shift(x) - x
    xr, xw, xk = x + xx * g_("x_r"), x + xx * g_("x_w"), x + xx * g_("x_k")
    xv, xa, xg = x + xx * g_("x_v"), x + xx * g_("x_a"), x + xx * g_("x_g")
    r = _lin(xr, g_("receptance.weight"))
    w = -F.softplus(-(g_("w0") + torch.tanh(xw @ g_("w1")) @ g_("w2"))) - 0.5
    k = _lin(xk, g_("key.weight"))
    v = _lin(xv, g_("value.weight"))
    if layer_id == 0:
        v_first = v
    else:
        v = v + (v_first - v) * torch.sigmoid(g_("v0") + (xv @ g_("v1")) @ g_("v2"))
    a = torch.sigmoid(g_("a0") + (xa @ g_("a1")) @ g_("a2"))
    g = torch.sigmoid(xg @ g_("g1")) @ g_("g2")
    kk = (k * g_("k_k")).reshape(B, T, H, N)
    kk = (kk / (torch.sqrt((kk * kk).sum(-1, keepdim=True)) + 1e-12)).reshape(B, T, C)
    k = k * (1 + (a - 1) * g_("k_a"))
    y = _wkv(r, w, k, v, -kk, kk * a, H, wkv)
    y = _groupnorm(y.reshape(B * T, C), H, g_("ln_x.weight"), g_("ln_x.bias"), 64e-5, gn).reshape(B, T, C)
    rh, kh, vh = r.reshape(B, T, H, N), k.reshape(B, T, H, N), v.reshape(B, T, H, N)
    y = y + ((rh * kh * g_("r_k")).sum(-1, keepdim=True) * vh).reshape(B, T, C)
    return _lin(y * g, g_("output.weight")), v_first


def _cmix(p, pre, x):
    xx = _shift(x) - x
    k = x + xx * p[pre + "x_k"]
    k = torch.relu(_lin(k, p[pre + "key.weight"])) ** 2
    return _lin(k, p[pre + "value.weight"])


def _lora_moe(p, pre, x, cfg):
    B, T, C = x.shape
    base = _cmix(p, pre + "base.", x)
    xn = x.reshape(B * T, C).double().numpy()
    inds, scores, aux, z, _ = moe_oracle.router(xn, p[pre + "router.gate.weight"].numpy(), cfg.moe_top_k)
    delta = moe_oracle.lora_moe_delta(xn, p[pre + "lora_A"].double().numpy(), p[pre + "lora_B"].double().numpy(),
                                      inds, scores)
    out = base + torch.from_numpy(delta).to(x.dtype).reshape(B, T, C)
    ortho = moe_oracle.orthogonal_loss(p[pre + "lora_A"].double().numpy())
    return out, aux, z, ortho


def _full_moe(p, pre, x, cfg):
    B, T, C = x.shape
    xn = x.reshape(B * T, C).double().numpy()
    inds, scores, aux, z, _ = moe_oracle.router(xn, p[pre + "router.gate.weight"].numpy(), cfg.moe_top_k)
    out = moe_oracle.full_moe(x.double().numpy(), p[pre + "x_k"].double().numpy(), p[pre + "expert_key"].double().numpy(),
                              p[pre + "expert_val"].double().numpy(), inds.reshape(B, T, -1), scores.reshape(B, T, -1))
    return torch.from_numpy(out).to(x.dtype), aux, z, 0.0  # no orthogonality loss (moe.py:241-242)


def _is_moe(cfg, i):
    return cfg.moe_num_experts > 0 and (not cfg.moe_layers or i in cfg.moe_layers)


def forward(p, cfg, idx, wkv="port", dtype=torch.float32, positions=None):
    """GPT-mode forward: idx (B, T) int -> (logits (B, T, V), aux_loss float).
    ``positions`` (optional index list): logits only at those positions (B, P, V)."""
    p = {k: v.to(dtype) for k, v in p.items()}
    H, N = cfg.n_head, cfg.head_size
    gn = getattr(cfg, "groupnorm", "mlx")
    x = p["emb.weight"][torch.as_tensor(idx)]
    v_first = torch.zeros_like(x)
    aux_total = 0.0
    for i in range(cfg.n_layer):
        pre = f"blocks.{i}."
        if i == 0:
            x = _ln(x, p[pre + "ln0.weight"], p[pre + "ln0.bias"])
        xa, v_first = _tmix(p, pre + "att.", _ln(x, p[pre + "ln1.weight"], p[pre + "ln1.bias"]), v_first, i, H, N, wkv, gn)
        x = x + xa
        x2 = _ln(x, p[pre + "ln2.weight"], p[pre + "ln2.bias"])
        if _is_moe(cfg, i):
            moe = _lora_moe if getattr(cfg, "moe_mode", "lora") == "lora" else _full_moe
            out, aux, z, ortho = moe(p, pre + "ffn.", x2, cfg)
            aux_total += cfg.moe_aux_loss_coeff * aux + cfg.moe_z_loss_coeff * z + cfg.moe_ortho_coeff * ortho
            x = x + out
        else:
            x = x + _cmix(p, pre + "ffn.", x2)
    if positions is not None:
        x = x[:, torch.as_tensor(positions)]
    x = _ln(x, p["ln_out.weight"], p["ln_out.bias"])
    return _lin(x, p["head.weight"]), aux_total


def init_state(cfg, dtype=torch.float64):
    st = []
    for _ in range(cfg.n_layer):
        st += [torch.zeros(cfg.n_embd, dtype=dtype), torch.zeros(cfg.n_head, cfg.head_size, cfg.head_size, dtype=dtype),
               torch.zeros(cfg.n_embd, dtype=dtype)]
    return st


def forward_rnn(p, cfg, token, state, dtype=torch.float64):
    """One RNN-mode token (model.py:377-421) for a plain (non-MoE) model."""
    p = {k: v.to(dtype) for k, v in p.items()}
    H, N = cfg.n_head, cfg.head_size
    gn = getattr(cfg, "groupnorm", "mlx")
    state = list(state)
    x = p["emb.weight"][int(token)]
    v_first = torch.zeros_like(x)
    lnv = lambda x, w, b: _ln(x, w, b)
    for i in range(cfg.n_layer):
        pre = f"blocks.{i}."
        if i == 0:
            x = lnv(x, p[pre + "ln0.weight"], p[pre + "ln0.bias"])
        xx = lnv(x, p[pre + "ln1.weight"], p[pre + "ln1.bias"])
        a_ = lambda n: p[pre + "att." + n].reshape(-1) if p[pre + "att." + n].dim() == 3 else p[pre + "att." + n]
        xp = state[3 * i]
        d = xp - xx
        xr, xw, xk = xx + d * a_("x_r"), xx + d * a_("x_w"), xx + d * a_("x_k")
        xv, xa, xg = xx + d * a_("x_v"), xx + d * a_("x_a"), xx + d * a_("x_g")
        r = a_("receptance.weight") @ xr
        w = torch.tanh(xw @ a_("w1")) @ a_("w2")
        k = a_("key.weight") @ xk
        v = a_("value.weight") @ xv
        a = torch.sigmoid(a_("a0") + (xa @ a_("a1")) @ a_("a2"))
        g = torch.sigmoid(xg @ a_("g1")) @ a_("g2")
        kk = (k * a_("k_k")).reshape(H, N)
        kk = (kk / (torch.sqrt((kk * kk).sum(-1, keepdim=True)) + 1e-12)).reshape(-1)
        k = k * (1 + (a - 1) * a_("k_a"))
        if i == 0:
            v_first = v
        else:
            v = v + (v_first - v) * torch.sigmoid(a_("v0") + (xv @ a_("v1")) @ a_("v2"))
        decay = torch.exp(-0.606531 * torch.sigmoid(a_("w0") + w))
        S = state[3 * i + 1]
        S = S * decay.reshape(H, 1, N) + S @ ((-kk).reshape(H, N, 1) @ (kk * a).reshape(H, 1, N)) \
            + v.reshape(H, N, 1) @ k.reshape(H, 1, N)
        out = (S @ r.reshape(H, N, 1)).reshape(-1)
        out = _groupnorm(out.reshape(1, -1), H, a_("ln_x.weight"), a_("ln_x.bias"), 64e-5, gn).reshape(-1)
        out = out + ((r * k * a_("r_k").reshape(-1)).reshape(H, N).sum(-1, keepdim=True) * v.reshape(H, N)).reshape(-1)
        x = x + a_("output.weight") @ (out * g)
        state[3 * i], state[3 * i + 1] = xx, S
        xx = lnv(x, p[pre + "ln2.weight"], p[pre + "ln2.bias"])
        f = lambda n: p[pre + "ffn." + n]
        d = state[3 * i + 2] - xx
        kf = xx + d * f("x_k").reshape(-1)
        kf = torch.relu(f("key.weight") @ kf) ** 2
        x = x + f("value.weight") @ kf
        state[3 * i + 2] = xx
    x = lnv(x, p["ln_out.weight"], p["ln_out.bias"])
    return p["head.weight"] @ x, state
