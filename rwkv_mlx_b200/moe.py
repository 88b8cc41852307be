"""LoRA-MoE ChannelMix with the reference's module interface, on the sm_100a kernels.

Reference (rwkv_mlx/moe.py):
  * ``Router(d_model, n_experts, top_k)(x) -> (inds, weights, aux_loss, z_loss)``
    (:35-86)                                              -> :class:`Router`
  * ``LoRAMoE_CMix(base, n_experts, lora_rank, top_k)(x) -> (out, aux, z)`` and
    ``.orthogonal_loss()`` (:93-163)                      -> :class:`LoRAMoE_CMix`

The reference evaluates every expert densely for every token and masks the
result (moe.py:138-145).  Here the routed (token, slot) entries are sorted by
expert with a stable counting sort (``rwkv_moe_permute``), the rank-r
down-projection runs per expert group (``rwkv_moe_lora_down``) and the
up-projection, score weighting and residual add are fused in one combine pass
(``rwkv_moe_lora_combine``).  Top-k ties go to the lower expert id; slots are in
descending logit order (the reference's argpartition leaves both unspecified).

These modules compute the forward pass only (no autograd through the kernels).
"""

from __future__ import annotations

import torch
from torch import nn

from . import _native as nat


def _stream(dev):
    return nat.stream_ptr(dev)


def router_forward(x2d: torch.Tensor, gate_w: torch.Tensor, top_k: int, bias=None,
                   want_logits: bool = False):
    """Route ``x2d`` (ntok, C).  Returns dict with inds (ntok, k) int32, scores
    (ntok, k) x.dtype, aux, z (0-d fp32), f (E,), counts (E,) int32, logits."""
    ntok, C = x2d.shape
    E = gate_w.shape[0]
    dev = x2d.device
    x2d = x2d.contiguous()
    gw = gate_w.to(torch.float32).contiguous()
    b = None if bias is None else bias.to(torch.float32).contiguous()
    inds = torch.empty((ntok, top_k), device=dev, dtype=torch.int32)
    scores = torch.empty((ntok, top_k), device=dev, dtype=x2d.dtype)
    stats = torch.empty(2 + E, device=dev, dtype=torch.float32)
    counts = torch.empty(E, device=dev, dtype=torch.int32)
    logits = torch.empty((ntok, E), device=dev, dtype=torch.float32) if want_logits else None
    L = nat.lib()
    ws_bytes = L.rwkv_moe_router_workspace_size(ntok, E)
    ws = torch.empty(max(1, ws_bytes), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        rc = L.rwkv_moe_router(nat.ptr(x2d), nat.ptr(gw), nat.ptr(b), nat.ptr(logits),
                               nat.ptr(inds), nat.ptr(scores), nat.ptr(stats), nat.ptr(counts),
                               nat.ptr(ws), ws_bytes, ntok, C, E, top_k, nat.dtype_code(x2d),
                               _stream(dev))
    nat.check(rc, "rwkv_moe_router")
    return {"inds": inds, "scores": scores, "aux": stats[0], "z": stats[1], "f": stats[2:],
            "counts": counts, "logits": logits}


def permute(inds: torch.Tensor, E: int):
    """Stable sort of the routing entries by expert -> (perm, inv, offsets)."""
    ntok, k = inds.shape
    dev = inds.device
    inds = inds.to(torch.int32).contiguous()
    n = ntok * k
    perm = torch.empty(n, device=dev, dtype=torch.int32)
    inv = torch.empty(n, device=dev, dtype=torch.int32)
    offsets = torch.empty(E + 1, device=dev, dtype=torch.int32)
    L = nat.lib()
    ws_bytes = L.rwkv_moe_permute_workspace_size(n, E)
    ws = torch.empty(max(1, ws_bytes), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        rc = L.rwkv_moe_permute(nat.ptr(inds), nat.ptr(perm), nat.ptr(inv), nat.ptr(offsets),
                                nat.ptr(ws), ws_bytes, ntok, k, E, _stream(dev))
    nat.check(rc, "rwkv_moe_permute")
    return perm, inv, offsets


def lora_down(x2d, A, perm, offsets, top_k):
    ntok, C = x2d.shape
    E, _, R = A.shape
    h = torch.empty((ntok * top_k, R), device=x2d.device, dtype=torch.float32)
    A = A.to(x2d.dtype).contiguous()
    L = nat.lib()
    with torch.cuda.device(x2d.device):
        rc = L.rwkv_moe_lora_down(nat.ptr(x2d), nat.ptr(A), nat.ptr(perm), nat.ptr(offsets),
                                  nat.ptr(h), ntok, C, R, E, top_k, nat.dtype_code(x2d),
                                  _stream(x2d.device))
    nat.check(rc, "rwkv_moe_lora_down")
    return h


def lora_combine(base2d, h, Bw, inds, scores, inv, out=None):
    ntok, k = inds.shape
    E, R, C = Bw.shape
    dt = scores.dtype
    if out is None:
        out = torch.empty((ntok, C), device=h.device, dtype=dt)
    Bw = Bw.to(dt).contiguous()
    base2d = None if base2d is None else base2d.to(dt).contiguous()
    L = nat.lib()
    with torch.cuda.device(h.device):
        rc = L.rwkv_moe_lora_combine(nat.ptr(base2d), nat.ptr(h), nat.ptr(Bw), nat.ptr(inds),
                                     nat.ptr(scores), nat.ptr(inv), nat.ptr(out), ntok, C, R, E,
                                     k, nat.dtype_code(out), _stream(h.device))
    nat.check(rc, "rwkv_moe_lora_combine")
    return out


def lora_apply_supported(C: int, R: int, E: int, top_k: int, dtype: torch.dtype) -> bool:
    return bool(nat.lib().rwkv_moe_lora_apply_supported(C, R, E, top_k, nat.dtype_code_of(dtype)))


def lora_apply(x2d, base2d, A, Bw, inds, scores, out=None):
    """out = base + sum_s scores[:, s] * (x @ A[e]) @ B[e] in one fused pass (moe.py:142-147)."""
    ntok, C = x2d.shape
    E, _, R = A.shape
    k = inds.shape[1]
    dt = x2d.dtype
    if out is None:
        out = torch.empty((ntok, C), device=x2d.device, dtype=dt)
    A = A.to(dt).contiguous()
    Bw = Bw.to(dt).contiguous()
    base2d = None if base2d is None else base2d.to(dt).contiguous()
    scores = None if scores is None else scores.to(dt).contiguous()
    L = nat.lib()
    with torch.cuda.device(x2d.device):
        rc = L.rwkv_moe_lora_apply(nat.ptr(x2d.contiguous()), nat.ptr(base2d), nat.ptr(A), nat.ptr(Bw),
                                   nat.ptr(inds.contiguous()), nat.ptr(scores), nat.ptr(out), ntok, C, R, E, k,
                                   nat.dtype_code(out), _stream(x2d.device))
    nat.check(rc, "rwkv_moe_lora_apply")
    return out


def ortho_loss(A: torch.Tensor) -> torch.Tensor:
    E, C, R = A.shape
    A = A.contiguous()
    out = torch.empty((), device=A.device, dtype=torch.float32)
    L = nat.lib()
    with torch.cuda.device(A.device):
        rc = L.rwkv_moe_ortho_loss(nat.ptr(A), nat.ptr(out), E, C, R, nat.dtype_code(A),
                                   _stream(A.device))
    nat.check(rc, "rwkv_moe_ortho_loss")
    return out


class Router(nn.Module):
    """Token router (moe.py:35-86): linear gate in fp32 -> top-k + aux losses.

    ``bias`` (optional, (E,) fp32) is added to the logits; the reference router has
    none (moe.py:47) and the default keeps it that way."""

    def __init__(self, d_model: int, n_experts: int, top_k: int = 2):
        super().__init__()
        self.gate = nn.Linear(d_model, n_experts, bias=False)
        self.n_experts = n_experts
        self.top_k = top_k
        self.bias = None

    def forward(self, x: torch.Tensor):
        B, T, C = x.shape
        r = router_forward(x.reshape(B * T, C), self.gate.weight, self.top_k, self.bias)
        return (r["inds"].reshape(B, T, self.top_k), r["scores"].reshape(B, T, self.top_k),
                r["aux"], r["z"])


class LoRAMoE_CMix(nn.Module):
    """ChannelMix with LoRA expert adapters on a shared frozen base (moe.py:93-163).

    out = base(x) + sum_{selected e} score_e * ((x @ A_e) @ B_e)."""

    def __init__(self, base: nn.Module, n_experts: int, lora_rank: int, top_k: int = 2):
        super().__init__()
        self.base = base
        self.n_experts = n_experts
        self.lora_rank = lora_rank
        self.top_k = top_k
        C = base.key.weight.shape[1]
        # same parameter layout and init as moe.py:122-125
        self.lora_A = nn.Parameter(torch.randn(n_experts, C, lora_rank) * 0.01)
        self.lora_B = nn.Parameter(torch.zeros(n_experts, lora_rank, C))
        self.router = Router(C, n_experts, top_k)

    def forward(self, x: torch.Tensor):
        B, T, C = x.shape
        with torch.no_grad():
            base_out = self.base(x)
        x2 = x.reshape(B * T, C).contiguous()
        r = router_forward(x2, self.router.gate.weight, self.top_k, self.router.bias)
        if lora_apply_supported(C, self.lora_rank, self.n_experts, self.top_k, x.dtype):
            out = lora_apply(x2, base_out.reshape(B * T, C), self.lora_A.detach(), self.lora_B.detach(),
                             r["inds"], r["scores"])
        else:  # sorted dispatch: grouped down-projection, then per-token combine
            perm, inv, offsets = permute(r["inds"], self.n_experts)
            h = lora_down(x2, self.lora_A.detach(), perm, offsets, self.top_k)
            out = lora_combine(base_out.reshape(B * T, C), h, self.lora_B.detach(), r["inds"],
                               r["scores"], inv)
        return out.reshape(B, T, C), r["aux"], r["z"]

    def orthogonal_loss(self) -> torch.Tensor:
        return ortho_loss(self.lora_A.detach())
