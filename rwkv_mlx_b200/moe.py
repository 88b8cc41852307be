"""LoRA-MoE ChannelMix with the reference's module interface, on the sm_100a kernels.

Reference (rwkv_mlx/moe.py):
  * ``Router(d_model, n_experts, top_k)(x) -> (inds, weights, aux_loss, z_loss)``
    (:35-86)                                              -> :class:`Router`
  * ``LoRAMoE_CMix(base, n_experts, lora_rank, top_k)(x) -> (out, aux, z)`` and
    ``.orthogonal_loss()`` (:93-163)                      -> :class:`LoRAMoE_CMix`
  * ``MoE_CMix(config, layer_id, n_experts, top_k)(x) -> (out, aux, z)`` and
    ``.orthogonal_loss()`` (:170-242)                     -> :class:`MoE_CMix`

The reference evaluates every expert densely for every token and masks the
result (moe.py:138-145).  Here the routed (token, slot) entries are sorted by
expert with a stable counting sort (``rwkv_moe_permute``), the rank-r
down-projection runs per expert group (``rwkv_moe_lora_down``) and the
up-projection, score weighting and residual add are fused in one combine pass
(``rwkv_moe_lora_combine``).  Top-k ties go to the lower expert id; slots are in
descending logit order (the reference's argpartition leaves both unspecified).

The full-expert ``MoE_CMix`` uses the same sorted dispatch: one kernel builds every
routed row with its expert's token-shift mix (``rwkv_moe_expert_mix_rows``), the two
products of each expert run as library GEMMs (cuBLAS) on that expert's contiguous row
range with the squared ReLU applied in place between them (``rwkv_relu_sq``), and
``rwkv_moe_combine_rows`` forms the score-weighted sum per token.

These modules compute the forward pass only (no autograd through the kernels): a call
with autograd enabled that would need gradients (an input that requires grad, or a
trainable adapter / router / expert parameter) raises instead of returning values
that silently carry no gradient.  Run them under ``torch.no_grad()`` /
``torch.inference_mode()``, or freeze the parameters.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from . import _native as nat
from .fused import grouped_gemm, relu_sq_


def _stream(dev):
    return nat.stream_ptr(dev)


def check_forward_only(name: str, x: torch.Tensor, params) -> None:
    """Raise if autograd would need gradients through these forward-only kernels.

    The reference's module is differentiable (finetune_moe.py trains the adapters and
    the router through it); these kernels have no backward, so a training call must
    fail loudly rather than yield zero gradients for the adapters, the router and the
    layers before it."""
    if not torch.is_grad_enabled():
        return
    if x.requires_grad or any(p.requires_grad for p in params):
        raise RuntimeError(
            f"{name}: the CUDA kernels of this module are forward-only (no backward); call it "
            "under torch.no_grad() / torch.inference_mode(), or freeze its parameters "
            "(requires_grad_(False)) and pass an input that does not require grad")


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


def lora_apply_routed_supported(C: int, R: int, E: int, top_k: int, dtype: torch.dtype) -> bool:
    """The router folded into the fused apply kernel: fp16, E <= 16, E * R in {32, 64, 128}."""
    return bool(nat.lib().rwkv_moe_lora_apply_routed_supported(C, R, E, top_k, nat.dtype_code_of(dtype)))


def lora_apply_routed(x2d, base2d, A, Bw, gate_w, top_k: int, bias=None, out=None):
    """Router (moe.py:51-86) and adapter apply (moe.py:142-147) in one pass over x:
    returns (out, routing dict like :func:`router_forward`, without logits)."""
    ntok, C = x2d.shape
    E, _, R = A.shape
    dt = x2d.dtype
    dev = x2d.device
    if out is None:
        out = torch.empty((ntok, C), device=dev, dtype=dt)
    A = A.to(dt).contiguous()
    Bw = Bw.to(dt).contiguous()
    base2d = None if base2d is None else base2d.to(dt).contiguous()
    gw = gate_w.to(torch.float32).contiguous()
    b = None if bias is None else bias.to(torch.float32).contiguous()
    inds = torch.empty((ntok, top_k), device=dev, dtype=torch.int32)
    scores = torch.empty((ntok, top_k), device=dev, dtype=dt)
    stats = torch.empty(2 + E, device=dev, dtype=torch.float32)
    counts = torch.empty(E, device=dev, dtype=torch.int32)
    L = nat.lib()
    ws_bytes = L.rwkv_moe_lora_apply_routed_workspace_size(ntok, C, E)
    ws = torch.empty(max(1, ws_bytes), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        rc = L.rwkv_moe_lora_apply_routed(nat.ptr(x2d.contiguous()), nat.ptr(base2d), nat.ptr(A), nat.ptr(Bw),
                                          nat.ptr(gw), nat.ptr(b), nat.ptr(inds), nat.ptr(scores), nat.ptr(stats),
                                          nat.ptr(counts), nat.ptr(ws), ws_bytes, nat.ptr(out), ntok, C, R, E,
                                          top_k, nat.dtype_code(x2d), _stream(dev))
    nat.check(rc, "rwkv_moe_lora_apply_routed")
    return out, {"inds": inds, "scores": scores, "aux": stats[0], "z": stats[1], "f": stats[2:],
                 "counts": counts, "logits": None}


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


def expert_mix_rows(x2d, prev, x_k, perm, offsets, T: int, top_k: int):
    """rows[p] = x[tok] + (x_prev - x[tok]) * x_k[e(p)] for the sorted routing entries
    (moe.py:231-233); x_prev from the same sequence of T tokens, else ``prev``."""
    ntok, C = x2d.shape
    E = x_k.shape[0]
    n = perm.numel()
    rows = torch.empty((n, C), device=x2d.device, dtype=x2d.dtype)
    xk = x_k.reshape(E, C).to(x2d.dtype).contiguous()
    prev = None if prev is None else prev.to(x2d.dtype).contiguous()
    L = nat.lib()
    with torch.cuda.device(x2d.device):
        rc = L.rwkv_moe_expert_mix_rows(nat.ptr(x2d), nat.ptr(prev), nat.ptr(xk), nat.ptr(perm), nat.ptr(offsets),
                                        nat.ptr(rows), n, T, C, top_k, E, nat.dtype_code(x2d), _stream(x2d.device))
    nat.check(rc, "rwkv_moe_expert_mix_rows")
    return rows


def combine_rows(base2d, rows, scores, inv, ntok: int):
    """out[t] = base[t] + sum_s scores[t, s] * rows[inv[t * k + s]] (base may be None)."""
    k = scores.shape[-1]
    C = rows.shape[1]
    out = torch.empty((ntok, C), device=rows.device, dtype=rows.dtype)
    L = nat.lib()
    with torch.cuda.device(rows.device):
        rc = L.rwkv_moe_combine_rows(nat.ptr(base2d), nat.ptr(rows), nat.ptr(scores.contiguous()), nat.ptr(inv),
                                     nat.ptr(out), ntok, C, k, nat.dtype_code(out), _stream(rows.device))
    nat.check(rc, "rwkv_moe_combine_rows")
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
        # the base is frozen (stop_gradient in moe.py:131); adapters and router are not
        check_forward_only("LoRAMoE_CMix", x, (self.lora_A, self.lora_B, self.router.gate.weight))
        B, T, C = x.shape
        with torch.no_grad():
            base_out = self.base(x)
        x2 = x.reshape(B * T, C).contiguous()
        if lora_apply_routed_supported(C, self.lora_rank, self.n_experts, self.top_k, x.dtype):
            # router folded into the adapter pass: x is read once
            b2 = base_out.reshape(B * T, C)
            out, r = lora_apply_routed(x2, b2, self.lora_A.detach(), self.lora_B.detach(), self.router.gate.weight,
                                       self.top_k, self.router.bias, out=b2)
            return out.reshape(B, T, C), r["aux"], r["z"]
        r = router_forward(x2, self.router.gate.weight, self.top_k, self.router.bias)
        if lora_apply_supported(C, self.lora_rank, self.n_experts, self.top_k, x.dtype):
            b2 = base_out.reshape(B * T, C)  # a temporary: the adapters are added into it in place
            out = lora_apply(x2, b2, self.lora_A.detach(), self.lora_B.detach(), r["inds"], r["scores"], out=b2)
        else:  # sorted dispatch: grouped down-projection, then per-token combine
            perm, inv, offsets = permute(r["inds"], self.n_experts)
            h = lora_down(x2, self.lora_A.detach(), perm, offsets, self.top_k)
            out = lora_combine(base_out.reshape(B * T, C), h, self.lora_B.detach(), r["inds"],
                               r["scores"], inv)
        return out.reshape(B, T, C), r["aux"], r["z"]

    def orthogonal_loss(self) -> torch.Tensor:
        return ortho_loss(self.lora_A.detach())


class MoE_CMix(nn.Module):
    """Sparse MoE ChannelMix with E full experts and top-k routing (moe.py:170-242).

    Each expert is a ChannelMix (token shift -> lerp with its own ``x_k`` -> key ->
    squared ReLU -> value); out = sum over the selected experts of score * expert(x).
    Parameter names, shapes and init follow the reference: ``router.gate.weight``
    (E, C), ``x_k`` (E, 1, 1, C) zeros, ``expert_key`` (E, D, C) orthogonal scaled by
    sqrt(D / C), ``expert_val`` (E, C, D) zeros.  The reference evaluates every expert
    for every token (moe.py:230-239); here only the routed (token, expert) rows are
    computed (see the module docstring)."""

    def __init__(self, config, layer_id: int, n_experts: int, top_k: int = 2):
        super().__init__()
        self.n_experts, self.top_k, self.layer_id = n_experts, top_k, layer_id
        C, D = config.n_embd, config.dim_ffn
        self.router = Router(C, n_experts, top_k)
        self.x_k = nn.Parameter(torch.zeros(n_experts, 1, 1, C))
        key = []
        for _ in range(n_experts):
            q, _ = torch.linalg.qr(torch.randn(D, C) if D >= C else torch.randn(C, D))
            q = q if D >= C else q.T
            key.append(q[:D, :C] * math.sqrt(D / C))
        self.expert_key = nn.Parameter(torch.stack(key))
        self.expert_val = nn.Parameter(torch.zeros(n_experts, C, D))

    def _experts(self, x2d: torch.Tensor, prev, T: int):
        """(ntok, C) tokens in sequences of T (prev: the token before each sequence,
        or None) -> (out (ntok, C), router result)."""
        ntok, C = x2d.shape
        E, k = self.n_experts, self.top_k
        D = self.expert_key.shape[1]
        dt = x2d.dtype
        r = router_forward(x2d, self.router.gate.weight, k, self.router.bias)
        perm, inv, offsets = permute(r["inds"], E)
        rows = expert_mix_rows(x2d, prev, self.x_k.detach(), perm, offsets, T, k)
        if dt in (torch.float16, torch.bfloat16):
            # the expert products on the tcgen05 grouped GEMM, sized on the device from the
            # offsets (no host read): key + squared ReLU, then value
            h = grouped_gemm(rows, self.expert_key.detach(), offsets, relu_sq=True)
            o = grouped_gemm(h, self.expert_val.detach(), offsets)
            return combine_rows(None, o, r["scores"], inv, ntok), r
        # fp32 activations: one library GEMM pair per expert over its contiguous rows,
        # sized on the host (one device -> host read of the E+1 offsets)
        offs = offsets.tolist()
        wk = self.expert_key.detach().to(dt)
        wv = self.expert_val.detach().to(dt)
        h = torch.empty((rows.shape[0], D), device=x2d.device, dtype=dt)
        o = torch.empty_like(rows)
        for e in range(E):
            a, b = offs[e], offs[e + 1]
            if b > a:
                torch.mm(rows[a:b], wk[e].t(), out=h[a:b])
        relu_sq_(h)
        for e in range(E):
            a, b = offs[e], offs[e + 1]
            if b > a:
                torch.mm(h[a:b], wv[e].t(), out=o[a:b])
        return combine_rows(None, o, r["scores"], inv, ntok), r

    def forward(self, x: torch.Tensor):
        """x (B, T, C) -> (out (B, T, C), aux_loss, z_loss)  (moe.py:224-239)."""
        check_forward_only("MoE_CMix", x, self.parameters())
        B, T, C = x.shape
        out, r = self._experts(x.reshape(B * T, C).contiguous(), None, T)
        return out.reshape(B, T, C), r["aux"], r["z"]

    def forward_rnn(self, x: torch.Tensor, x_prev: torch.Tensor) -> torch.Tensor:
        """One token per sequence: x, x_prev (Bs, C) -> (Bs, C).  The reference's RNN
        mode has no MoE branch; this is the ChannelMix RNN step (model.py:498-506) per
        selected expert, weighted like the GPT-mode output."""
        check_forward_only("MoE_CMix", x, self.parameters())
        out, _ = self._experts(x.contiguous(), x_prev, 1)
        return out

    def orthogonal_loss(self) -> torch.Tensor:
        """No orthogonality loss for full experts (moe.py:241-242)."""
        return torch.zeros((), device=self.x_k.device, dtype=torch.float32)
