"""RWKV-v7 model shell on the B200 kernels (the callers of the two hot paths).

Mirrors rwkv_mlx/model.py: ``RWKVConfig`` (:18-64), ``RWKV_Tmix_x070`` (:119-240),
``RWKV_CMix_x070`` (:243-263), ``Block`` (:266-327), ``RWKV`` with GPT-mode
``forward`` (:346-375), RNN-mode ``forward_rnn`` (:377-421) and ``init_state``
(:423-431), plus the weight init of rwkv_mlx/train.py:209-310.  Parameter names
and shapes follow the reference so its safetensors names map one to one.

The WKV-7 recurrence runs on ``wkv7_recurrent`` / ``wkv7_with_state`` /
``wkv7_step``; LoRA-MoE ChannelMix on ``LoRAMoE_CMix``.  Dense projections are
cuBLAS GEMMs through torch.  Additions over the reference: a batched RNN step
(``forward_rnn_batch``) and a GPT-mode forward that also returns the RNN state
(``forward_with_state``), so a prompt can be prefilled in parallel and then
decoded step by step.

``ln_x`` grouping: the reference builds ``nn.GroupNorm(H, C)`` with MLX's default
``pytorch_compatible=False``; MLX then forms group g from the channels
c = g (mod H) (strided), not from the contiguous 64 channels of head g.  That is
the default here (``RWKVConfig.groupnorm = "mlx"``); ``"per_head"`` gives the
contiguous grouping of upstream RWKV-7 / PyTorch.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import nn

from . import fused as fz
from .wkv7 import wkv7_recurrent, wkv7_step, wkv7_with_state


@dataclass
class RWKVConfig:
    """Same fields and defaults as rwkv_mlx/model.py:18-64 (+ ``groupnorm``)."""

    n_layer: int = 12
    n_embd: int = 768
    vocab_size: int = 65568
    head_size: int = 64
    ctx_len: int = 4096
    dim_att: int = 0
    dim_ffn: int = 0
    d_decay_lora: int = 0
    d_aaa_lora: int = 0
    d_mv_lora: int = 0
    d_gate_lora: int = 0
    moe_num_experts: int = 0
    moe_top_k: int = 2
    moe_mode: str = "lora"
    moe_lora_rank: int = 64
    moe_layers: tuple = ()
    moe_aux_loss_coeff: float = 0.01
    moe_z_loss_coeff: float = 0.001
    moe_ortho_coeff: float = 0.001
    groupnorm: str = "mlx"
    fused: bool = True  # fused element-wise kernels around WKV (False: op-by-op torch path)

    def __post_init__(self):
        if self.dim_att <= 0:
            self.dim_att = self.n_embd
        if self.dim_ffn <= 0:
            self.dim_ffn = int((self.n_embd * 3.5) // 32 * 32)

    @property
    def n_head(self) -> int:
        return self.dim_att // self.head_size

    def lora_dim(self, kind: str) -> int:
        C = self.n_embd
        if kind == "decay":
            return self.d_decay_lora or max(32, int(round((2.5 * (C ** 0.5)) / 32) * 32))
        if kind == "aaa":
            return self.d_aaa_lora or max(32, int(round((2.5 * (C ** 0.5)) / 32) * 32))
        if kind == "mv":
            return self.d_mv_lora or max(32, int(round((1.7 * (C ** 0.5)) / 32) * 32))
        if kind == "gate":
            return self.d_gate_lora or max(32, int(round((5.0 * (C ** 0.5)) / 32) * 32))
        raise ValueError(f"Unknown LoRA kind: {kind}")


def time_shift(x: torch.Tensor) -> torch.Tensor:
    """Prepend a zero row along T and drop the last (model.py:67-75)."""
    return F.pad(x, (0, 0, 1, -1))


class GroupNormMLX(nn.Module):
    """GroupNorm over (N, C) with MLX's grouping (see the module docstring)."""

    def __init__(self, num_groups: int, dims: int, eps: float = 1e-5, mode: str = "mlx"):
        super().__init__()
        self.num_groups, self.dims, self.eps, self.mode = num_groups, dims, eps, mode
        self.weight = nn.Parameter(torch.ones(dims))
        self.bias = nn.Parameter(torch.zeros(dims))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        n, C = x.shape
        G = self.num_groups
        xf = x.float()
        if self.mode == "mlx":
            xg = xf.view(n, C // G, G)
            mean = xg.mean(1, keepdim=True)
            var = xg.var(1, unbiased=False, keepdim=True)
        else:
            xg = xf.view(n, G, C // G)
            mean = xg.mean(2, keepdim=True)
            var = xg.var(2, unbiased=False, keepdim=True)
        y = ((xg - mean) * torch.rsqrt(var + self.eps)).view(n, C)
        return (y * self.weight.float() + self.bias.float()).to(x.dtype)


class RWKV_Tmix_x070(nn.Module):
    """Time mixing (model.py:119-240)."""

    def __init__(self, config: RWKVConfig, layer_id: int):
        super().__init__()
        self.config, self.layer_id = config, layer_id
        self.head_size, self.n_head = config.head_size, config.n_head
        C, H, N = config.n_embd, config.n_head, config.head_size
        z = lambda *s: nn.Parameter(torch.zeros(*s))
        self.x_r, self.x_w, self.x_k, self.x_v, self.x_a, self.x_g = (z(1, 1, C) for _ in range(6))
        D = config.lora_dim("decay")
        self.w0, self.w1, self.w2 = z(1, 1, C), z(C, D), z(D, C)
        D = config.lora_dim("aaa")
        self.a0, self.a1, self.a2 = z(1, 1, C), z(C, D), z(D, C)
        D = config.lora_dim("mv")
        self.v0, self.v1, self.v2 = z(1, 1, C), z(C, D), z(D, C)
        D = config.lora_dim("gate")
        self.g1, self.g2 = z(C, D), z(D, C)
        self.k_k, self.k_a, self.r_k = z(1, 1, C), z(1, 1, C), z(H, N)
        self.receptance = nn.Linear(C, C, bias=False)
        self.key = nn.Linear(C, C, bias=False)
        self.value = nn.Linear(C, C, bias=False)
        self.output = nn.Linear(C, C, bias=False)
        self.ln_x = GroupNormMLX(H, C, eps=64e-5, mode=config.groupnorm)
        self._packed, self._packed_key = None, None
        self._lora, self._lora_key = None, None

    def _packed_weights(self):
        """The six token-shift mixes as one (6, C) tensor and W_r, W_k, W_v stacked for one
        batched product, rebuilt only when a parameter changes (storage, dtype or an
        in-place update), so inference steps launch no copies for them."""
        ps = (self.x_r, self.x_k, self.x_v, self.x_w, self.x_a, self.x_g,
              self.receptance.weight, self.key.weight, self.value.weight)
        key = tuple((p.data_ptr(), p.dtype, p._version) for p in ps)
        if self._packed_key != key:
            C = self.x_r.shape[-1]
            with torch.no_grad():
                mix = torch.cat([p.detach() for p in ps[:6]]).view(6, C)
                wrkv = torch.stack([p.detach() for p in ps[6:]]).transpose(1, 2)
            self._packed, self._packed_key = (mix, wrkv), key
        return self._packed

    def _packed_lora(self):
        """The four LoRA pairs in the order of the mixes v, w, a, g (slices 2..5 of the
        packed mixes), zero-padded to one rank, stacked for two batched products:
        (4, C, D) and (4, D, C).  Zero padding is exact: padded first-stage columns are 0,
        and the padded second-stage rows are 0 whatever tanh / sigmoid makes of them."""
        ps = (self.v1, self.w1, self.a1, self.g1, self.v2, self.w2, self.a2, self.g2)
        key = tuple((p.data_ptr(), p.dtype, p._version) for p in ps)
        if self._lora_key != key:
            C = self.v1.shape[0]
            D = max(p.shape[1] for p in ps[:4])
            with torch.no_grad():
                w1 = torch.zeros(4, C, D, device=self.v1.device, dtype=self.v1.dtype)
                w2 = torch.zeros(4, D, C, device=self.v1.device, dtype=self.v1.dtype)
                for i in range(4):
                    w1[i, :, : ps[i].shape[1]] = ps[i].detach()
                    w2[i, : ps[4 + i].shape[0]] = ps[4 + i].detach()
            self._lora, self._lora_key = (w1, w2), key
        return self._lora

    def _lora_products(self, X):
        """wl, al, vl, g of the fused paths from the mixes X (6, rows, C) in two batched
        products (3 launches instead of 10)."""
        w1, w2 = self._packed_lora()
        h = fz.lora_act_(torch.bmm(X[2:6], w1))  # (4, rows, D): v, tanh(w), a, sigmoid(g)
        o = torch.bmm(h, w2)
        return o[1], o[2], o[0], o[3]

    def _project(self, x, xx, v_first):
        """Shared by GPT and RNN mode: returns r, w(log-log), k, v, a, g, kk, v_first."""
        H, N = self.n_head, self.head_size
        xr, xw, xk = x + xx * self.x_r, x + xx * self.x_w, x + xx * self.x_k
        xv, xa, xg = x + xx * self.x_v, x + xx * self.x_a, x + xx * self.x_g
        r = self.receptance(xr)
        w = -F.softplus(-(self.w0 + torch.tanh(xw @ self.w1) @ self.w2)) - 0.5
        k = self.key(xk)
        v = self.value(xv)
        if self.layer_id == 0:
            v_first = v
        else:
            v = v + (v_first - v) * torch.sigmoid(self.v0 + (xv @ self.v1) @ self.v2)
        a = torch.sigmoid(self.a0 + (xa @ self.a1) @ self.a2)
        g = torch.sigmoid(xg @ self.g1) @ self.g2
        kk = k * self.k_k
        kk_h = kk.view(*kk.shape[:-1], H, N)
        kk = (kk_h / (torch.sqrt((kk_h * kk_h).sum(-1, keepdim=True)) + 1e-12)).view(kk.shape)
        k = k * (1 + (a - 1) * self.k_a)
        return r, w, k, v, a, g, kk, v_first

    def _post(self, y, r, k, v, g):
        H, N = self.n_head, self.head_size
        shp = y.shape
        C = shp[-1]
        y = self.ln_x(y.reshape(-1, C)).view(shp)
        rh, kh, vh = r.view(*shp[:-1], H, N), k.view(*shp[:-1], H, N), v.view(*shp[:-1], H, N)
        bonus = ((rh * kh * self.r_k).sum(-1, keepdim=True) * vh).view(shp)
        y = y + bonus
        return self.output((y * g).to(self.output.weight.dtype))

    def _forward_fused(self, x, v_first, s0, return_state):
        B, T, C = x.shape
        H, N = self.n_head, self.head_size
        mix, wrkv = self._packed_weights()
        X = fz.lerp(x, mix, T)  # (6, B*T, C): r, k, v, w, a, g inputs
        rkv = torch.bmm(X[0:3], wrkv)
        r, k, v = rkv[0], rkv[1], rkv[2]
        wl, al, vl, g = self._lora_products(X)
        layer0 = self.layer_id == 0
        if layer0:
            vl = None
        vf = None if layer0 else v_first.reshape(B * T, C)
        w, k2, v2, a_in, b_in = fz.tmix_mid(k, v, wl, al, vl, vf, self.w0.view(-1), self.a0.view(-1),
                                             self.v0.view(-1), self.k_k.view(-1), self.k_a.view(-1), layer0)
        sh = (B, T, C)
        r, w, k2, v2, a_in, b_in = (t.view(sh) for t in (r, w, k2, v2, a_in, b_in))
        if layer0:
            v_first = v2
        if return_state or s0 is not None:
            y, sT = wkv7_with_state(r, w, k2, v2, a_in, b_in, s0=s0, head_size=N)
        else:
            y, sT = wkv7_recurrent(r, w, k2, v2, a_in, b_in, N), None
        pre = fz.tmix_post(y, r, k2, v2, g.view(sh), self.ln_x.weight, self.ln_x.bias, self.r_k, H,
                           self.ln_x.eps, self.config.groupnorm != "mlx")
        out = self.output(pre)
        return (out, v_first, sT) if return_state else (out, v_first)

    def forward(self, x, v_first, s0=None, return_state=False):
        if self.config.fused and not torch.is_grad_enabled() and x.is_cuda:
            return self._forward_fused(x, v_first, s0, return_state)
        xx = time_shift(x) - x
        r, w, k, v, a, g, kk, v_first = self._project(x, xx, v_first)
        if return_state or s0 is not None:
            y, sT = wkv7_with_state(r, w, k, v, -kk, kk * a, s0=s0, head_size=self.head_size)
        else:
            y, sT = wkv7_recurrent(r, w, k, v, -kk, kk * a, self.head_size), None
        out = self._post(y, r, k, v, g)
        return (out, v_first, sT) if return_state else (out, v_first)

    def _forward_rnn_fused(self, x, x_prev, v_first, state, update_prev=False):
        """forward_rnn on the fused kernels: x, x_prev (Bs, C); v_first (Bs, C) or None for
        layer 0.  Returns (out (Bs, C), v_first)."""
        Bs, C = x.shape
        H = self.n_head
        mix, wrkv = self._packed_weights()
        # (6, Bs, C); with update_prev the same pass stores x as the next shift state
        X = fz.lerp(x, mix, 1, prev=x_prev, prev_out=x_prev if update_prev else None)
        rkv = torch.bmm(X[0:3], wrkv)
        r, k, v = rkv[0], rkv[1], rkv[2]
        wl, al, vl, g = self._lora_products(X)
        layer0 = self.layer_id == 0
        if layer0:
            vl = None
        w, k2, v2, a_in, b_in = fz.tmix_mid(k, v, wl, al, vl, None if layer0 else v_first, self.w0.view(-1),
                                             self.a0.view(-1), self.v0.view(-1), self.k_k.view(-1),
                                             self.k_a.view(-1), layer0)
        if layer0:
            v_first = v2
        y = wkv7_step(state, r, w, k2, v2, a_in, b_in, w_is_decay=False)
        pre = fz.tmix_post(y, r, k2, v2, g, self.ln_x.weight, self.ln_x.bias, self.r_k, H, self.ln_x.eps,
                           self.config.groupnorm != "mlx")
        return self.output(pre), v_first

    def forward_rnn(self, x, x_prev, v_first, state):
        """Batched RNN step (model.py:441-495): x, x_prev (Bs, C); state (Bs,H,N,N)
        fp32 updated in place.  Returns (out, x, state, v_first)."""
        # run the GPT-mode projections on (Bs, 1, C) so parameter broadcasting matches
        xx = (x_prev - x)[:, None]
        r, w, k, v, a, g, kk, v_first = self._project(x[:, None], xx, v_first[:, None])
        # model.py:475-477 forms the decay as exp(-0.606531*sigmoid(w0 + w_lora)); that is
        # exp(-exp(w)) of GPT mode's w = -softplus(-(w0 + w_lora)) - 0.5, which the kernel
        # evaluates (the constant differs from e^-0.5 by 6e-8)
        y = wkv7_step(state, r, w, k, v, -kk, kk * a, w_is_decay=False)
        out = self._post(y.view(r.shape), r, k, v, g)
        return out[:, 0], x, state, v_first[:, 0]


_FUSED_KEY_MIN_ROWS = 24576


class RWKV_CMix_x070(nn.Module):
    """Channel mixing (model.py:243-263)."""

    def __init__(self, config: RWKVConfig, layer_id: int):
        super().__init__()
        self.config, self.layer_id = config, layer_id
        C = config.n_embd
        self.x_k = nn.Parameter(torch.zeros(1, 1, C))
        self.key = nn.Linear(C, config.dim_ffn, bias=False)
        self.value = nn.Linear(config.dim_ffn, C, bias=False)

    def forward(self, x):
        if self.config.fused and not torch.is_grad_enabled() and x.is_cuda:
            k = fz.lerp(x, self.x_k.view(1, -1), x.shape[1])[0]  # (rows, C)
            wk = self.key.weight
            if (x.dtype in (torch.float16, torch.bfloat16) and wk.dtype == x.dtype and k.shape[1] % 8 == 0
                    and k.shape[0] >= _FUSED_KEY_MIN_ROWS):
                # key product and squared ReLU in one tcgen05 GEMM (no extra pass over the
                # (rows, dim_ffn) activations); below ~24 k rows the library GEMM's smaller
                # tiles plus the separate pass are faster (measured: 4096 rows 22 vs 28 us,
                # 32768 rows 181 vs 165 us)
                h = fz.grouped_gemm(k, wk.view(1, *wk.shape), None, relu_sq=True)
                return self.value(h).view(x.shape)
            return self.value(fz.relu_sq_(self.key(k.view(x.shape))))
        xx = time_shift(x) - x
        k = x + xx * self.x_k
        k = torch.relu(self.key(k)) ** 2
        return self.value(k)

    def forward_rnn_fused(self, x, x_prev, update_prev=False):
        k = fz.lerp(x, self.x_k.view(1, -1), 1, prev=x_prev, prev_out=x_prev if update_prev else None)[0]
        return self.value(fz.relu_sq_(self.key(k)))

    def forward_rnn(self, x, x_prev):
        """model.py:498-506 (batched)."""
        xx = x_prev - x
        k = x + xx * self.x_k.view(-1)
        k = torch.relu(self.key(k)) ** 2
        return self.value(k), x


class Block(nn.Module):
    """LayerNorm -> TimeMix -> LayerNorm -> ChannelMix / LoRA-MoE (model.py:266-327)."""

    def __init__(self, config: RWKVConfig, layer_id: int):
        super().__init__()
        self.config, self.layer_id = config, layer_id
        self.is_moe = False
        C = config.n_embd
        if layer_id == 0:
            self.ln0 = nn.LayerNorm(C)
        self.ln1 = nn.LayerNorm(C)
        self.ln2 = nn.LayerNorm(C)
        self.att = RWKV_Tmix_x070(config, layer_id)
        use_moe = config.moe_num_experts > 0 and (not config.moe_layers or layer_id in config.moe_layers)
        if use_moe:
            self.is_moe = True
            if config.moe_mode == "lora":
                from .moe import LoRAMoE_CMix

                self.ffn = LoRAMoE_CMix(RWKV_CMix_x070(config, layer_id), config.moe_num_experts,
                                        config.moe_lora_rank, config.moe_top_k)
            else:  # "full": E independent ChannelMix experts (model.py:306-308)
                from .moe import MoE_CMix

                self.ffn = MoE_CMix(config, layer_id, config.moe_num_experts, config.moe_top_k)
        else:
            self.ffn = RWKV_CMix_x070(config, layer_id)

    def forward_fused(self, x, pending, v_first, return_state=False):
        """Block with the residual adds folded into the LayerNorm passes: ``pending``
        is the previous block's ChannelMix output, not yet added to ``x``.  Returns
        (x, pending_ffn_out, v_first, moe_losses, extra)."""
        if self.layer_id == 0:
            _, x = fz.add_layernorm(x, None, self.ln0.weight, self.ln0.bias, self.ln0.eps)
        x, x1 = fz.add_layernorm(x, pending, self.ln1.weight, self.ln1.bias, self.ln1.eps)
        res = self.att(x1, v_first, return_state=return_state)
        x, x2 = fz.add_layernorm(x, res[0], self.ln2.weight, self.ln2.bias, self.ln2.eps)
        extra = {}
        if return_state:
            extra = {"att_x_prev": x1[:, -1], "att_state": res[2], "ffn_x_prev": x2[:, -1]}
        if self.is_moe:
            ffn_out, aux, z = self.ffn(x2)
            return x, ffn_out, res[1], (aux, z, self.ffn.orthogonal_loss()), extra
        return x, self.ffn(x2), res[1], None, extra

    def forward(self, x, v_first, s0=None, return_state=False):
        if self.layer_id == 0:
            x = self.ln0(x)
        x1 = self.ln1(x)
        res = self.att(x1, v_first, s0=s0, return_state=return_state)
        x_attn, v_first = res[0], res[1]
        x = x + x_attn
        x2 = self.ln2(x)
        extra = {}
        if return_state:
            extra = {"att_x_prev": x1[:, -1], "att_state": res[2], "ffn_x_prev": x2[:, -1]}
        if self.is_moe:
            ffn_out, aux, z = self.ffn(x2)
            x = x + ffn_out
            return x, v_first, (aux, z, self.ffn.orthogonal_loss()), extra
        x = x + self.ffn(x2)
        return x, v_first, None, extra


class RWKV(nn.Module):
    """RWKV-v7 language model (model.py:330-431)."""

    def __init__(self, config: RWKVConfig):
        super().__init__()
        self.config = config
        self.emb = nn.Embedding(config.vocab_size, config.n_embd)
        self.blocks = nn.ModuleList([Block(config, i) for i in range(config.n_layer)])
        self.ln_out = nn.LayerNorm(config.n_embd)
        self.head = nn.Linear(config.n_embd, config.vocab_size, bias=False)

    def _run(self, idx, return_state=False, head=True):
        x = self.emb(idx)
        v_first = torch.zeros_like(x)
        aux_loss = torch.zeros((), device=x.device, dtype=torch.float32)
        cfg = self.config
        states = []
        if cfg.fused and not torch.is_grad_enabled() and x.is_cuda:
            pending = None
            for blk in self.blocks:
                x, pending, v_first, moe, extra = blk.forward_fused(x, pending, v_first, return_state)
                if moe is not None:
                    aux, z, ortho = moe
                    aux_loss = aux_loss + cfg.moe_aux_loss_coeff * aux + cfg.moe_z_loss_coeff * z \
                        + cfg.moe_ortho_coeff * ortho
                if return_state:
                    states.append(extra)
            _, x = fz.add_layernorm(x, pending, self.ln_out.weight, self.ln_out.bias, self.ln_out.eps)
            return (self.head(x) if head else x), aux_loss, states
        for blk in self.blocks:
            x, v_first, moe, extra = blk(x, v_first, return_state=return_state)
            if moe is not None:
                aux, z, ortho = moe
                aux_loss = aux_loss + cfg.moe_aux_loss_coeff * aux + cfg.moe_z_loss_coeff * z \
                    + cfg.moe_ortho_coeff * ortho
            if return_state:
                states.append(extra)
        x = self.ln_out(x)
        return (self.head(x) if head else x), aux_loss, states

    def forward(self, idx):
        """GPT mode: idx (B, T) -> (logits (B, T, V), aux_loss)  (model.py:346-375)."""
        logits, aux, _ = self._run(idx)
        return logits, aux

    def forward_loss(self, idx, targets, mask=None, chunk: int = 8192):
        """The reference's training objective (train.py:483-489):
        ``l2_wrap_loss(logits, targets)`` (masked when ``mask`` is given) + the MoE aux
        loss, with the output head fused into the loss so the (B, T, V) logits are never
        held (``loss.head_l2_wrap_loss``)."""
        from .loss import head_l2_wrap_loss

        x, aux, _ = self._run(idx, head=False)
        return head_l2_wrap_loss(x, self.head.weight, targets, mask, chunk) + aux

    def forward_with_state(self, idx):
        """GPT-mode prefill that also returns the RNN state after the last token,
        as a list of per-layer dicts {att_x_prev (B,C), att_state (B,H,N,N) fp32,
        ffn_x_prev (B,C)} for :meth:`forward_rnn_batch`."""
        logits, aux, states = self._run(idx, return_state=True)
        return logits, aux, states

    # ---- RNN mode --------------------------------------------------------
    def init_state(self, batch: int | None = None):
        """Zero state.  ``batch=None``: the reference's flat list layout
        [att_x_prev (C), att_state (H,N,N), ffn_x_prev (C)] * n_layer (model.py:423-431);
        otherwise per-layer dicts with a leading batch dimension."""
        cfg = self.config
        dev = self.emb.weight.device
        dt = self.emb.weight.dtype
        C, H, N = cfg.n_embd, cfg.n_head, cfg.head_size
        if batch is None:
            st = []
            for _ in range(cfg.n_layer):
                st += [torch.zeros(C, device=dev, dtype=dt),
                       torch.zeros(H, N, N, device=dev, dtype=torch.float32),
                       torch.zeros(C, device=dev, dtype=dt)]
            return st
        return [{"att_x_prev": torch.zeros(batch, C, device=dev, dtype=dt),
                 "att_state": torch.zeros(batch, H, N, N, device=dev, dtype=torch.float32),
                 "ffn_x_prev": torch.zeros(batch, C, device=dev, dtype=dt)} for _ in range(cfg.n_layer)]

    def forward_rnn_batch(self, tokens: torch.Tensor, states: list):
        """One decode step for a batch of sequences: tokens (Bs,) -> logits (Bs, V).
        ``states`` (per-layer dicts) is updated in place: every state tensor keeps its
        storage, so a step can be captured in a CUDA graph (see :class:`DecodeGraph`)."""
        x = self.emb(tokens)
        if self.config.fused and not torch.is_grad_enabled() and x.is_cuda:
            return self._forward_rnn_batch_fused(x, states)
        v_first = torch.zeros_like(x)
        for i, blk in enumerate(self.blocks):
            if i == 0:
                x = blk.ln0(x)
            xx = blk.ln1(x)
            st = states[i]
            out, _, _, v_first = blk.att.forward_rnn(xx, st["att_x_prev"], v_first, st["att_state"])
            st["att_x_prev"].copy_(xx)
            x = x + out
            xx = blk.ln2(x)
            if blk.is_moe and not hasattr(blk.ffn, "base"):  # full experts
                x = x + blk.ffn.forward_rnn(xx, st["ffn_x_prev"])
            elif blk.is_moe:
                # the reference's RNN path cannot run MoE layers (model.py:498-506 reads
                # ffn.x_k / ffn.key); here the LoRA-MoE layer runs on the single token
                ffn = blk.ffn
                base, _ = ffn.base.forward_rnn(xx, st["ffn_x_prev"])
                delta = _moe_rnn(ffn, xx)
                x = x + base + delta
            else:
                out, _ = blk.ffn.forward_rnn(xx, st["ffn_x_prev"])
                x = x + out
            st["ffn_x_prev"].copy_(xx)
        x = self.ln_out(x)
        return self.head(x)

    def _forward_rnn_batch_fused(self, x, states):
        """forward_rnn_batch with the residual adds folded into the LayerNorm passes."""
        v_first, pending = None, None
        for i, blk in enumerate(self.blocks):
            if i == 0:
                _, x = fz.add_layernorm(x, None, blk.ln0.weight, blk.ln0.bias, blk.ln0.eps)
            x, xx = fz.add_layernorm(x, pending, blk.ln1.weight, blk.ln1.bias, blk.ln1.eps)
            st = states[i]
            out, v_first = blk.att._forward_rnn_fused(xx, st["att_x_prev"], v_first, st["att_state"],
                                                      update_prev=True)
            x, xx = fz.add_layernorm(x, out, blk.ln2.weight, blk.ln2.bias, blk.ln2.eps)
            if blk.is_moe and not hasattr(blk.ffn, "base"):  # full experts
                pending = blk.ffn.forward_rnn(xx, st["ffn_x_prev"])
            elif blk.is_moe:
                ffn = blk.ffn
                pending = ffn.base.forward_rnn_fused(xx, st["ffn_x_prev"]) + _moe_rnn(ffn, xx)
            else:
                pending = blk.ffn.forward_rnn_fused(xx, st["ffn_x_prev"], update_prev=True)
                continue
            st["ffn_x_prev"].copy_(xx)
        _, x = fz.add_layernorm(x, pending, self.ln_out.weight, self.ln_out.bias, self.ln_out.eps)
        return self.head(x)

    def forward_rnn(self, token: int, state: list):
        """Mirror of model.py:377-421 for one sequence: returns (logits (V,), state)."""
        cfg = self.config
        states = []
        for i in range(cfg.n_layer):
            states.append({"att_x_prev": state[3 * i].view(1, -1),
                           "att_state": state[3 * i + 1].view(1, cfg.n_head, cfg.head_size, cfg.head_size).contiguous(),
                           "ffn_x_prev": state[3 * i + 2].view(1, -1)})
        tok = torch.tensor([int(token)], device=self.emb.weight.device)
        logits = self.forward_rnn_batch(tok, states)
        new = []
        for st in states:
            new += [st["att_x_prev"].view(-1), st["att_state"].view(cfg.n_head, cfg.head_size, cfg.head_size),
                    st["ffn_x_prev"].view(-1)]
        return logits.view(-1), new


class DecodeGraph:
    """Greedy batched decode step captured once in a CUDA graph and replayed.

    ``states`` (from :meth:`RWKV.init_state` / :meth:`RWKV.forward_with_state`) and the
    token buffer keep their storage across steps; :meth:`step` replays the graph:
    logits = forward_rnn_batch(tokens, states); tokens = argmax(logits).

    The graph reads the weights as they were packed at capture (the stacked mixes,
    W_r/W_k/W_v and LoRA pairs are copies).  :meth:`step` therefore checks that no
    parameter has been updated in place or replaced since the capture and raises if
    one has: build a new DecodeGraph after loading or changing weights."""

    def __init__(self, model: "RWKV", states: list, tokens: torch.Tensor, warmup: int = 2):
        self.model, self.states = model, states
        self.tokens = tokens.clone()
        # states must own contiguous storage the graph can update in place
        for st in states:
            for k_ in st:
                st[k_] = st[k_].contiguous().clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.no_grad():
            saved = [{k_: v.clone() for k_, v in st.items()} for st in states]
            tok0 = self.tokens.clone()
            for _ in range(warmup):
                self.model.forward_rnn_batch(self.tokens, states)
            for st, sv in zip(states, saved):  # warm-up must not advance the sequences
                for k_ in st:
                    st[k_].copy_(sv[k_])
            self.tokens.copy_(tok0)
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.logits = self.model.forward_rnn_batch(self.tokens, states)
            if self.tokens.dtype == torch.int64 and self.tokens.is_contiguous() and self.logits.dim() == 2:
                fz.argmax_rows(self.logits, out=self.tokens)  # one launch, straight into the token buffer
            else:
                self.tokens.copy_(self.logits.argmax(-1))
        self._params = list(model.parameters())
        self._fingerprint = self._weights_fingerprint()

    def _weights_fingerprint(self):
        return tuple((p.data_ptr(), p._version) for p in self._params)

    def step(self):
        if self._weights_fingerprint() != self._fingerprint:
            raise RuntimeError("DecodeGraph: a model parameter was updated or replaced after the graph was "
                               "captured; the graph would decode with stale packed weights. Build a new "
                               "DecodeGraph.")
        self.graph.replay()
        return self.tokens


class PrefillGraph:
    """GPT-mode forward (:meth:`RWKV.forward`) of a fixed (B, T) batch captured once in a
    CUDA graph and replayed: one launch per step instead of ~17 per layer from Python,
    which matters when each GPU holds few sequences (strong scaling) and the host would
    otherwise bound the step.

    ``graph(idx)`` copies ``idx`` (any device or pinned host tensor of shape (B, T)) into
    the captured input buffer on the current stream, replays, and returns the captured
    ``(logits, aux)`` buffers (overwritten by the next replay).  Like
    :class:`DecodeGraph`, a replay refuses to run after a parameter was updated in place
    or replaced (the graph holds packed copies of some weights)."""

    def __init__(self, model: "RWKV", batch: int, seq_len: int, warmup: int = 2):
        self.model = model
        dev = model.emb.weight.device
        self.idx = torch.zeros((batch, seq_len), dtype=torch.long, device=dev)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(warmup):  # lazy one-time set-up (packed weights, kernel attributes) outside the capture
                model(self.idx)
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.logits, self.aux = model(self.idx)
        self._params = list(model.parameters())
        self._fingerprint = self._weights_fingerprint()

    def _weights_fingerprint(self):
        return tuple((p.data_ptr(), p._version) for p in self._params)

    def __call__(self, idx: torch.Tensor | None = None):
        if self._weights_fingerprint() != self._fingerprint:
            raise RuntimeError("PrefillGraph: a model parameter was updated or replaced after the graph was "
                               "captured; build a new PrefillGraph.")
        if idx is not None:
            self.idx.copy_(idx, non_blocking=True)
        self.graph.replay()
        return self.logits, self.aux


# ---------------------------------------------------------------------------
# The reference's module-level RNN-mode functions (model.py:441-506), same signatures
# ---------------------------------------------------------------------------
def _time_mixing_rnn(layer_id: int, H: int, N: int, x: torch.Tensor, x_prev: torch.Tensor,
                     v_first: torch.Tensor, state: torch.Tensor, att: RWKV_Tmix_x070):
    """RNN-mode time mixing of one token (model.py:441-495).

    x, x_prev, v_first (C,); state (H, N, N) fp32 -> (out (C,), x, new state (H, N, N),
    v_first).  Like the reference (immutable MLX arrays) the caller's ``state`` is not
    modified: the update runs in place on a copy (the batched kernel behind
    :meth:`RWKV_Tmix_x070.forward_rnn`, one sequence).  For ``layer_id == 0`` the value
    is returned as the new ``v_first``."""
    if layer_id != att.layer_id:
        raise ValueError(f"layer_id={layer_id} but att belongs to layer {att.layer_id}")
    if H != att.config.n_head or N != att.config.head_size:
        raise ValueError(f"H={H}, N={N} do not match the layer ({att.config.n_head}, {att.config.head_size})")
    C = H * N
    S = state.detach().to(torch.float32).reshape(1, H, N, N).clone()
    out, _, S, vf = att.forward_rnn(x.reshape(1, C), x_prev.reshape(1, C), v_first.reshape(1, C), S)
    return out.reshape(C), x, S.reshape(H, N, N), vf.reshape(C)


def _channel_mixing_rnn(x: torch.Tensor, x_prev: torch.Tensor, ffn: RWKV_CMix_x070):
    """RNN-mode channel mixing of one token (model.py:498-506): x, x_prev (C,) ->
    (out (C,), x).  Like the reference it needs a plain ChannelMix (``ffn.x_k``,
    ``ffn.key``)."""
    C = x.shape[-1]
    out, _ = ffn.forward_rnn(x.reshape(1, C), x_prev.reshape(1, C))
    return out.reshape(C), x


def _moe_rnn(ffn, x):
    from .moe import (check_forward_only, lora_apply, lora_apply_supported, lora_combine, lora_down, permute,
                      router_forward)

    check_forward_only("LoRAMoE_CMix", x, (ffn.lora_A, ffn.lora_B, ffn.router.gate.weight))
    r = router_forward(x.contiguous(), ffn.router.gate.weight, ffn.top_k, ffn.router.bias)
    C = x.shape[-1]
    if lora_apply_supported(C, ffn.lora_rank, ffn.n_experts, ffn.top_k, x.dtype):
        return lora_apply(x.contiguous(), None, ffn.lora_A.detach(), ffn.lora_B.detach(), r["inds"], r["scores"])
    perm, inv, off = permute(r["inds"], ffn.n_experts)
    h = lora_down(x.contiguous(), ffn.lora_A.detach(), perm, off, ffn.top_k)
    return lora_combine(None, h, ffn.lora_B.detach(), r["inds"], r["scores"], inv)


# ---------------------------------------------------------------------------
# Weight init (rwkv_mlx/train.py:209-310)
# ---------------------------------------------------------------------------
def _ortho(shape, scale, gen, device):
    rows, cols = shape
    flat = torch.randn(rows, cols, generator=gen, device=device, dtype=torch.float32)
    q, _ = torch.linalg.qr(flat if rows >= cols else flat.T)
    q = q.T if rows < cols else q
    q = q[:rows, :cols]
    gain = math.sqrt(rows / cols) if rows > cols else 1.0
    return q * gain * scale


@torch.no_grad()
def init_weights(model: RWKV, seed: int = 0):
    """Random init following train.py:209-310 (fp32 values)."""
    cfg = model.config
    C, H, N, L = cfg.n_embd, cfg.n_head, cfg.head_size, cfg.n_layer
    dev = model.emb.weight.device
    gen = torch.Generator(device=dev).manual_seed(seed)
    model.emb.weight.uniform_(-1e-4, 1e-4, generator=gen)
    V = cfg.vocab_size
    h_scale = 0.5 * math.sqrt(V / C) if V > C else 0.5
    model.head.weight.copy_(_ortho(model.head.weight.shape, h_scale, gen, dev))
    ar = torch.arange(C, device=dev, dtype=torch.float32)
    for lid, blk in enumerate(model.blocks):
        att = blk.att
        r01 = lid / (L - 1) if L > 1 else 0.0
        r1a0 = 1.0 - lid / L
        ddd = ar / C
        att.x_r.copy_((1.0 - ddd ** (0.2 * r1a0)).view(1, 1, C))
        att.x_w.copy_((1.0 - ddd ** (0.9 * r1a0)).view(1, 1, C))
        att.x_k.copy_((1.0 - ddd ** (0.7 * r1a0)).view(1, 1, C))
        att.x_v.copy_((1.0 - ddd ** (0.7 * r1a0)).view(1, 1, C))
        att.x_a.copy_((1.0 - ddd ** (0.9 * r1a0)).view(1, 1, C))
        att.x_g.copy_((1.0 - ddd ** (0.2 * r1a0)).view(1, 1, C))
        linear = ar / (C - 1) - 0.5
        n = torch.arange(C, device=dev, dtype=torch.float32) % N
        zig = (n - (N - 1) / 2) / ((N - 1) / 2)
        zig = zig * zig.abs()
        www = -6 + 6 * (ar / (C - 1)) ** (1 + r01 ** 0.3)
        att.w0.copy_((www + 0.5 + zig * 2.5).view(1, 1, C))
        att.w1.zero_()
        att.w2.copy_(_ortho(att.w2.shape, 0.1, gen, dev))
        att.a0.copy_((-0.19 + zig * 0.3 + linear * 0.4).view(1, 1, C))
        att.a1.zero_()
        att.a2.copy_(_ortho(att.a2.shape, 0.1, gen, dev))
        att.v0.copy_((0.73 - linear * 0.4).view(1, 1, C))
        att.v1.zero_()
        att.v2.copy_(_ortho(att.v2.shape, 0.1, gen, dev))
        att.g1.zero_()
        att.g2.copy_(_ortho(att.g2.shape, 0.1, gen, dev))
        att.k_k.copy_((0.71 - linear * 0.1).view(1, 1, C))
        att.k_a.fill_(1.02)
        att.r_k.fill_(-0.04)
        att.receptance.weight.copy_(_ortho(att.receptance.weight.shape, 1.0, gen, dev))
        att.key.weight.copy_(_ortho(att.key.weight.shape, 0.1, gen, dev))
        att.value.weight.copy_(_ortho(att.value.weight.shape, 1.0, gen, dev))
        att.output.weight.zero_()
        att.ln_x.weight.fill_(((1 + lid) / L) ** 0.7)
        xk = (1.0 - ddd ** ((1.0 - lid / L) ** 4)).view(1, 1, C)
        if blk.is_moe and not hasattr(blk.ffn, "base"):
            # full experts: the ChannelMix schedule for every expert's x_k, orthogonal keys
            # scaled by sqrt(D / C) and zero values as MoE_CMix.__init__ (moe.py:196-215)
            ffn = blk.ffn
            ffn.x_k.copy_(xk.expand_as(ffn.x_k[0]).unsqueeze(0).expand_as(ffn.x_k))
            for e in range(ffn.n_experts):
                ffn.expert_key[e].copy_(_ortho(ffn.expert_key[e].shape, 1.0, gen, dev))
            ffn.expert_val.zero_()
            continue
        ffn = blk.ffn.base if blk.is_moe else blk.ffn
        ffn.x_k.copy_(xk)
        ffn.key.weight.copy_(_ortho(ffn.key.weight.shape, 1.0, gen, dev))
        ffn.value.weight.zero_()
    return model


def cast_for_inference(model: RWKV, dtype=torch.float16) -> RWKV:
    """Cast every parameter to ``dtype`` except the decay biases ``w0`` (kept fp32,
    as the reference's converter does, convert.py:80-91)."""
    for name, p in model.named_parameters():
        if name.endswith(".w0"):
            p.data = p.data.float()
        else:
            p.data = p.data.to(dtype)
    return model
