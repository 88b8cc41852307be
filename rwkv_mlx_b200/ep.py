"""Expert-parallel LoRA-MoE ChannelMix over torch.distributed (NCCL on NVLink).

The reference runs every expert on one device (rwkv_mlx/moe.py:129-147).  Here expert
e lives on rank e // (E / world_size); each rank routes its own tokens, sends every
routed (token, slot) row to the rank that owns the chosen expert, receives the rows
its experts must process, applies the rank-r adapters, returns the results, and
combines them with the router scores and the frozen base output:

    router -> stable sort of the entries by expert (= by destination rank)
    -> all_to_all of counts -> all_to_all of rows and expert ids
    -> local adapters (fused x @ A_e @ B_e per row, or sorted + grouped for other shapes)
    -> all_to_all back -> out[t] = base[t] + sum_slot score * row

The aux and z losses are reduced over ranks exactly (sums of the per-rank partial
statistics weighted by token counts), so they equal the single-device values for
the concatenated batch.  Tokens never leave their rank except as routed rows.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from . import moe as gpu_moe


class GpuOps:
    """The B200 kernels behind each local step (the default)."""

    router = staticmethod(lambda x2, w, k, bias: gpu_moe.router_forward(x2, w, k, bias, want_logits=True))
    permute = staticmethod(gpu_moe.permute)
    ortho_loss = staticmethod(gpu_moe.ortho_loss)

    @staticmethod
    def gather_rows(x2, perm, topk):
        from . import _native as nat

        n, C = perm.numel(), x2.shape[1]
        rows = torch.empty((n, C), device=x2.device, dtype=x2.dtype)
        if n:
            L = nat.lib()
            with torch.cuda.device(x2.device):
                rc = L.rwkv_moe_gather_rows(nat.ptr(x2), nat.ptr(perm), nat.ptr(rows), n, C, topk,
                                            nat.dtype_code(x2), nat.stream_ptr(x2.device))
            nat.check(rc, "rwkv_moe_gather_rows")
        return rows

    @staticmethod
    def lora_down(rows, A, perm, offsets):
        return gpu_moe.lora_down(rows, A, perm, offsets, 1)

    @staticmethod
    def apply_local(rows, A, Bw, e_loc):
        """rows[i] @ A[e] @ B[e] with e = e_loc[i] in one fused pass, or None when the shape
        is outside the fused kernel (then the sorted path runs)."""
        E, C, R = A.shape
        if not gpu_moe.lora_apply_supported(C, R, E, 1, rows.dtype):
            return None
        return gpu_moe.lora_apply(rows, None, A, Bw, e_loc, None)

    @staticmethod
    def lora_up(h, Bw, offsets, out_index, dtype):
        from . import _native as nat

        n = h.shape[0]
        E, R, C = Bw.shape
        y = torch.empty((n, C), device=h.device, dtype=dtype)
        L = nat.lib()
        Bw = Bw.to(dtype).contiguous()
        with torch.cuda.device(h.device):
            rc = L.rwkv_moe_lora_up(nat.ptr(h), nat.ptr(Bw), nat.ptr(offsets), nat.ptr(out_index), nat.ptr(y), n,
                                    C, R, E, nat.dtype_code(y), nat.stream_ptr(h.device))
        nat.check(rc, "rwkv_moe_lora_up")
        return y

    @staticmethod
    def combine_rows(base2d, rows, scores, inv):
        from . import _native as nat

        ntok, k = scores.shape
        C = base2d.shape[1]
        out = torch.empty_like(base2d)
        L = nat.lib()
        with torch.cuda.device(out.device):
            rc = L.rwkv_moe_combine_rows(nat.ptr(base2d), nat.ptr(rows), nat.ptr(scores), nat.ptr(inv), nat.ptr(out),
                                         ntok, C, k, nat.dtype_code(out), nat.stream_ptr(out.device))
        nat.check(rc, "rwkv_moe_combine_rows")
        return out


def _a2a(out, inp, out_splits, in_splits, group):
    dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)
    return out


class ExpertParallelLoRAMoE(nn.Module):
    """LoRA-MoE ChannelMix (moe.py:93-163 semantics) with experts sharded over ranks.

    Holds the frozen base, the (replicated) router and the adapters of this rank's
    experts only: ``lora_A`` (E/ws, C, R), ``lora_B`` (E/ws, R, C)."""

    def __init__(self, base: nn.Module, n_experts: int, lora_rank: int, top_k: int = 2, group=None, ops=None):
        super().__init__()
        self.group = group
        self.ws = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_experts % self.ws:
            raise ValueError(f"n_experts={n_experts} must be a multiple of the world size {self.ws}")
        self.base, self.n_experts, self.lora_rank, self.top_k = base, n_experts, lora_rank, top_k
        self.local = n_experts // self.ws
        C = base.key.weight.shape[1]
        self.lora_A = nn.Parameter(torch.randn(self.local, C, lora_rank) * 0.01)
        self.lora_B = nn.Parameter(torch.zeros(self.local, lora_rank, C))
        self.router = gpu_moe.Router(C, n_experts, top_k)
        self.ops = ops or GpuOps

    @torch.no_grad()
    def load_experts(self, A_all: torch.Tensor, B_all: torch.Tensor):
        """Take this rank's slice of full (E, C, R) / (E, R, C) adapter tensors."""
        lo, hi = self.rank * self.local, (self.rank + 1) * self.local
        self.lora_A.copy_(A_all[lo:hi])
        self.lora_B.copy_(B_all[lo:hi])

    def forward(self, x: torch.Tensor):
        gpu_moe.check_forward_only("ExpertParallelLoRAMoE", x, (self.lora_A, self.lora_B, self.router.gate.weight))
        ops, g, k, E, El = self.ops, self.group, self.top_k, self.n_experts, self.local
        B, T, C = x.shape
        ntok = B * T
        x2 = x.reshape(ntok, C).contiguous()
        with torch.no_grad():
            base_out = self.base(x).reshape(ntok, C).contiguous()
        r = ops.router(x2, self.router.gate.weight, k, self.router.bias)
        inds, scores = r["inds"], r["scores"]
        perm, inv, offsets = ops.permute(inds, E)
        bounds = offsets[0:E + 1:El].to(torch.int64)
        send_counts = (bounds[1:] - bounds[:-1]).contiguous()
        recv_counts = torch.empty_like(send_counts)
        _a2a(recv_counts, send_counts, None, None, g)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        n_send, n_recv = sum(sc), sum(rc)

        x_send = ops.gather_rows(x2, perm, k)
        e_send = inds.reshape(-1)[perm.long()].contiguous()
        x_recv = _a2a(x2.new_empty((n_recv, C)), x_send, rc, sc, g)
        e_recv = _a2a(e_send.new_empty((n_recv,)), e_send, rc, sc, g)
        if n_recv:
            e_loc = (e_recv - self.rank * El).reshape(-1, 1).to(torch.int32).contiguous()
            y_recv = None
            if hasattr(ops, "apply_local"):
                y_recv = ops.apply_local(x_recv, self.lora_A.detach().to(x.dtype), self.lora_B.detach().to(x.dtype), e_loc)
            if y_recv is None:  # sorted by local expert: grouped down, then up in arrival order
                perm2, _, off2 = ops.permute(e_loc, El)
                h = ops.lora_down(x_recv, self.lora_A.detach(), perm2, off2)
                y_recv = ops.lora_up(h, self.lora_B.detach(), off2, perm2, x.dtype)
        else:
            y_recv = x2.new_empty((0, C))
        y_back = _a2a(x2.new_empty((n_send, C)), y_recv, sc, rc, g)
        out = ops.combine_rows(base_out, y_back, scores, inv)

        # aux / z over the whole (all-rank) batch
        p_loc = torch.softmax(r["logits"].float(), -1).sum(0)
        cnt = r.get("counts")  # per-expert counts from the router (no device -> host sync)
        f_cnt = (cnt if cnt is not None else torch.bincount(inds.reshape(-1).long(), minlength=E)).to(p_loc.dtype)
        z_sum = r["z"].float() * ntok
        red = torch.cat([p_loc, f_cnt, z_sum.reshape(1), torch.tensor([float(ntok)], device=p_loc.device)])
        dist.all_reduce(red, group=g)
        ntot = red[-1]
        p_e, f_e = red[:E] / ntot, red[E:2 * E] / (ntot * k)
        aux = E * (f_e * p_e).sum()
        z = red[2 * E] / ntot
        return out.reshape(B, T, C), aux, z

    def orthogonal_loss(self) -> torch.Tensor:
        """Sum over all expert pairs (moe.py:149-163): gathers every rank's A."""
        parts = [torch.empty_like(self.lora_A) for _ in range(self.ws)]
        dist.all_gather(parts, self.lora_A.detach().contiguous(), group=self.group)
        return self.ops.ortho_loss(torch.cat(parts))
