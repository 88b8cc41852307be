"""Training loss of the reference on the chunked cross-entropy kernels (``csrc/loss.cu``).

Reference (rwkv_mlx/train.py):
  * ``l2_wrap_loss(logits, targets)`` (:317-334)             -> :func:`l2_wrap_loss`
  * ``l2_wrap_loss_masked(logits, targets, mask)`` (:337-362) -> :func:`l2_wrap_loss_masked`
    mean (or mask-weighted mean) cross-entropy + 1e-4 / (B*T) * 0.5 * sum (max logit)^2.

:func:`head_l2_wrap_loss` fuses the output head with the loss.  For fp16 / bf16 the
logits ``x @ head.weight^T`` are formed on the tcgen05 tensor cores and folded into
per-token softmax statistics inside the GEMM's epilogue (``rwkv_head_ce_stats``), so no
logit is ever written to memory (B=32, T=4096, V=65568 would need 17 GB of them in fp16);
the backward recomputes one vocabulary chunk at a time and the same kernel writes
``d loss / d logits`` directly (``rwkv_head_ce_grad``) before the two library products of
the head's gradient.  Other dtypes form each chunk with a library GEMM and fold it with
``rwkv_ce_chunk`` / ``rwkv_ce_chunk_grad``.  All three functions are autograd functions.
"""

from __future__ import annotations

import torch

from . import _native as nat

DEFAULT_CHUNK = 8192


def _i32(t):
    return t.reshape(-1).to(torch.int32).contiguous()


def _mask(m, n):
    return None if m is None else m.reshape(-1).to(torch.float32).contiguous()


def _chunk_stats(logits2d, ld, targets, state, col0, ncols, first):
    L = nat.lib()
    with torch.cuda.device(logits2d.device):
        rc = L.rwkv_ce_chunk(nat.ptr(logits2d), ld, nat.ptr(targets), nat.ptr(state), targets.numel(), col0, ncols,
                             1 if first else 0, nat.dtype_code(logits2d), nat.stream_ptr(logits2d.device))
    nat.check(rc, "rwkv_ce_chunk")


def _finalize(state, mask, l2_factor):
    out = torch.empty(4, device=state.device, dtype=torch.float32)
    L = nat.lib()
    with torch.cuda.device(state.device):
        rc = L.rwkv_ce_finalize(nat.ptr(state), nat.ptr(mask), float(l2_factor), nat.ptr(out), state.shape[0],
                                nat.stream_ptr(state.device))
    nat.check(rc, "rwkv_ce_finalize")
    return out


def _chunk_grad(logits2d, ld, targets, state, mask, out, g, l2_factor, scaled, dlog, col0, ncols):
    L = nat.lib()
    with torch.cuda.device(logits2d.device):
        rc = L.rwkv_ce_chunk_grad(nat.ptr(logits2d), ld, nat.ptr(targets), nat.ptr(state), nat.ptr(mask),
                                  nat.ptr(out), nat.ptr(g), float(l2_factor), 1 if scaled else 0, nat.ptr(dlog),
                                  dlog.stride(0), targets.numel(), col0, ncols, nat.dtype_code(dlog),
                                  nat.stream_ptr(logits2d.device))
    nat.check(rc, "rwkv_ce_chunk_grad")


_FP32_OUT = [True]  # the GEMM with a 16-bit product and an fp32 output is available


def _accumulate_fp32(acc, a, b):
    """acc (fp32) + a @ b for 16-bit a, b: one GEMM accumulating into fp32 where the
    library offers it, else the product in a's type added in fp32."""
    if _FP32_OUT[0]:
        try:
            return torch.addmm(acc, a, b, out_dtype=torch.float32)
        except (RuntimeError, TypeError, NotImplementedError):
            _FP32_OUT[0] = False
    return acc.add_(torch.mm(a, b).float())


class _LossOnLogits(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits2d, targets, mask, l2_factor):
        n, V = logits2d.shape
        state = torch.empty((n, 4), device=logits2d.device, dtype=torch.float32)
        _chunk_stats(logits2d, V, targets, state, 0, V, True)
        out = _finalize(state, mask, l2_factor)
        ctx.save_for_backward(logits2d, targets, state, out)
        ctx.mask, ctx.l2_factor = mask, l2_factor
        return out[0].clone()

    @staticmethod
    def backward(ctx, g):
        logits2d, targets, state, out = ctx.saved_tensors
        n, V = logits2d.shape
        dlog = torch.empty_like(logits2d)
        g = g.to(torch.float32).reshape(1).contiguous()
        _chunk_grad(logits2d, V, targets, state, ctx.mask, out, g, ctx.l2_factor, True, dlog, 0, V)
        return dlog, None, None, None


def _fused_ok(x2d, weight):
    """The tcgen05 head kernels take fp16 / bf16 operands of one dtype with C % 8 == 0."""
    return (x2d.dtype in (torch.float16, torch.bfloat16) and weight.dtype == x2d.dtype
            and x2d.shape[1] % 8 == 0 and weight.is_contiguous())


def _head_stats(x2d, weight, targets, state):
    n, C = x2d.shape
    V = weight.shape[0]
    L = nat.lib()
    ws_bytes = L.rwkv_head_ce_workspace_size(n, V)
    ws = torch.empty(max(16, ws_bytes), device=x2d.device, dtype=torch.uint8)
    with torch.cuda.device(x2d.device):
        rc = L.rwkv_head_ce_stats(nat.ptr(x2d), nat.ptr(weight), nat.ptr(targets), nat.ptr(state), n, V, C,
                                  nat.ptr(ws), ws_bytes, nat.dtype_code(x2d), nat.stream_ptr(x2d.device))
    nat.check(rc, "rwkv_head_ce_stats")


def _head_grad(x2d, w_chunk, targets, state, mask, out, g, l2_factor, dlog, col0):
    n, C = x2d.shape
    L = nat.lib()
    with torch.cuda.device(x2d.device):
        rc = L.rwkv_head_ce_grad(nat.ptr(x2d), nat.ptr(w_chunk), nat.ptr(targets), nat.ptr(state), nat.ptr(mask),
                                 nat.ptr(out), nat.ptr(g), float(l2_factor), 0, nat.ptr(dlog), dlog.stride(0), n,
                                 w_chunk.shape[0], C, col0, nat.dtype_code(x2d), nat.stream_ptr(x2d.device))
    nat.check(rc, "rwkv_head_ce_grad")


class _HeadLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2d, weight, targets, mask, l2_factor, chunk):
        n = x2d.shape[0]
        V = weight.shape[0]
        state = torch.empty((n, 4), device=x2d.device, dtype=torch.float32)
        if _fused_ok(x2d, weight):
            # logits and their softmax statistics in one tcgen05 launch: no logit in HBM
            _head_stats(x2d, weight, targets, state)
        else:
            for c0 in range(0, V, chunk):
                c1 = min(V, c0 + chunk)
                lg = torch.mm(x2d, weight[c0:c1].t())
                _chunk_stats(lg, c1 - c0, targets, state, c0, c1 - c0, c0 == 0)
        out = _finalize(state, mask, l2_factor)
        ctx.save_for_backward(x2d, weight, targets, state, out)
        ctx.mask, ctx.l2_factor, ctx.chunk = mask, l2_factor, chunk
        return out[0].clone()

    @staticmethod
    def backward(ctx, g):
        x2d, weight, targets, state, out = ctx.saved_tensors
        V = weight.shape[0]
        g = g.to(torch.float32).reshape(1).contiguous()
        dx = torch.zeros(x2d.shape, device=x2d.device, dtype=torch.float32)
        dw = torch.empty_like(weight)
        fused = _fused_ok(x2d, weight)
        for c0 in range(0, V, ctx.chunk):
            c1 = min(V, c0 + ctx.chunk)
            # unscaled d loss / d logits (O(1) entries); g / den is applied to the products
            if fused:  # logits recomputed and turned into gradients inside one tcgen05 launch
                lg = torch.empty((x2d.shape[0], c1 - c0), device=x2d.device, dtype=x2d.dtype)
                _head_grad(x2d, weight[c0:c1], targets, state, ctx.mask, out, g, ctx.l2_factor, lg, c0)
            else:
                lg = torch.mm(x2d, weight[c0:c1].t())
                _chunk_grad(lg, c1 - c0, targets, state, ctx.mask, out, g, ctx.l2_factor, False, lg, c0, c1 - c0)
            dx = _accumulate_fp32(dx, lg, weight[c0:c1])
            dw[c0:c1] = torch.mm(lg.t(), x2d)
        s = g / out[3]
        dx.mul_(s)
        dw.mul_(s.to(dw.dtype))
        return dx.to(x2d.dtype), dw, None, None, None, None


def l2_wrap_loss(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """logits (B, T, V), targets (B, T) -> scalar fp32 (train.py:317-334)."""
    B, T, V = logits.shape
    return _LossOnLogits.apply(logits.reshape(B * T, V).contiguous(), _i32(targets), None, 1e-4 / (B * T))


def l2_wrap_loss_masked(logits: torch.Tensor, targets: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """Cross-entropy over mask = 1 positions + the L2 term over all (train.py:337-362)."""
    B, T, V = logits.shape
    return _LossOnLogits.apply(logits.reshape(B * T, V).contiguous(), _i32(targets), _mask(mask, B * T),
                               1e-4 / (B * T))


def head_l2_wrap_loss(x: torch.Tensor, head_weight: torch.Tensor, targets: torch.Tensor,
                      mask: torch.Tensor | None = None, chunk: int = DEFAULT_CHUNK) -> torch.Tensor:
    """``l2_wrap_loss(x @ head_weight^T, targets)`` (masked when ``mask`` is given)
    without holding the (B, T, V) logits: x (B, T, C), head_weight (V, C)."""
    B, T, C = x.shape
    if chunk % 8:
        raise ValueError("chunk must be a multiple of 8")
    return _HeadLoss.apply(x.reshape(B * T, C).contiguous(), head_weight, _i32(targets), _mask(mask, B * T),
                           1e-4 / (B * T), chunk)
