"""Python front-ends of the fused element-wise kernels (csrc/fused.cu) and of the
tcgen05 grouped GEMM (csrc/gemm_tc.cu).

They replace chains of separate torch element-wise passes in the block around the
WKV-7 call (rwkv_mlx/model.py:187-263, 312-327); see include/rwkv_b200.h for the
exact formulas.  Activations are contiguous CUDA tensors (B, T, C) or (rows, C).
"""

from __future__ import annotations

import torch

from . import _native as nat


def _call(name, *args):
    rc = getattr(nat.lib(), name)(*args)
    nat.check(rc, name)


def lerp(x: torch.Tensor, mix: torch.Tensor, T: int, prev: torch.Tensor = None,
         prev_out: torch.Tensor = None) -> torch.Tensor:
    """x (..., C) with rows grouped in sequences of length T; mix (M, C) -> (M, rows, C).
    ``prev`` (rows / T, C): the token before each sequence (zeros when None).
    ``prev_out`` (rows / T, C): receives each sequence's last row of x, the next shift
    state (may be ``prev`` when T == 1: an RNN state updated in place)."""
    C = x.shape[-1]
    x = x.contiguous()
    rows = x.numel() // C
    mix = mix.to(x.dtype).contiguous().view(-1, C)
    out = torch.empty((mix.shape[0], rows, C), device=x.device, dtype=x.dtype)
    if prev is not None:
        prev = prev.to(x.dtype).contiguous()  # a copy only for another dtype / layout
    direct = prev_out is not None and prev_out.dtype == x.dtype and prev_out.is_contiguous()
    if prev is None and prev_out is None:
        _call("rwkv_lerp", nat.ptr(x), nat.ptr(mix), nat.ptr(out), mix.shape[0], rows, T, C, nat.dtype_code(x),
              nat.stream_ptr(x.device))
    else:
        _call("rwkv_lerp_prev_state", nat.ptr(x), nat.ptr(prev), nat.ptr(mix), nat.ptr(out),
              nat.ptr(prev_out if direct else None), mix.shape[0], rows, T, C, nat.dtype_code(x),
              nat.stream_ptr(x.device))
    if prev_out is not None and not direct:
        prev_out.copy_(x.view(rows // T, T, C)[:, -1].reshape(prev_out.shape))
    return out


def tmix_mid(k, v, wl, al, vl, v_first, w0, a0, v0, k_k, k_a, layer0: bool):
    C = k.shape[-1]
    rows = k.numel() // C
    dt = k.dtype
    c = lambda t: None if t is None else t.to(dt).contiguous()
    w_out = torch.empty(k.shape, device=k.device, dtype=torch.float32)
    k_out, v_out, a_out, b_out = (torch.empty_like(k) for _ in range(4))
    args = [c(k), c(v), c(wl), c(al), c(vl), c(v_first)]
    _call("rwkv_tmix_mid", *[nat.ptr(t) for t in args], nat.ptr(w0.float().contiguous()), nat.ptr(c(a0)),
          nat.ptr(c(v0)), nat.ptr(c(k_k)), nat.ptr(c(k_a)), nat.ptr(w_out), nat.ptr(k_out), nat.ptr(v_out),
          nat.ptr(a_out), nat.ptr(b_out), rows, C, 1 if layer0 else 0, nat.dtype_code(k), nat.stream_ptr(k.device))
    return w_out, k_out, v_out, a_out, b_out


def tmix_post(y, r, k, v, g, ln_w, ln_b, r_k, H: int, eps: float, per_head: bool):
    C = y.shape[-1]
    rows = y.numel() // C
    dt = y.dtype
    c = lambda t: t.to(dt).contiguous()
    out = torch.empty_like(y)
    _call("rwkv_tmix_post", nat.ptr(c(y)), nat.ptr(c(r)), nat.ptr(c(k)), nat.ptr(c(v)), nat.ptr(c(g)),
          nat.ptr(c(ln_w)), nat.ptr(c(ln_b)), nat.ptr(c(r_k)), nat.ptr(out), rows, C, H, float(eps),
          1 if per_head else 0, nat.dtype_code(y), nat.stream_ptr(y.device))
    return out


def lora_act_(h: torch.Tensor) -> torch.Tensor:
    """In place on the stacked LoRA hidden h (4, rows, D): tanh on h[1], sigmoid on h[3]."""
    _call("rwkv_lora_act", nat.ptr(h), h[0].numel(), nat.dtype_code(h), nat.stream_ptr(h.device))
    return h


def relu_sq_(x: torch.Tensor) -> torch.Tensor:
    _call("rwkv_relu_sq", nat.ptr(x), x.numel(), nat.dtype_code(x), nat.stream_ptr(x.device))
    return x


def add_layernorm(x, delta, w, b, eps: float = 1e-5):
    """Returns (x + delta, LayerNorm(x + delta)); with delta None returns (x, LayerNorm(x))."""
    C = x.shape[-1]
    rows = x.numel() // C
    x = x.contiguous()
    y = torch.empty_like(x)
    x_out = torch.empty_like(x) if delta is not None else None
    d = None if delta is None else delta.to(x.dtype).contiguous()
    _call("rwkv_add_layernorm", nat.ptr(x), nat.ptr(d), nat.ptr(w.to(x.dtype).contiguous()),
          nat.ptr(b.to(x.dtype).contiguous()), nat.ptr(x_out), nat.ptr(y), rows, C, float(eps), nat.dtype_code(x),
          nat.stream_ptr(x.device))
    return (x_out if delta is not None else x), y


def argmax_rows(x: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    """torch.argmax(x, -1) for 2-d x (first index of the maximum), int64, into ``out``."""
    rows, V = x.shape
    if x.stride(1) != 1:
        x = x.contiguous()
    if out is None:
        out = torch.empty(rows, device=x.device, dtype=torch.int64)
    _call("rwkv_argmax_rows", nat.ptr(x), x.stride(0), rows, V, nat.ptr(out), nat.dtype_code(x),
          nat.stream_ptr(x.device))
    return out


def grouped_gemm(a: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor | None = None, relu_sq: bool = False,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """out[m] = a[m] @ w[g]^T for the rows m in [offsets[g], offsets[g+1]) (squared ReLU of
    the product when ``relu_sq``), on the tcgen05 grouped GEMM (``rwkv_grouped_gemm``).
    a (M, K), w (G, N, K) fp16 / bf16; offsets (G+1,) int32 on the device, or None for
    one group over all rows.  Rows outside every group are left as they were in ``out``."""
    M, K = a.shape
    G, N, K2 = w.shape
    if K2 != K or (offsets is None and G != 1):
        raise ValueError("grouped_gemm: shape mismatch")
    if offsets is not None and (offsets.dtype != torch.int32 or offsets.numel() != G + 1
                                or not offsets.is_contiguous() or offsets.device != a.device):
        raise ValueError("grouped_gemm: offsets must be a contiguous int32 (G + 1,) tensor on a's device")
    a = a.contiguous()
    w = w.to(a.dtype).contiguous()
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=a.dtype)
    elif out.shape != (M, N) or out.stride(1) != 1 or out.dtype != a.dtype:
        raise ValueError("grouped_gemm: out must be (M, N) in a's dtype with unit column stride")
    L = nat.lib()
    with torch.cuda.device(a.device):
        rc = L.rwkv_grouped_gemm(nat.ptr(a), nat.ptr(w), nat.ptr(offsets), nat.ptr(out), M, N, K, G, out.stride(0),
                                 1 if relu_sq else 0, nat.dtype_code(a), nat.stream_ptr(a.device))
    nat.check(rc, "rwkv_grouped_gemm")
    return out
