"""WKV-7 operators with the reference's call signatures, on the sm_100a kernels.

Reference interface (rwkv_mlx):
  * ``wkv7_metal_forward(r, w, k, v, a, b, head_size=64) -> (y, s, sa)``
    (kernels/wkv7_metal.py:250-279)                      -> :func:`wkv7_forward`
  * ``wkv7_metal_backward(r, w, k, v, a, b, dy, s, sa, head_size=64)``
    (kernels/wkv7_metal.py:282-319)                      -> :func:`wkv7_backward`
  * ``wkv7_metal(r, w, k, v, a, b, head_size=64)`` (:322-326) -> :func:`wkv7`
  * ``wkv7_recurrent(r, w, k, v, a, b, head_size=64)`` with the custom VJP of
    ``_wkv7_custom`` (model.py:81-116)                  -> :func:`wkv7_recurrent`
  * the state update of ``_time_mixing_rnn`` (model.py:475-483) -> :func:`wkv7_step`

Inputs are torch CUDA tensors shaped (B, T, C) with C = H * 64.  ``w`` is the
log-log decay (decay = exp(-exp(w))).  Unlike the reference, the backward is
exact (states are replayed from checkpoints rather than reconstructed by
dividing by the decay), any T is accepted (the reference's backward silently
needs T % 16 == 0), and an initial / final state can be passed in / out.
"""

from __future__ import annotations

import torch

from . import _native as nat

HEAD_SIZE = 64
CKPT_LEN = 16  # snapshot interval; 16 reproduces the reference's `s` layout exactly


def _check_head(head_size: int):
    if head_size != HEAD_SIZE:
        # same contract as the reference's assert (model.py:115)
        raise AssertionError(f"WKV kernel only supports head_size=64, got {head_size}")


def _prep(r, w, k, v, a, b, head_size):
    _check_head(head_size)
    if r.dim() != 3:
        raise ValueError("expected (B, T, C) tensors")
    B, T, C = r.shape
    if C % head_size:
        raise ValueError(f"C={C} is not a multiple of head_size={head_size}")
    dt = r.dtype
    if dt not in nat.DTYPE_CODE:
        raise TypeError(f"unsupported dtype {dt}")
    xs = []
    for name, t in zip("rkvab", (r, k, v, a, b)):
        if t.shape != r.shape:
            raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(r.shape)}")
        if not t.is_cuda:
            raise nat.RwkvNativeError("inputs must be CUDA tensors (no CPU fallback)")
        xs.append(t.to(dt).contiguous())
    if w.shape != r.shape:
        raise ValueError("w shape mismatch")
    w = w.contiguous() if w.dtype in (dt, torch.float32) else w.to(torch.float32).contiguous()
    return B, T, C // head_size, xs, w


def _fwd(r, w, k, v, a, b, head_size=64, s0=None, want_ckpt=True, want_sa=False,
         want_state=False, ckpt_len=CKPT_LEN):
    B, T, H, (r, k, v, a, b), w = _prep(r, w, k, v, a, b, head_size)
    dev = r.device
    y = torch.empty_like(r)
    nck = T // ckpt_len
    ckpt = torch.empty(B * H * nck * 64 * 64, device=dev, dtype=torch.float32) if want_ckpt else None
    sa = torch.empty((B, T, H, 64), device=dev, dtype=torch.float32) if want_sa else None
    sT = torch.empty((B, H, 64, 64), device=dev, dtype=torch.float32) if want_state else None
    if s0 is not None:
        s0 = s0.to(torch.float32).contiguous()
        if s0.numel() != B * H * 64 * 64:
            raise ValueError("s0 must be (B, H, 64, 64)")
    L = nat.lib()
    # segments of the sequence run in parallel when B*H leaves SMs idle (workspace > 0)
    ws_bytes = L.rwkv_wkv7_forward_workspace_size(B, T, H, 64, nat.dtype_code(r))
    ws = torch.empty((ws_bytes + 3) // 4, device=dev, dtype=torch.float32) if ws_bytes else None
    ev = _timing_events(dev)
    with torch.cuda.device(dev):
        if ev:
            ev[0].record()
        rc = L.rwkv_wkv7_forward_ws(
            nat.ptr(r), nat.ptr(w), nat.ptr(k), nat.ptr(v), nat.ptr(a), nat.ptr(b), nat.ptr(s0),
            nat.ptr(y), nat.ptr(sT), nat.ptr(ckpt) if (ckpt is not None and ckpt.numel()) else None,
            nat.ptr(sa), B, T, H, 64, nat.dtype_code(r), nat.dtype_code(w), ckpt_len,
            nat.ptr(ws), ws_bytes, nat.stream_ptr(dev))
        if ev:
            ev[1].record()
    nat.check(rc, "rwkv_wkv7_forward_ws", kernels=3 if ws_bytes else 1)
    return y, ckpt, sa, sT


# Optional per-launch CUDA-event timing of the forward kernel (used by bench.py to
# measure the kernel inside the timed region, on the stream it is launched on).
fwd_timings: list | None = None


def _timing_events(dev):
    if fwd_timings is None:
        return None
    pair = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    fwd_timings.append(pair)
    return pair


def _bwd(r, w, k, v, a, b, dy, ckpt, head_size=64, s0=None, dsT=None, want_ds0=False,
         ckpt_len=CKPT_LEN):
    B, T, H, (r, k, v, a, b), w = _prep(r, w, k, v, a, b, head_size)
    dev = r.device
    dy = dy.to(r.dtype).contiguous()
    grads = [torch.empty_like(r) for _ in range(6)]
    ds0 = torch.empty((B, H, 64, 64), device=dev, dtype=torch.float32) if want_ds0 else None
    if s0 is not None:
        s0 = s0.to(torch.float32).contiguous()
    if dsT is not None:
        dsT = dsT.to(torch.float32).contiguous()
    if ckpt is not None:
        ckpt = ckpt.contiguous()
        if ckpt.numel() != B * H * (T // ckpt_len) * 64 * 64:
            raise ValueError("checkpoint buffer does not match (B, H, T // ckpt_len, 64, 64)")
    L = nat.lib()
    ws_bytes = L.rwkv_wkv7_backward_workspace_size(B, T, H, 64)
    ws = torch.empty(max(1, (ws_bytes + 3) // 4), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        rc = L.rwkv_wkv7_backward_ws(
            nat.ptr(r), nat.ptr(w), nat.ptr(k), nat.ptr(v), nat.ptr(a), nat.ptr(b), nat.ptr(dy),
            nat.ptr(s0), nat.ptr(dsT), nat.ptr(ckpt) if (ckpt is not None and ckpt.numel()) else None,
            *[nat.ptr(g) for g in grads], nat.ptr(ds0), B, T, H, 64, nat.dtype_code(r),
            nat.dtype_code(w), ckpt_len, nat.ptr(ws), ws_bytes, nat.stream_ptr(dev))
        kernels = L.rwkv_wkv7_backward_launch_count(B, T, H, 64)  # depends on the device's SM count
    nat.check(rc, "rwkv_wkv7_backward_ws", kernels=kernels)
    # dw is produced in r.dtype like the reference's (wkv7_metal.py:317), whatever w's dtype
    return tuple(grads), ds0


def wkv7_forward(r, w, k, v, a, b, head_size: int = 64):
    """Mirror of ``wkv7_metal_forward``: returns ``(y, s, sa)``.

    ``y`` is (B, T, C) in r.dtype; ``s`` the flat fp32 state snapshots after every
    16th step (same size and layout as the reference's, wkv7_metal.py:276-278);
    ``sa`` (B, T, H, 64) fp32 with sa_t = S_{t-1} a_t.
    """
    y, s, sa, _ = _fwd(r, w, k, v, a, b, head_size, want_ckpt=True, want_sa=True)
    return y, s, sa


def wkv7_backward(r, w, k, v, a, b, dy, s, sa=None, head_size: int = 64):
    """Mirror of ``wkv7_metal_backward``: returns ``(dr, dw, dk, dv, da, db)``.

    ``s`` is the snapshot buffer from :func:`wkv7_forward`; ``sa`` is accepted for
    signature compatibility and not needed (states are replayed exactly).
    """
    grads, _ = _bwd(r, w, k, v, a, b, dy, s, head_size)
    return grads


def wkv7(r, w, k, v, a, b, head_size: int = 64):
    """Forward only (mirror of the legacy ``wkv7_metal``)."""
    y, _, _, _ = _fwd(r, w, k, v, a, b, head_size, want_ckpt=False)
    return y


def wkv7_with_state(r, w, k, v, a, b, s0=None, head_size: int = 64):
    """Forward from an initial state ``s0`` (B, H, 64, 64); returns ``(y, sT)``.

    Hands a GPT-mode prefill to RNN-mode decoding (the reference has no way to do
    this: its forward always starts from zero and returns no state)."""
    y, _, _, sT = _fwd(r, w, k, v, a, b, head_size, s0=s0, want_ckpt=False, want_state=True)
    return y, sT


class _WKV7Function(torch.autograd.Function):
    """Autograd boundary of ``_wkv7_custom`` (model.py:81-98).

    The reference's VJP re-runs the forward to regenerate its saved tensors
    (model.py:93-94); here the forward keeps its snapshots instead."""

    @staticmethod
    def forward(ctx, r, w, k, v, a, b):
        y, ckpt, _, _ = _fwd(r, w, k, v, a, b, HEAD_SIZE, want_ckpt=True)
        ctx.save_for_backward(r, w, k, v, a, b, ckpt)
        ctx.w_dtype = w.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        r, w, k, v, a, b, ckpt = ctx.saved_tensors
        (dr, dw, dk, dv, da, db), _ = _bwd(r, w, k, v, a, b, dy, ckpt, HEAD_SIZE)
        return dr, dw.to(ctx.w_dtype), dk, dv, da, db


def wkv7_recurrent(r, w, k, v, a, b, head_size: int = 64):
    """Mirror of ``wkv7_recurrent`` (model.py:101-116): y = WKV7(r, w, k, v, a, b)
    with an exact backward through autograd."""
    _check_head(head_size)
    if torch.is_grad_enabled() and any(t.requires_grad for t in (r, w, k, v, a, b)):
        return _WKV7Function.apply(r, w, k, v, a, b)
    # inference: no snapshots are written
    return _fwd(r, w, k, v, a, b, head_size, want_ckpt=False)[0]


def wkv7_step(S, r, w, k, v, a, b, w_is_decay: bool = True):
    """Batched single-token WKV-7 step; ``S`` (Bs, H, 64, 64) fp32 is updated in place.

    ``r, w, k, v, a, b`` are (Bs, H*64) or (Bs, H, 64).  With ``w_is_decay`` (the
    RNN-mode convention of model.py:476-477) ``w`` is the decay itself, otherwise
    the log-log w of GPT mode.  Returns y (Bs, H*64) in r.dtype, computed from the
    updated state (model.py:482-483)."""
    if S.dtype != torch.float32 or not S.is_contiguous() or S.dim() != 4 or S.shape[-1] != 64:
        raise ValueError("S must be a contiguous fp32 (Bs, H, 64, 64) tensor")
    Bs, H = S.shape[0], S.shape[1]
    dt = r.dtype
    xs = [t.reshape(Bs, H * 64).to(dt).contiguous() for t in (r, k, v, a, b)]
    w = w.reshape(Bs, H * 64)
    w = w.contiguous() if w.dtype in (dt, torch.float32) else w.to(torch.float32).contiguous()
    y = torch.empty_like(xs[0])
    L = nat.lib()
    with torch.cuda.device(S.device):
        rc = L.rwkv_wkv7_step(nat.ptr(S), nat.ptr(xs[0]), nat.ptr(w), nat.ptr(xs[1]),
                              nat.ptr(xs[2]), nat.ptr(xs[3]), nat.ptr(xs[4]), nat.ptr(y), Bs, H,
                              64, nat.dtype_code(xs[0]), nat.dtype_code(w),
                              1 if w_is_decay else 0, nat.stream_ptr(S.device))
    nat.check(rc, "rwkv_wkv7_step")
    return y
