"""WKV-7 CUDA kernels vs the float64 oracle (parity tests proper; need a B200).

Tolerances are relative to the RMS of the oracle output.  The step-sequential
kernels compute in fp32 throughout: fp32 inputs 2e-5.  The chunked tensor-core
kernels use TF32 operands (fp32 accumulate, fp32 state): 2e-3 for fp32 and fp16
inputs (the north-star bound for fp16 inputs with fp32 state).  bf16 inputs 6e-3
(bf16 output rounding alone is ~2e-3).
"""

import numpy as np
import pytest
import torch

from oracle import wkv7_oracle as wo
from tests.inputs import rel_rms, wkv_inputs

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 2e-3, torch.float16: 2e-3, torch.bfloat16: 6e-3}  # default (chunked) path
TOL_SEQ = {torch.float32: 2e-5, torch.float16: 2e-3, torch.bfloat16: 6e-3}


def _dev(x, dt):
    return torch.tensor(np.ascontiguousarray(x), dtype=dt, device="cuda")


def _bt(x):  # (B,T,H,N) -> (B,T,C)
    return x.reshape(x.shape[0], x.shape[1], -1)


def _rounded(inp, dt, w_dt=None):
    """Device tensors in dt (w in w_dt) and the float64 values they hold."""
    dev, host = {}, {}
    for n, x in inp.items():
        t = _dev(_bt(x), w_dt if (n == "w" and w_dt is not None) else dt)
        dev[n] = t
        host[n] = t.double().cpu().numpy().reshape(x.shape)
    return dev, host


@pytest.mark.parametrize("impl", [1, 2, 3])
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B,T,H", [(1, 256, 4), (2, 100, 3), (1, 17, 1)])
def test_forward_matches_oracle(dt, B, T, H, impl):
    """impl 1: step-sequential, 2: chunked on mma.sync, 3: chunked on tcgen05 (fp16/bf16)."""
    from rwkv_mlx_b200 import wkv7

    if impl == 3 and dt == torch.float32:
        pytest.skip("the tcgen05 kernel takes fp16/bf16 activations")
    d, h = _rounded(wkv_inputs(B, T, H, seed=B * 1000 + T), dt)
    _set_impl(impl)
    try:
        y, s, sa = wkv7.wkv7_forward(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"])
        torch.cuda.synchronize()
    finally:
        _set_impl(0)
    tol = (TOL_SEQ if impl == 1 else TOL)[dt]
    ye, sae, _, states = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], keep_states=True)
    assert rel_rms(y.double().cpu().numpy(), _bt(ye)) < tol
    assert rel_rms(sa.cpu().numpy(), sae) < max(tol, 1e-5)
    if T >= 16:
        ck = wo.checkpoints_from_states(states, 16).reshape(-1)
        assert rel_rms(s.cpu().numpy(), ck) < max(tol, 1e-5)


def test_forward_fp32_decay_with_fp16_inputs():
    """w in fp32 with the other inputs in fp16 (what the model feeds)."""
    from rwkv_mlx_b200 import wkv7

    d, h = _rounded(wkv_inputs(2, 128, 2, seed=7), torch.float16, w_dt=torch.float32)
    assert d["w"].dtype == torch.float32
    y = wkv7.wkv7(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"])
    ye = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"])[0]
    assert rel_rms(y.double().cpu().numpy(), _bt(ye)) < TOL[torch.float16]


def test_state_in_out_composes():
    """Running T as two halves with the state handed over equals one pass."""
    from rwkv_mlx_b200 import wkv7

    d, h = _rounded(wkv_inputs(2, 96, 2, seed=3), torch.float32)
    y, sT = wkv7.wkv7_with_state(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"])
    half = {n: t[:, :40] for n, t in d.items()}
    rest = {n: t[:, 40:] for n, t in d.items()}
    y1, s1 = wkv7.wkv7_with_state(half["r"], half["w"], half["k"], half["v"], half["a"], half["b"])
    y2, s2 = wkv7.wkv7_with_state(rest["r"], rest["w"], rest["k"], rest["v"], rest["a"], rest["b"], s0=s1)
    ye, _, sTe, _ = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"])
    assert rel_rms(torch.cat([y1, y2], 1).cpu().numpy(), _bt(ye)) < TOL[torch.float32]
    assert rel_rms(s2.cpu().numpy(), sTe) < TOL[torch.float32]
    assert rel_rms(sT.cpu().numpy(), sTe) < TOL[torch.float32]


@pytest.mark.parametrize("dt", [torch.float32, torch.float16])
@pytest.mark.parametrize("B,T,H", [(1, 256, 4), (2, 72, 2), (1, 9, 1)])
def test_backward_matches_exact_oracle(dt, B, T, H):
    from rwkv_mlx_b200 import wkv7

    inp = wkv_inputs(B, T, H, seed=11 + T)
    d, h = _rounded(inp, dt)
    y, s, sa = wkv7.wkv7_forward(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"])
    grads = wkv7.wkv7_backward(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], d["dy"], s, sa)
    torch.cuda.synchronize()
    ge = wo.wkv7_backward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], h["dy"])
    for name, g, e in zip(["dr", "dw", "dk", "dv", "da", "db"], grads, ge[:6]):
        err = rel_rms(g.double().cpu().numpy(), _bt(e))
        assert err < TOL[dt], f"{name}: {err}"


def test_autograd_function_and_state_grads():
    from rwkv_mlx_b200 import wkv7

    d, h = _rounded(wkv_inputs(1, 48, 2, seed=5), torch.float32)
    leaves = {n: d[n].clone().requires_grad_(True) for n in "rwkvab"}
    y = wkv7.wkv7_recurrent(*[leaves[n] for n in "rwkvab"])
    y.backward(d["dy"])
    ge = wo.wkv7_backward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], h["dy"])
    for n, e in zip("rwkvab", ge[:6]):
        assert rel_rms(leaves[n].grad.double().cpu().numpy(), _bt(e)) < TOL[torch.float32], n


def test_backward_with_initial_state_and_state_grad():
    from rwkv_mlx_b200 import wkv7

    B, T, H = 1, 40, 2
    d, h = _rounded(wkv_inputs(B, T, H, seed=21), torch.float32)
    rng = np.random.default_rng(1)
    s0 = rng.standard_normal((B, H, 64, 64)) * 0.3
    dsT = rng.standard_normal((B, H, 64, 64)) * 0.1
    s0d, dsTd = _dev(s0, torch.float32), _dev(dsT, torch.float32)
    _, ck, _, _ = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], s0=s0d)
    grads, ds0 = wkv7._bwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], d["dy"], ck,
                           s0=s0d, dsT=dsTd, want_ds0=True)
    ge = wo.wkv7_backward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], h["dy"], s0=s0, dsT=dsT)
    for name, g, e in zip(["dr", "dw", "dk", "dv", "da", "db"], grads, ge[:6]):
        assert rel_rms(g.double().cpu().numpy(), _bt(e)) < TOL[torch.float32], name
    assert rel_rms(ds0.cpu().numpy(), ge[6]) < TOL[torch.float32]


@pytest.mark.parametrize("dt", [torch.float32, torch.float16])
def test_step_matches_oracle(dt):
    from rwkv_mlx_b200 import wkv7

    rng = np.random.default_rng(4)
    Bs, H = 5, 3
    S0 = rng.standard_normal((Bs, H, 64, 64))
    inp = {n: rng.standard_normal((Bs, H, 64)) for n in "rkv"}
    kk = rng.standard_normal((Bs, H, 64))
    kk /= np.linalg.norm(kk, axis=-1, keepdims=True)
    inp["a"], inp["b"] = -kk, kk * 0.6
    inp["w"] = np.exp(-0.606531 / (1 + np.exp(-rng.standard_normal((Bs, H, 64)))))
    S = _dev(S0, torch.float32)
    d = {n: _dev(x.reshape(Bs, -1), dt) for n, x in inp.items()}
    dw32 = _dev(inp["w"].reshape(Bs, -1), torch.float32)
    hv = {n: d[n].double().cpu().numpy().reshape(Bs, H, 64) for n in d}
    y = wkv7.wkv7_step(S, d["r"], dw32, d["k"], d["v"], d["a"], d["b"], w_is_decay=True)
    ye, Se = wo.wkv7_step_exact(S0, hv["r"], inp["w"], hv["k"], hv["v"], hv["a"], hv["b"])
    assert rel_rms(S.cpu().numpy(), Se) < 1e-6
    assert rel_rms(y.double().cpu().numpy().reshape(Bs, H, 64), ye) < TOL[dt]


def test_step_chain_equals_forward():
    """T single steps (log-log w) reproduce the sequence kernel's y and final state."""
    from rwkv_mlx_b200 import wkv7

    B, T, H = 3, 20, 2
    d, _ = _rounded(wkv_inputs(B, T, H, seed=9), torch.float32)
    y, sT = wkv7.wkv7_with_state(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"])
    S = torch.zeros(B, H, 64, 64, device="cuda")
    ys = []
    for t in range(T):
        ys.append(wkv7.wkv7_step(S, *[d[n][:, t] for n in "rwkvab"], w_is_decay=False))
    assert rel_rms(torch.stack(ys, 1).cpu().numpy(), y.cpu().numpy()) < TOL[torch.float32]
    assert rel_rms(S.cpu().numpy(), sT.cpu().numpy()) < TOL[torch.float32]


def test_bad_head_size_raises():
    from rwkv_mlx_b200 import wkv7

    x = torch.zeros(1, 4, 96, device="cuda")
    with pytest.raises(AssertionError):
        wkv7.wkv7_recurrent(x, x, x, x, x, x, head_size=32)


def _set_impl(i):
    from rwkv_mlx_b200 import _native

    assert _native.lib().rwkv_set_wkv_impl(i) == 0


@pytest.mark.parametrize("B,T,H", [(2, 64, 3), (1, 333, 2), (3, 16, 1), (1, 1, 1)])
def test_chunked_and_sequential_kernels_agree(B, T, H):
    from rwkv_mlx_b200 import _native, wkv7

    d, h = _rounded(wkv_inputs(B, T, H, seed=T + 17), torch.float32)
    outs = {}
    try:
        for impl in (1, 2):
            _set_impl(impl)
            outs[impl] = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], want_ckpt=True,
                                   want_sa=True, want_state=True)
    finally:
        _set_impl(0)
    torch.cuda.synchronize()
    assert _native.lib().rwkv_device_error(1) == 0
    ye, sae, sTe, st = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], keep_states=True)
    for impl, (y, ck, sa, sT) in outs.items():
        assert rel_rms(y.cpu().numpy(), _bt(ye)) < 2e-3, impl  # chunked: TF32 operands
        assert rel_rms(sa.cpu().numpy(), sae) < 2e-3, impl
        assert rel_rms(sT.cpu().numpy(), sTe) < 2e-3, impl
        if T >= 16:
            assert rel_rms(ck.cpu().numpy(), wo.checkpoints_from_states(st, 16).reshape(-1)) < 2e-3, impl


@pytest.mark.parametrize("dt", [torch.float32, torch.float16])
def test_chunked_kernel_extreme_decays(dt):
    """Per-step decays down to exp(-exp(3)) ~ 2e-9: chunks whose cumulative decay
    leaves the factored range take the element-wise path and stay exact (fp32 inputs:
    mma.sync kernel; fp16: tcgen05 kernel)."""
    from rwkv_mlx_b200 import _native, wkv7

    d, h = _rounded(wkv_inputs(1, 80, 2, seed=8, w_lo=-1.0, w_hi=3.0), dt, w_dt=torch.float32)
    y = wkv7.wkv7(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"])
    torch.cuda.synchronize()
    assert _native.lib().rwkv_device_error(1) == 0
    ye = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"])[0]
    assert rel_rms(y.double().cpu().numpy(), _bt(ye)) < TOL[dt]


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_long_sequence_error_stays_bounded(dt):
    """T = 4096 (256 chunks): TF32 rounding of the chunk operands must not build up
    along the state chain (slow decays keep old state alive the longest)."""
    from rwkv_mlx_b200 import _native, wkv7

    d, h = _rounded(wkv_inputs(1, 4096, 2, seed=21, w_lo=-6.0, w_hi=-3.0), dt, w_dt=torch.float32)
    y, _, sa, sT = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], want_sa=True, want_state=True)
    torch.cuda.synchronize()
    assert _native.lib().rwkv_device_error(1) == 0
    ye, sae, sTe, _ = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"])
    assert rel_rms(y.double().cpu().numpy(), _bt(ye)) < TOL[dt]
    assert rel_rms(sa.cpu().numpy(), sae) < 2e-3
    assert rel_rms(sT.cpu().numpy(), sTe) < 2e-3


def test_misaligned_inputs_use_the_sequential_kernel():
    from rwkv_mlx_b200 import wkv7

    B, T, H = 1, 40, 1
    d, h = _rounded(wkv_inputs(B, T, H, seed=12), torch.float32)
    # storage offset of one element: not 16-byte aligned
    shifted = {}
    for n in "rwkvab":
        buf = torch.empty(d[n].numel() + 1, device="cuda", dtype=torch.float32)
        buf[1:] = d[n].reshape(-1)
        shifted[n] = buf[1:].view(B, T, H * 64)
    y = wkv7.wkv7(*[shifted[n] for n in "rwkvab"])
    ye = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"])[0]
    assert rel_rms(y.cpu().numpy(), _bt(ye)) < 2e-5


@pytest.mark.parametrize("T", [16, 48, 333, 1024])
def test_tcgen05_kernel_with_state_and_checkpoints(T):
    """tcgen05 forward with an initial state, final state, sa and 16-step snapshots (fp16)."""
    from rwkv_mlx_b200 import _native, wkv7

    B, H = 2, 3
    d, h = _rounded(wkv_inputs(B, T, H, seed=T), torch.float16, w_dt=torch.float32)
    rng = np.random.default_rng(T)
    s0 = rng.standard_normal((B, H, 64, 64)) * 0.5
    _set_impl(3)
    try:
        y, ck, sa, sT = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], s0=_dev(s0, torch.float32),
                                  want_ckpt=True, want_sa=True, want_state=True)
        torch.cuda.synchronize()
    finally:
        _set_impl(0)
    assert _native.lib().rwkv_device_error(1) == 0
    ye, sae, sTe, st = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], s0=s0, keep_states=True)
    assert rel_rms(y.double().cpu().numpy(), _bt(ye)) < 2e-3
    assert rel_rms(sa.cpu().numpy(), sae) < 2e-3
    assert rel_rms(sT.cpu().numpy(), sTe) < 2e-3
    if T >= 16:
        assert rel_rms(ck.cpu().numpy(), wo.checkpoints_from_states(st, 16).reshape(-1)) < 2e-3


@pytest.mark.parametrize("scale_s,scale_v,scale_ab", [(3e4, 300.0, 1.0), (1e-6, 1e-4, 1.0), (1.0, 1.0, 1.4)])
def test_tcgen05_kernel_across_ranges(scale_s, scale_v, scale_ab):
    """fp16 activations with states far outside the fp16 range (entries ~1e5), tiny
    states, and larger |a|, |b| (larger triangular-solve entries): the state and the
    TF32 operands are fp32-ranged, so accuracy does not depend on the magnitudes."""
    from rwkv_mlx_b200 import _native, wkv7

    B, T, H = 2, 160, 2
    inp = wkv_inputs(B, T, H, seed=31)
    inp["v"] = inp["v"] * scale_v
    inp["a"] = inp["a"] * scale_ab
    inp["b"] = inp["b"] * scale_ab
    d, h = _rounded(inp, torch.float16, w_dt=torch.float32)
    rng = np.random.default_rng(5)
    s0 = rng.standard_normal((B, H, 64, 64)) * scale_s
    y, _, sa, sT = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], s0=_dev(s0, torch.float32),
                             want_sa=True, want_state=True)
    torch.cuda.synchronize()
    assert _native.lib().rwkv_device_error(1) == 0
    ye, sae, sTe, _ = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], s0=s0)
    if np.abs(ye).max() < 6e4:  # y itself is an fp16 output
        assert rel_rms(y.double().cpu().numpy(), _bt(ye)) < 2e-3
    assert rel_rms(sa.cpu().numpy(), sae) < 2e-3
    assert rel_rms(sT.cpu().numpy(), sTe) < 2e-3
