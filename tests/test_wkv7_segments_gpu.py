"""Segment-parallel tcgen05 WKV-7 forward, segmented backward chain, and the abort path
(need a B200).

The sequence is cut into segments whose affine state maps are computed by a
transition pass and composed by a scan; every output (y, sa, 16-step snapshots,
final state) must match the float64 oracle run over the whole sequence, within the
chunked kernels' TF32 tolerance (2e-3 relative to RMS for fp16 and fp32, 6e-3 for
bf16).  The backward's adjoint chain is segmented the same way (affine maps of the
state gradient, composed top down); its gradients, including the initial-state
gradient with a final-state gradient given, must match the float64 oracle too.
"""

import numpy as np
import pytest
import torch

from oracle import wkv7_oracle as wo
from tests.inputs import rel_rms, wkv_inputs

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 6e-3}


def _bt(x):
    return x.reshape(x.shape[0], x.shape[1], -1)


def _inputs(B, T, H, seed, dt):
    inp = wkv_inputs(B, T, H, seed=seed)
    dev, host = {}, {}
    for n, x in inp.items():
        t = torch.tensor(_bt(x), dtype=torch.float32 if n == "w" else dt, device="cuda")
        dev[n], host[n] = t, t.double().cpu().numpy().reshape(x.shape)
    return dev, host


def _segments(n):
    from rwkv_mlx_b200 import _native

    _native.check(_native.lib().rwkv_set_wkv_segments(n), "rwkv_set_wkv_segments")


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B,T,H,nseg", [(1, 1024, 2, 3), (2, 777, 1, 5), (1, 2048, 3, 8), (1, 256, 1, 16)])
def test_segmented_forward_matches_oracle(dt, B, T, H, nseg):
    """Forced segment counts (including one chunk per segment and a ragged last
    segment), with an initial state, sa, snapshots and the final state."""
    from rwkv_mlx_b200 import _native, wkv7

    d, h = _inputs(B, T, H, seed=T + nseg, dt=dt)
    rng = np.random.default_rng(nseg)
    s0 = rng.standard_normal((B, H, 64, 64)) * 0.5
    s0d = torch.tensor(s0, dtype=torch.float32, device="cuda")
    _segments(nseg)
    try:
        assert _native.lib().rwkv_wkv7_forward_workspace_size(B, T, H, 64, _native.dtype_code_of(dt)) > 0
        y, ck, sa, sT = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], s0=s0d, want_ckpt=True,
                                  want_sa=True, want_state=True)
        torch.cuda.synchronize()
    finally:
        _segments(0)
    assert _native.lib().rwkv_device_error(1) == 0
    ye, sae, sTe, st = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], s0=s0, keep_states=True)
    tol = TOL[dt]
    assert rel_rms(y.double().cpu().numpy(), _bt(ye)) < tol
    assert rel_rms(sa.cpu().numpy(), sae) < tol
    assert rel_rms(sT.cpu().numpy(), sTe) < tol
    assert rel_rms(ck.cpu().numpy(), wo.checkpoints_from_states(st, 16).reshape(-1)) < tol


def test_automatic_segments_at_one_sequence_per_gpu():
    """B=1, T=4096, H=12 (BASELINE configs[1] split over 8 GPUs): the automatic choice
    segments the sequence; the result matches the oracle and the unsegmented kernel."""
    from rwkv_mlx_b200 import _native, wkv7

    B, T, H = 1, 4096, 12
    d, h = _inputs(B, T, H, seed=3, dt=torch.float16)
    assert _native.lib().rwkv_wkv7_forward_workspace_size(B, T, H, 64, 1) > 0
    y, _, _, sT = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], want_ckpt=False, want_state=True)
    _segments(1)
    try:
        y1, _, _, sT1 = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], want_ckpt=False, want_state=True)
    finally:
        _segments(0)
    torch.cuda.synchronize()
    assert _native.lib().rwkv_device_error(1) == 0
    ye, _, sTe, _ = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"])
    assert rel_rms(y.double().cpu().numpy(), _bt(ye)) < 2e-3
    assert rel_rms(sT.cpu().numpy(), sTe) < 2e-3
    assert rel_rms(y.double().cpu().numpy(), y1.double().cpu().numpy()) < 2e-3


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("B,T,H,nseg", [(1, 1024, 2, 3), (2, 777, 1, 5), (1, 256, 2, 16)])
def test_segmented_backward_matches_oracle(dt, B, T, H, nseg):
    """Forced segment counts for the backward's adjoint chain (a ragged top segment,
    three-chunk segments), with an initial state, a final-state gradient and ds0."""
    from rwkv_mlx_b200 import _native, wkv7

    inp = wkv_inputs(B, T, H, seed=T + 7 * nseg)
    d, h = {}, {}
    for n, x in inp.items():
        t = torch.tensor(_bt(x), dtype=torch.float32 if n == "w" else dt, device="cuda")
        d[n], h[n] = t, t.double().cpu().numpy().reshape(x.shape)
    rng = np.random.default_rng(nseg + 1)
    s0 = rng.standard_normal((B, H, 64, 64)) * 0.3
    dsT = rng.standard_normal((B, H, 64, 64)) * 0.1
    s0d = torch.tensor(s0, dtype=torch.float32, device="cuda")
    dsTd = torch.tensor(dsT, dtype=torch.float32, device="cuda")
    _, ck, _, _ = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], s0=s0d, want_ckpt=True)
    _segments(nseg)
    try:
        grads, ds0 = wkv7._bwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], d["dy"], ck, s0=s0d, dsT=dsTd,
                               want_ds0=True)
        torch.cuda.synchronize()
    finally:
        _segments(0)
    assert _native.lib().rwkv_device_error(1) == 0
    ge = wo.wkv7_backward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], h["dy"], s0=s0, dsT=dsT)
    tol = 6e-3 if dt == torch.bfloat16 else 2e-3
    for name, g, e in zip(["dr", "dw", "dk", "dv", "da", "db"], grads, ge[:6]):
        err = rel_rms(g.double().cpu().numpy(), _bt(e))
        assert err < tol, f"{name}: {err}"
    assert rel_rms(ds0.cpu().numpy(), ge[6]) < tol


def test_automatic_backward_segments_at_one_sequence_per_gpu():
    """B=1, T=4096, H=12: the automatic choice segments the adjoint chain; the gradients
    match the oracle and the unsegmented chain."""
    from rwkv_mlx_b200 import _native, wkv7

    B, T, H = 1, 4096, 12
    inp = wkv_inputs(B, T, H, seed=31)
    d, h = {}, {}
    for n, x in inp.items():
        t = torch.tensor(_bt(x), dtype=torch.float32 if n == "w" else torch.float16, device="cuda")
        d[n], h[n] = t, t.double().cpu().numpy().reshape(x.shape)
    _, ck, _, _ = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], want_ckpt=True)
    grads, _ = wkv7._bwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], d["dy"], ck)
    _segments(1)
    try:
        grads1, _ = wkv7._bwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], d["dy"], ck)
    finally:
        _segments(0)
    torch.cuda.synchronize()
    assert _native.lib().rwkv_device_error(1) == 0
    ge = wo.wkv7_backward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], h["dy"])
    for name, g, g1, e in zip(["dr", "dw", "dk", "dv", "da", "db"], grads, grads1, ge[:6]):
        assert rel_rms(g.double().cpu().numpy(), _bt(e)) < 2e-3, name
        assert rel_rms(g.double().cpu().numpy(), g1.double().cpu().numpy()) < 2e-3, name


def test_backward_launch_count_follows_the_plan():
    """The launch count the binding reports for the chunked backward: segmented chain at
    one sequence (transition, scan, final, per-chunk gradients), the chain in four parts
    at eight sequences (four launches of each pass), two launches for a short sequence."""
    from rwkv_mlx_b200 import _native

    L = _native.lib()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert L.rwkv_wkv7_backward_launch_count(1, 4096, 12, 64) == (4 if sms // 12 >= 4 else 2 + 6 * (sms - 12 >= 32))
    assert L.rwkv_wkv7_backward_launch_count(8, 4096, 12, 64) == (8 if sms - 96 >= 32 else 2)
    assert L.rwkv_wkv7_backward_launch_count(1, 96, 2, 64) == 2


def test_host_set_device_error_raises():
    """The Python check surfaces the device error word (set here from the host)."""
    import rwkv_mlx_b200 as rb
    from rwkv_mlx_b200 import _native

    rb.check_device_error()  # clean
    _native.check(_native.lib().rwkv_debug_set_device_error(8), "rwkv_debug_set_device_error")
    with pytest.raises(rb.RwkvDeviceError):
        rb.check_device_error()
    rb.check_device_error()  # the failed check cleared it


@pytest.mark.parametrize("nseg", [1, 3])
def test_forced_wait_timeout_fills_outputs_with_nan(nseg):
    """Every bounded wait of the tcgen05 forward gives up at once (a flag set from the
    host: no stall, no fault): the kernel exits, its outputs are NaN and the error is
    reported; the next call without the flag is correct again."""
    import rwkv_mlx_b200 as rb
    from rwkv_mlx_b200 import _native, wkv7

    B, T, H = 1, 768, 2
    d, h = _inputs(B, T, H, seed=9, dt=torch.float16)
    L = _native.lib()
    _segments(nseg)
    _native.check(L.rwkv_debug_force_wait_timeout(1), "rwkv_debug_force_wait_timeout")
    try:
        y, ck, sa, sT = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], want_ckpt=True, want_sa=True,
                                  want_state=True)
        torch.cuda.synchronize()
    finally:
        _native.check(L.rwkv_debug_force_wait_timeout(0), "rwkv_debug_force_wait_timeout")
    assert torch.isnan(y).all() and torch.isnan(sT).all() and torch.isnan(sa).all() and torch.isnan(ck).all()
    with pytest.raises(rb.RwkvDeviceError):
        rb.check_device_error()
    try:
        y2 = wkv7.wkv7(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"])
        torch.cuda.synchronize()
    finally:
        _segments(0)
    rb.check_device_error()
    ye = wo.wkv7_forward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"])[0]
    assert rel_rms(y2.double().cpu().numpy(), _bt(ye)) < 2e-3


def test_backward_after_an_abort_returns_nan_gradients():
    """A set backward error word (here set from the host, as a pass-1 abort would set it)
    makes the chunked backward write NaN gradients instead of values built on an
    invalid state-gradient chain; once the error is read and cleared it is exact again."""
    import rwkv_mlx_b200 as rb
    from rwkv_mlx_b200 import _native, wkv7

    B, T, H = 1, 96, 2
    d, h = _inputs(B, T, H, seed=12, dt=torch.float16)
    dy = torch.tensor(_bt(wkv_inputs(B, T, H, seed=12)["dy"]), dtype=torch.float16, device="cuda")
    _, ck, _, _ = wkv7._fwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], want_ckpt=True)
    torch.cuda.synchronize()
    rb.check_device_error()
    _native.check(_native.lib().rwkv_debug_set_device_error(1), "rwkv_debug_set_device_error")
    grads, _ = wkv7._bwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], dy, ck)
    torch.cuda.synchronize()
    assert all(torch.isnan(g).all() for g in grads)
    with pytest.raises(rb.RwkvDeviceError):
        rb.check_device_error()
    grads, _ = wkv7._bwd(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], dy, ck)
    torch.cuda.synchronize()
    rb.check_device_error()
    ge = wo.wkv7_backward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], dy.double().cpu().numpy().reshape(B, T, H, 64))
    for g, e in zip(grads, ge[:6]):
        assert rel_rms(g.double().cpu().numpy(), _bt(e)) < 2e-3
