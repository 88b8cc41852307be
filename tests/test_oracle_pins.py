"""Pin the CPU oracles to the reference's own code (CPU-only).

* ``oracle/_ref``: the reference's Metal kernel bodies (wkv7_metal.py:20-215)
  compiled as C++ by ``oracle/build_ref.py``.  Our C restatement
  (``oracle/wkv7_metal_port.c``) must agree with it bit for bit, and the float64
  exact oracle must agree with its forward to fp32 rounding.
* ``tests/golden/*.npz``: outputs of the reference's own Python (model.py, moe.py,
  wkv7_metal.py) run by ``tests/golden/make_golden.py``; the oracles must
  reproduce them.
"""

import numpy as np
import pytest

from oracle import cpu_wkv7 as cw
from oracle import wkv7_oracle as wo
from tests.inputs import rel_rms, wkv_inputs

needs_ref = pytest.mark.skipif(not cw.ref_available(), reason="oracle/_ref not built (needs the reference sources)")


def _in(B, T, H, seed, dt=np.float32):
    d = wkv_inputs(B, T, H, seed=seed)
    return {k: v.astype(dt) for k, v in d.items()}


@needs_ref
@pytest.mark.parametrize("B,T,H", [(1, 64, 2), (2, 48, 1)])
def test_port_is_bit_exact_with_reference_build(B, T, H):
    d = _in(B, T, H, seed=T)
    args = [d[n] for n in "rwkvab"]
    yr, sr, sar = cw.ref_forward(*args)
    yp, sp, sap = cw.port_forward(*args)
    np.testing.assert_array_equal(yr, yp)
    np.testing.assert_array_equal(sr, sp)
    np.testing.assert_array_equal(sar, sap)
    gr = cw.ref_backward(*args, d["dy"], sr, sar)
    gp = cw.port_backward(*args, d["dy"], sp, sap)
    for a, b in zip(gr, gp):
        np.testing.assert_array_equal(a, b)


@needs_ref
def test_exact_oracle_matches_reference_forward():
    d = _in(1, 64, 2, seed=1)
    yr, sr, sar = cw.ref_forward(*[d[n] for n in "rwkvab"])
    ye, sae, _, st = wo.wkv7_forward_exact(*[d[n] for n in "rwkvab"], keep_states=True)
    assert rel_rms(yr, ye) < 1e-6
    assert rel_rms(sar, sae) < 1e-6
    assert rel_rms(sr, wo.checkpoints_from_states(st, 16).reshape(-1)) < 1e-6


@needs_ref
def test_reference_fp16_kernel_matches_oracle_on_rounded_inputs():
    d = _in(1, 32, 2, seed=2, dt=np.float16)
    yr, _, _ = cw.ref_forward(*[d[n] for n in "rwkvab"])
    ye = wo.wkv7_forward_exact(*[d[n].astype(np.float64) for n in "rwkvab"])[0]
    assert rel_rms(yr.astype(np.float64), ye) < 1e-3


@needs_ref
def test_reference_backward_is_close_to_exact_in_the_model_decay_range():
    """The reference's reverse reconstruction divides by the decay; with decays in
    [0.545, 1) (the range the model produces) its error stays small."""
    d = _in(1, 64, 2, seed=3)
    args = [d[n] for n in "rwkvab"]
    yr, sr, sar = cw.ref_forward(*args)
    gr = cw.ref_backward(*args, d["dy"], sr, sar)
    ge = wo.wkv7_backward_exact(*args, d["dy"])
    for a, e in zip(gr, ge[:6]):
        assert rel_rms(a, e) < 1e-4


def test_port_forward_matches_exact_oracle():
    d = _in(2, 40, 2, seed=4)
    yp, _, sap = cw.port_forward(*[d[n] for n in "rwkvab"])
    ye, sae, _, _ = wo.wkv7_forward_exact(*[d[n] for n in "rwkvab"])
    assert rel_rms(yp, ye) < 1e-6
    assert rel_rms(sap, sae) < 1e-6


def test_exact_backward_matches_finite_differences():
    """The float64 reverse mode is the true derivative (central differences)."""
    d = wkv_inputs(1, 6, 1, seed=5)
    args = [d[n] for n in "rwkvab"]
    g = wo.wkv7_backward_exact(*args, d["dy"])
    rng = np.random.default_rng(0)
    for which, grad in zip(range(6), g[:6]):
        idx = tuple(rng.integers(0, s) for s in d["r"].shape)
        eps = 1e-6
        plus = [a.copy() for a in args]
        minus = [a.copy() for a in args]
        plus[which][idx] += eps
        minus[which][idx] -= eps
        fp = (wo.wkv7_forward_exact(*plus)[0] * d["dy"]).sum()
        fm = (wo.wkv7_forward_exact(*minus)[0] * d["dy"]).sum()
        assert abs((fp - fm) / (2 * eps) - grad[idx]) < 1e-6 * max(1.0, abs(grad[idx]))


def test_step_oracle_is_one_sequence_step():
    d = wkv_inputs(2, 5, 3, seed=6)
    y, _, sT, st = wo.wkv7_forward_exact(*[d[n] for n in "rwkvab"], keep_states=True)
    S = st[:, :, 3]
    ys, Sn = wo.wkv7_step_exact(S, *[d[n][:, 3] for n in "rwkvab"], w_is_decay=False)
    np.testing.assert_allclose(ys, y[:, 3], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(Sn, st[:, :, 4], rtol=1e-12, atol=1e-12)
