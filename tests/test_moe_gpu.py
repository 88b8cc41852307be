"""LoRA-MoE CUDA kernels vs the numpy oracle of rwkv_mlx/moe.py (need a B200).

Routing indices and the permutation are compared bit-exactly; the router is fed
identical fp32 logits on both sides (the GPU's own logits) so that GEMM rounding
cannot flip a near-tie.  Float outputs: relative-to-RMS 2e-3 for fp16.
"""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tests.inputs import rel_rms

pytestmark = pytest.mark.gpu


def _x(ntok, C, seed, dt=torch.float16):
    rng = np.random.default_rng(seed)
    return torch.tensor(rng.standard_normal((ntok, C)), dtype=torch.float32, device="cuda").to(dt)


@pytest.mark.parametrize("dt,C", [(torch.float16, 768), (torch.bfloat16, 768), (torch.float32, 768),
                                  (torch.float16, 72), (torch.bfloat16, 264)])
@pytest.mark.parametrize("E,k,with_bias", [(8, 2, False), (8, 2, True), (4, 1, False), (16, 3, False), (32, 4, True)])
def test_router_bit_exact_indices(dt, C, E, k, with_bias):
    """16-bit x: tensor-core kernel with split gate weights (C = 72, 264: partial
    32-column blocks and load batches); fp32 x: the FMA kernel."""
    from rwkv_mlx_b200.moe import router_forward

    ntok = 3000
    x = _x(ntok, C, E * 10 + k, dt)
    rng = np.random.default_rng(E)
    gw = torch.tensor(rng.standard_normal((E, C)) * 0.02, dtype=torch.float32, device="cuda")
    bias = torch.tensor(rng.normal(0, 1.5, E), dtype=torch.float32, device="cuda") if with_bias else None
    r = router_forward(x, gw, k, bias, want_logits=True)
    torch.cuda.synchronize()
    lg = r["logits"].cpu().numpy()
    # logits themselves: fp32 GEMM, different summation order
    ref_lg = mo.gate_logits(x.float().cpu().numpy(), gw.cpu().numpy(), None if bias is None else bias.cpu().numpy())
    assert np.max(np.abs(lg - ref_lg)) < 1e-4 * max(1.0, np.abs(ref_lg).max())
    inds, scores, aux, z, f = mo.router(None, None, k, logits=lg)
    np.testing.assert_array_equal(r["inds"].cpu().numpy(), inds)
    assert rel_rms(r["scores"].double().cpu().numpy(), scores) < 2e-3
    assert abs(float(r["aux"]) - aux) < 1e-4 * max(1, abs(aux))
    assert abs(float(r["z"]) - z) < 1e-4 * max(1, abs(z))
    np.testing.assert_allclose(r["f"].cpu().numpy(), f, rtol=1e-6)
    np.testing.assert_array_equal(r["counts"].cpu().numpy(), np.bincount(inds.reshape(-1), minlength=E))


def test_router_config4_routing_vs_oracle_own_logits():
    """BASELINE configs[3]'s router: 65,536 fp16 tokens, C=768, E=8, top-2, per-expert
    logit bias N(0, 1.5).  The GPU's indices are compared with the oracle routing on its
    OWN logits (x.astype(f32) @ W^T + bias, moe.py:56, evaluated in float64), not the
    GPU's.  Any token that differs must be a provable near-tie: the two competing
    logits differ by less than the worst-case fp32 summation error of a 768-term dot
    product (768 * 2^-24 * sum |x_i w_i|, plus the bias rounding)."""
    from rwkv_mlx_b200.moe import router_forward

    ntok, C, E, k = 65536, 768, 8, 2
    x = _x(ntok, C, 4, torch.float16)
    rng = np.random.default_rng(5)
    gw = torch.tensor(rng.standard_normal((E, C)) / np.sqrt(C), dtype=torch.float32, device="cuda")
    bias = torch.tensor(rng.normal(0, 1.5, E), dtype=torch.float32, device="cuda")
    r = router_forward(x, gw, k, bias)
    torch.cuda.synchronize()
    xn, wn, bn = x.float().cpu().numpy(), gw.cpu().numpy(), bias.cpu().numpy()
    lg = mo.gate_logits(xn, wn, bn)
    ref = mo.topk_from_logits(lg, k)
    got = r["inds"].cpu().numpy().astype(np.int64)
    bad = np.nonzero((got != ref).any(-1))[0]
    mag = np.abs(xn.astype(np.float64)) @ np.abs(wn.astype(np.float64)).T  # sum_i |x_i w_ie|
    bound = C * 2.0 ** -24 * mag + 2.0 ** -24 * np.abs(bn)
    for t in bad:
        # the sets differ only where the boundary logits are within the error bound
        for e_g, e_r in zip(got[t], ref[t]):
            if e_g != e_r:
                assert abs(lg[t, e_g] - lg[t, e_r]) <= bound[t, e_g] + bound[t, e_r], (t, e_g, e_r)
    print(f"config-4 routing: {len(bad)} of {ntok} tokens differ from the oracle (near-ties)")
    assert len(bad) <= 8


def test_router_ties_go_to_lower_id():
    from rwkv_mlx_b200.moe import router_forward

    C, E = 64, 8
    x = torch.zeros(40, C, dtype=torch.float16, device="cuda")
    x[20:] = 1.0
    gw = torch.zeros(E, C, device="cuda")
    gw[5] = 1.0 / C
    gw[6] = 1.0 / C  # experts 5 and 6 tie for tokens 20..39
    r = router_forward(x, gw, 2)
    inds = r["inds"].cpu().numpy()
    assert (inds[:20] == [0, 1]).all()  # all logits 0: lowest ids
    assert (inds[20:] == [5, 6]).all()


@pytest.mark.parametrize("ntok,k,E", [(1, 1, 8), (5000, 2, 8), (4097, 3, 5), (70000, 2, 64)])
def test_permute_bit_exact(ntok, k, E):
    from rwkv_mlx_b200.moe import permute

    rng = np.random.default_rng(ntok)
    # skewed load, empty experts included
    p = rng.dirichlet(np.ones(E) * 0.3)
    inds = rng.choice(E, size=(ntok, k), p=p).astype(np.int32)
    perm, inv, off = permute(torch.tensor(inds, device="cuda"), E)
    flat = inds.reshape(-1)
    ref_perm = np.argsort(flat, kind="stable")
    np.testing.assert_array_equal(perm.cpu().numpy(), ref_perm)
    ref_inv = np.empty_like(ref_perm)
    ref_inv[ref_perm] = np.arange(len(ref_perm))
    np.testing.assert_array_equal(inv.cpu().numpy(), ref_inv)
    np.testing.assert_array_equal(off.cpu().numpy(), np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=E))]))


@pytest.mark.parametrize("R", [8, 16, 32])
def test_lora_down_and_combine(R):
    from rwkv_mlx_b200.moe import lora_combine, lora_down, permute, router_forward

    ntok, C, E, k = 2000, 768, 8, 2
    x = _x(ntok, C, 3)
    rng = np.random.default_rng(R)
    A = torch.tensor(rng.normal(0, 0.02, (E, C, R)), dtype=torch.float16, device="cuda")
    Bw = torch.tensor(rng.normal(0, 0.02, (E, R, C)), dtype=torch.float16, device="cuda")
    gw = torch.tensor(rng.standard_normal((E, C)) * 0.02, dtype=torch.float32, device="cuda")
    base = _x(ntok, C, 4)
    r = router_forward(x, gw, k)
    perm, inv, off = permute(r["inds"], E)
    h = lora_down(x, A, perm, off, k)
    out = lora_combine(base, h, Bw, r["inds"], r["scores"], inv)
    torch.cuda.synchronize()
    xn, An, Bn = x.double().cpu().numpy(), A.double().cpu().numpy(), Bw.double().cpu().numpy()
    inds, sc = r["inds"].cpu().numpy(), r["scores"].double().cpu().numpy()
    # h in sorted order
    ent = perm.cpu().numpy()
    tok = ent // k
    e_of = inds.reshape(-1)[ent]
    h_ref = np.einsum("pc,pcr->pr", xn[tok], An[e_of])
    assert rel_rms(h.cpu().numpy(), h_ref) < 1e-5
    ref = base.double().cpu().numpy() + mo.lora_moe_delta(xn, An, Bn, inds, sc)
    assert rel_rms(out.double().cpu().numpy(), ref) < 2e-3


def test_lora_moe_cmix_module_matches_oracle():
    from rwkv_mlx_b200.model import RWKV_CMix_x070, RWKVConfig
    from rwkv_mlx_b200.moe import LoRAMoE_CMix

    torch.manual_seed(0)
    cfg = RWKVConfig(n_layer=2, n_embd=256, dim_ffn=512)
    base = RWKV_CMix_x070(cfg, 1).cuda()
    with torch.no_grad():
        base.x_k.uniform_(0, 1)
        base.key.weight.normal_(0, 0.05)
        base.value.weight.normal_(0, 0.05)
    m = LoRAMoE_CMix(base, n_experts=8, lora_rank=16, top_k=2).cuda()
    with torch.no_grad():
        m.lora_A.normal_(0, 0.02)
        m.lora_B.normal_(0, 0.02)
        m.router.gate.weight.normal_(0, 0.05)
    m = m.half()
    x = torch.randn(2, 64, 256, device="cuda").half()
    with torch.no_grad():
        out, aux, z = m(x)
        lg = (x.float().reshape(-1, 256) @ m.router.gate.weight.float().T).cpu().numpy()
    xn = x.double().cpu().numpy()
    npy = lambda t: t.detach().double().cpu().numpy()
    base_ref = mo.cmix(xn, npy(base.x_k), npy(base.key.weight), npy(base.value.weight))
    inds, sc, aux_r, z_r, _ = mo.router(None, None, 2, logits=lg)
    ref = base_ref + mo.lora_moe_delta(xn, npy(m.lora_A), npy(m.lora_B), inds.reshape(2, 64, 2),
                                       sc.reshape(2, 64, 2))
    assert rel_rms(out.double().cpu().numpy(), ref) < 3e-3
    assert abs(float(aux) - aux_r) < 1e-3
    assert abs(float(z) - z_r) < 1e-3 * max(1, z_r)
    ol = m.orthogonal_loss()
    ol_ref = mo.orthogonal_loss(npy(m.lora_A))
    assert abs(float(ol) - ol_ref) < 1e-3 * max(1e-6, ol_ref)


@pytest.fixture(params=[2, 1], ids=["tcgen05", "mma_sync"])
def apply_impl(request):
    """Run a test on each kernel of rwkv_moe_lora_apply (process-wide switch, reset after)."""
    from rwkv_mlx_b200 import _native

    assert _native.lib().rwkv_moe_set_apply_impl(request.param) == 0
    yield request.param
    assert _native.lib().rwkv_moe_set_apply_impl(0) == 0


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ntok,C,E,R,k,with_base", [(2000, 768, 8, 16, 2, True), (4097, 1024, 4, 8, 1, False),
                                                    (77, 64, 8, 8, 3, True), (130, 128, 16, 8, 4, True),
                                                    (65, 768, 2, 16, 2, True), (40000, 768, 8, 16, 2, True)])
def test_lora_apply_matches_oracle(apply_impl, dt, ntok, C, E, R, k, with_base):
    """Fused adapter apply (dense over E*R columns, routing mask) vs the float64 sum;
    40000 tokens = 313 tiles of 128, more than one per SM for the persistent kernel."""
    from rwkv_mlx_b200.moe import lora_apply, lora_apply_supported, router_forward

    assert lora_apply_supported(C, R, E, k, dt)
    x = _x(ntok, C, 5, dt)
    rng = np.random.default_rng(ntok + C)
    A = torch.tensor(rng.normal(0, 0.05, (E, C, R)), dtype=dt, device="cuda")
    Bw = torch.tensor(rng.normal(0, 0.05, (E, R, C)), dtype=dt, device="cuda")
    gw = torch.tensor(rng.standard_normal((E, C)) * 0.05, dtype=torch.float32, device="cuda")
    base = _x(ntok, C, 6, dt) if with_base else None
    r = router_forward(x, gw, k)
    out = lora_apply(x, base, A, Bw, r["inds"], r["scores"])
    torch.cuda.synchronize()
    npy = lambda t: t.double().cpu().numpy()
    delta = mo.lora_moe_delta(npy(x), npy(A), npy(Bw), r["inds"].cpu().numpy(), npy(r["scores"]))
    # without a base the delta is checked on its own; with one, the output (which is
    # rounded to the activation dtype at the magnitude of base + delta)
    ref = delta + (npy(base) if with_base else 0.0)
    tol = {torch.float16: 2e-3, torch.bfloat16: 8e-3}[dt] if with_base else {torch.float16: 4e-3, torch.bfloat16: 2e-2}[dt]
    assert rel_rms(npy(out), ref) < tol
    from rwkv_mlx_b200 import _native

    assert _native.lib().rwkv_device_error(1) == 0


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ntok,C,E,R,k,with_scores", [(300, 256, 8, 16, 1, False), (5000, 768, 8, 16, 2, True),
                                                      (333, 64, 4, 8, 2, True)])
def test_lora_apply_in_place(apply_impl, dt, ntok, C, E, R, k, with_scores):
    """out aliasing base (the tcgen05 kernel then adds into out in L2 with TMA
    reduce-add stores); scores NULL (all 1) is the EP local step's form."""
    from rwkv_mlx_b200 import _native
    from rwkv_mlx_b200.moe import lora_apply

    x = _x(ntok, C, 8, dt)
    rng = np.random.default_rng(9 + ntok)
    A = torch.tensor(rng.normal(0, 0.05, (E, C, R)), dtype=dt, device="cuda")
    Bw = torch.tensor(rng.normal(0, 0.05, (E, R, C)), dtype=dt, device="cuda")
    inds = torch.tensor(np.argsort(rng.random((ntok, E)), axis=1)[:, :k], dtype=torch.int32, device="cuda")
    sc = torch.tensor(rng.random((ntok, k)), dtype=dt, device="cuda") if with_scores else None
    base = _x(ntok, C, 10, dt)
    base_np = base.double().cpu().numpy()
    out = lora_apply(x, base, A, Bw, inds, sc, out=base)
    torch.cuda.synchronize()
    assert out.data_ptr() == base.data_ptr()
    npy = lambda t: t.double().cpu().numpy()
    delta = mo.lora_moe_delta(npy(x), npy(A), npy(Bw), inds.cpu().numpy(),
                              npy(sc) if with_scores else np.ones((ntok, k)))
    assert rel_rms(npy(out), base_np + delta) < {torch.float16: 2e-3, torch.bfloat16: 8e-3}[dt]
    assert _native.lib().rwkv_device_error(1) == 0


def test_lora_moe_cmix_unsupported_shape_uses_sorted_dispatch():
    """E*R = 256 is outside the fused kernel: the module takes the permutation path."""
    from rwkv_mlx_b200.model import RWKV_CMix_x070, RWKVConfig
    from rwkv_mlx_b200.moe import LoRAMoE_CMix, lora_apply_supported

    assert not lora_apply_supported(256, 32, 8, 2, torch.float16)
    torch.manual_seed(1)
    cfg = RWKVConfig(n_layer=2, n_embd=256, dim_ffn=512)
    base = RWKV_CMix_x070(cfg, 1).cuda()
    m = LoRAMoE_CMix(base, n_experts=8, lora_rank=32, top_k=2).cuda()
    with torch.no_grad():
        m.lora_B.normal_(0, 0.02)
        m.router.gate.weight.normal_(0, 0.05)
    m = m.half()
    x = torch.randn(2, 40, 256, device="cuda").half()
    with torch.no_grad():
        out, _, _ = m(x)
        lg = (x.float().reshape(-1, 256) @ m.router.gate.weight.float().T).cpu().numpy()
    npy = lambda t: t.detach().double().cpu().numpy()
    xn = x.double().cpu().numpy()
    inds, sc, _, _, _ = mo.router(None, None, 2, logits=lg)
    ref = mo.cmix(xn, npy(base.x_k), npy(base.key.weight), npy(base.value.weight)) + mo.lora_moe_delta(
        xn, npy(m.lora_A), npy(m.lora_B), inds.reshape(2, 40, 2), sc.reshape(2, 40, 2))
    assert rel_rms(out.double().cpu().numpy(), ref) < 3e-3


def _full_moe(C, D, E, k, dt, seed):
    from rwkv_mlx_b200.model import RWKVConfig
    from rwkv_mlx_b200.moe import MoE_CMix

    torch.manual_seed(seed)
    fm = MoE_CMix(RWKVConfig(n_layer=2, n_embd=C, dim_ffn=D), 1, E, k).cuda()
    rng = np.random.default_rng(seed)
    with torch.no_grad():
        fm.x_k.copy_(torch.tensor(rng.uniform(0, 1, (E, 1, 1, C))))
        fm.expert_key.copy_(torch.tensor(rng.standard_normal((E, D, C)) / np.sqrt(C)))
        fm.expert_val.copy_(torch.tensor(rng.standard_normal((E, C, D)) / np.sqrt(D)))
        fm.router.gate.weight.copy_(torch.tensor(rng.standard_normal((E, C)) * 0.05))
    return fm.to(dt)


def _full_moe_oracle(fm, x, inds, scores):
    g = lambda t: t.detach().double().cpu().numpy()
    return mo.full_moe(g(x), g(fm.x_k), g(fm.expert_key), g(fm.expert_val), inds, scores)


# float tolerance, relative to RMS: every intermediate (mixed rows, key activations,
# their squares, expert outputs) is rounded to the activation dtype once
_TOL = {torch.float16: 4e-3, torch.bfloat16: 3e-2, torch.float32: 1e-4}


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("B,T,C,D,E,k", [(2, 300, 256, 512, 4, 2), (3, 77, 128, 384, 8, 1), (1, 1, 64, 128, 5, 3),
                                         (4, 129, 768, 3072, 8, 2)])
def test_full_moe_cmix_matches_oracle(dt, B, T, C, D, E, k):
    """MoE_CMix on the sorted dispatch vs the reference's dense expert loop (moe.py:226-239),
    the oracle routed with the GPU's own fp32 logits (identical inputs on both sides)."""
    from rwkv_mlx_b200.moe import router_forward

    fm = _full_moe(C, D, E, k, dt, seed=B * 1000 + T)
    x = _x(B * T, C, seed=T, dt=dt).view(B, T, C)
    with torch.no_grad():
        out, aux, z = fm(x)
        r = router_forward(x.view(B * T, C), fm.router.gate.weight, k, want_logits=True)
    torch.cuda.synchronize()
    inds, scores, aux_o, z_o, _ = mo.router(None, None, k, logits=r["logits"].cpu().numpy())
    np.testing.assert_array_equal(r["inds"].cpu().numpy(), inds)
    ref = _full_moe_oracle(fm, x, inds.reshape(B, T, k), r["scores"].double().cpu().numpy().reshape(B, T, k))
    assert rel_rms(out.double().cpu().numpy(), ref) < _TOL[dt]
    assert abs(float(aux) - aux_o) < 1e-4 and abs(float(z) - z_o) < 1e-3 * max(1.0, z_o)


def test_full_moe_cmix_rnn_step_matches_oracle():
    """One token per sequence with the stored previous token (RNN mode)."""
    from rwkv_mlx_b200.moe import router_forward

    Bs, C, D, E, k = 37, 256, 512, 8, 2
    fm = _full_moe(C, D, E, k, torch.float16, seed=11)
    x, xp = _x(Bs, C, seed=1), _x(Bs, C, seed=2)
    with torch.no_grad():
        out = fm.forward_rnn(x, xp)
        r = router_forward(x, fm.router.gate.weight, k, want_logits=True)
    torch.cuda.synchronize()
    inds, _, _, _, _ = mo.router(None, None, k, logits=r["logits"].cpu().numpy())
    g = lambda t: t.detach().double().cpu().numpy()
    ref = mo.full_moe_step(g(x), g(xp), g(fm.x_k), g(fm.expert_key), g(fm.expert_val), inds,
                           r["scores"].double().cpu().numpy())
    assert rel_rms(out.double().cpu().numpy(), ref) < _TOL[torch.float16]


@pytest.mark.parametrize("ntok,C,E,R,k,with_bias", [(3000, 768, 8, 16, 2, True), (65536, 768, 8, 16, 2, True),
                                                     (1000, 256, 4, 8, 1, False), (777, 512, 16, 8, 3, True)])
def test_routed_apply_matches_oracle(ntok, C, E, R, k, with_bias):
    """The router folded into the tcgen05 apply kernel (one pass over x): expert sets equal
    the oracle's routing on its own float64 logits except provable near-ties (fp32
    summation-order bound, as in the config-4 router test); scores, aux, z, counts and the
    output (out = base in place) against the oracle and the unfused router + apply."""
    from rwkv_mlx_b200.moe import lora_apply, lora_apply_routed, lora_apply_routed_supported, router_forward

    assert lora_apply_routed_supported(C, R, E, k, torch.float16)
    x = _x(ntok, C, 3 + E, torch.float16)
    rng = np.random.default_rng(E + k)
    gw = torch.tensor(rng.standard_normal((E, C)) / np.sqrt(C), dtype=torch.float32, device="cuda")
    bias = torch.tensor(rng.normal(0, 1.5, E), dtype=torch.float32, device="cuda") if with_bias else None
    A = torch.tensor(rng.normal(0, 0.02, (E, C, R)), dtype=torch.float16, device="cuda")
    Bw = torch.tensor(rng.normal(0, 0.02, (E, R, C)), dtype=torch.float16, device="cuda")
    base = _x(ntok, C, 99, torch.float16)
    out = base.clone()
    out, rf = lora_apply_routed(x, out, A, Bw, gw, k, bias, out=out)  # in place, as the module calls it
    ru = router_forward(x, gw, k, bias)
    out_u = lora_apply(x, base, A, Bw, ru["inds"], ru["scores"])
    torch.cuda.synchronize()
    xn, wn = x.float().cpu().numpy(), gw.cpu().numpy()
    bn = None if bias is None else bias.cpu().numpy()
    lg = mo.gate_logits(xn, wn, bn)
    ref = mo.topk_from_logits(lg, k)
    got = rf["inds"].cpu().numpy().astype(np.int64)
    bad = np.nonzero((got != ref).any(-1))[0]
    mag = np.abs(xn.astype(np.float64)) @ np.abs(wn.astype(np.float64)).T
    bound = C * 2.0 ** -24 * mag + (0 if bn is None else 2.0 ** -24 * np.abs(bn))
    for t in bad:
        for e_g, e_r in zip(got[t], ref[t]):
            if e_g != e_r:
                assert abs(lg[t, e_g] - lg[t, e_r]) <= bound[t, e_g] + bound[t, e_r], (t, e_g, e_r)
    assert len(bad) <= max(2, ntok // 20000)
    # everything else against the oracle on the fused routing
    inds_r, sc_r, aux_r, z_r, f_r = mo.router(None, None, k, logits=lg)
    sel = np.take_along_axis(lg, got, -1)
    sc = np.exp(sel - sel.max(-1, keepdims=True))
    sc = sc / sc.sum(-1, keepdims=True)
    assert np.abs(rf["scores"].double().cpu().numpy() - sc).max() < 1e-3  # fp16 scores
    assert abs(float(rf["aux"]) - aux_r) < 1e-4 * max(1.0, abs(aux_r))
    assert abs(float(rf["z"]) - z_r) < 1e-4 * max(1.0, abs(z_r))
    np.testing.assert_array_equal(rf["counts"].cpu().numpy(), np.bincount(got.reshape(-1), minlength=E))
    xd = x.double().cpu().numpy()
    ref_out = base.double().cpu().numpy() + mo.lora_moe_delta(xd, A.double().cpu().numpy(), Bw.double().cpu().numpy(),
                                                               got, rf["scores"].double().cpu().numpy())
    assert rel_rms(out.double().cpu().numpy(), ref_out) < 2e-3
    same = np.nonzero((got == ru["inds"].cpu().numpy()).all(-1))[0]
    assert rel_rms(out.double().cpu().numpy()[same], out_u.double().cpu().numpy()[same]) < 1e-3
