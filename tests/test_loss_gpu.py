"""Chunked cross-entropy kernels (csrc/loss.cu) vs the float64 restatement of
rwkv_mlx/train.py:317-362 (oracle/loss_oracle.py, pinned to the reference's own
functions).  Needs a GPU.  Loss: 1e-5 relative in fp32, 1e-3 for 16-bit logits (the
oracle then reads the same rounded logits); gradients relative to RMS."""

import numpy as np
import pytest
import torch

from oracle import loss_oracle as lo
from tests.golden.golden import golden
from tests.inputs import rel_rms

pytestmark = pytest.mark.gpu


def test_losses_match_reference_golden():
    from rwkv_mlx_b200.loss import l2_wrap_loss, l2_wrap_loss_masked

    G = golden()
    lg = torch.tensor(G["loss_logits"], device="cuda")
    tg = torch.tensor(G["loss_targets"], device="cuda")
    mk = torch.tensor(G["loss_mask"], device="cuda")
    assert abs(float(l2_wrap_loss(lg, tg)) - float(G["loss_l2wrap"])) < 1e-5
    assert abs(float(l2_wrap_loss_masked(lg, tg, mk)) - float(G["loss_l2wrap_masked"])) < 1e-5


def _case(B, T, V, C, dt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(B, T, C, device="cuda", generator=g)).to(dt)
    w = (torch.randn(V, C, device="cuda", generator=g) * (2.0 / C ** 0.5)).to(dt)
    tg = torch.randint(0, V, (B, T), device="cuda", generator=g)
    mk = (torch.rand(B, T, device="cuda", generator=g) < 0.7).float()
    return x, w, tg, mk


@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("masked", [False, True])
@pytest.mark.parametrize("B,T,V,C,chunk", [(2, 37, 1000, 64, 256), (1, 5, 65568, 128, 8192), (3, 64, 777, 96, 776)])
def test_head_loss_and_gradients_match_oracle(dt, masked, B, T, V, C, chunk):
    from rwkv_mlx_b200.loss import head_l2_wrap_loss

    x, w, tg, mk = _case(B, T, V, C, dt, seed=V + T)
    xg, wg = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    loss = head_l2_wrap_loss(xg, wg, tg, mk if masked else None, chunk=chunk)
    loss.backward()
    # oracle on the logits the GPU GEMM produces (rounded to dt), float64
    xd = x.double().cpu().requires_grad_(True)
    wd = w.double().cpu().requires_grad_(True)
    lg = xd @ wd.T
    ref = lo.l2_wrap_loss_masked(lg, tg.cpu(), mk.cpu().double()) if masked else lo.l2_wrap_loss(lg, tg.cpu())
    ref.backward()
    tol = 1e-5 if dt == torch.float32 else 2e-2
    assert abs(float(loss.detach()) - float(ref.detach())) < tol * max(1.0, abs(float(ref.detach())))
    gtol = 1e-4 if dt == torch.float32 else 3e-2
    assert rel_rms(xg.grad.double().cpu().numpy(), xd.grad.numpy()) < gtol
    assert rel_rms(wg.grad.double().cpu().numpy(), wd.grad.numpy()) < gtol


@pytest.mark.parametrize("dt", [torch.float32, torch.float16])
def test_loss_on_logits_and_its_gradient(dt):
    from rwkv_mlx_b200.loss import l2_wrap_loss

    g = torch.Generator(device="cuda").manual_seed(3)
    lg = (torch.randn(2, 50, 3001, device="cuda", generator=g) * 4).to(dt).requires_grad_(True)
    tg = torch.randint(0, 3001, (2, 50), device="cuda", generator=g)
    loss = l2_wrap_loss(lg, tg)
    loss.backward()
    ld = lg.detach().double().cpu().requires_grad_(True)
    ref = lo.l2_wrap_loss(ld, tg.cpu())
    ref.backward()
    assert abs(float(loss.detach()) - float(ref.detach())) < 1e-5 * abs(float(ref.detach()))
    assert rel_rms(lg.grad.double().cpu().numpy(), ld.grad.numpy()) < (1e-5 if dt == torch.float32 else 5e-3)


def test_model_forward_loss_equals_loss_on_full_logits():
    """RWKV.forward_loss (fused head + loss) = l2_wrap_loss on the model's logits + aux."""
    from rwkv_mlx_b200.loss import l2_wrap_loss
    from rwkv_mlx_b200.model import RWKV, RWKVConfig, init_weights

    torch.manual_seed(0)
    cfg = RWKVConfig(n_layer=2, n_embd=128, vocab_size=1000, dim_ffn=256, moe_num_experts=4, moe_top_k=2,
                     moe_mode="full")
    m = RWKV(cfg).cuda()
    init_weights(m, seed=1)
    with torch.no_grad():
        for p in m.parameters():
            p.add_(torch.randn_like(p) * 0.02)
    idx = torch.randint(0, 1000, (2, 40), device="cuda")
    tg = torch.randint(0, 1000, (2, 40), device="cuda")
    with torch.no_grad():
        fused = m.forward_loss(idx, tg, chunk=256)
        logits, aux = m(idx)
        full = l2_wrap_loss(logits, tg) + aux
    assert abs(float(fused) - float(full)) < 1e-5 * abs(float(full))


def test_masked_loss_with_an_empty_mask_is_the_l2_term():
    """mask all zero: the cross-entropy term is 0 / (0 + 1e-9) = 0 (train.py:355-356) and
    the loss is the L2 max-logit term alone; its gradient flows only through the maxima."""
    from rwkv_mlx_b200.loss import head_l2_wrap_loss

    x, w, tg, _ = _case(2, 20, 500, 64, torch.float32, seed=9)
    mk = torch.zeros(2, 20, device="cuda")
    xg, wg = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    loss = head_l2_wrap_loss(xg, wg, tg, mk, chunk=128)
    loss.backward()
    xd = x.double().cpu().requires_grad_(True)
    wd = w.double().cpu().requires_grad_(True)
    ref = lo.l2_wrap_loss_masked(xd @ wd.T, tg.cpu(), mk.cpu().double())
    ref.backward()
    assert abs(float(loss.detach()) - float(ref.detach())) < 1e-6 * max(1.0, abs(float(ref.detach())))
    assert rel_rms(xg.grad.double().cpu().numpy(), xd.grad.numpy()) < 1e-4
    assert rel_rms(wg.grad.double().cpu().numpy(), wd.grad.numpy()) < 1e-4
