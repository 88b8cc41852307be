"""Host-side model logic that needs no GPU: the stacked, zero-padded LoRA weights of the
fused TimeMix paths and the rebuild of their cache when a parameter changes."""
import torch

from rwkv_mlx_b200.model import RWKV_Tmix_x070, RWKVConfig


def _tmix():
    torch.manual_seed(0)
    cfg = RWKVConfig(n_layer=2, n_embd=128, d_decay_lora=32, d_aaa_lora=16, d_mv_lora=8, d_gate_lora=48)
    m = RWKV_Tmix_x070(cfg, 1)
    with torch.no_grad():
        for p in (m.v1, m.w1, m.a1, m.g1, m.v2, m.w2, m.a2, m.g2):
            p.normal_(0, 0.1)
    return m


def test_packed_lora_products_equal_the_four_pairs():
    """bmm over the padded stack, tanh on the decay slice and sigmoid on the gate slice,
    equals the four separate LoRA products (model.py:204-212 in the reference)."""
    m = _tmix()
    w1, w2 = m._packed_lora()
    D = max(m.v1.shape[1], m.w1.shape[1], m.a1.shape[1], m.g1.shape[1])
    assert w1.shape == (4, 128, D) and w2.shape == (4, D, 128)
    X = torch.randn(6, 37, 128, dtype=torch.float64)
    h = torch.bmm(X[2:6], w1.double())
    h[1] = torch.tanh(h[1])
    h[3] = torch.sigmoid(h[3])
    o = torch.bmm(h, w2.double())
    xv, xw, xa, xg = X[2], X[3], X[4], X[5]
    d = lambda p: p.detach().double()
    ref = [(xv @ d(m.v1)) @ d(m.v2), torch.tanh(xw @ d(m.w1)) @ d(m.w2), (xa @ d(m.a1)) @ d(m.a2),
           torch.sigmoid(xg @ d(m.g1)) @ d(m.g2)]
    for i in range(4):
        assert torch.allclose(o[i], ref[i], rtol=1e-12, atol=1e-12)


def test_packed_lora_cache_follows_parameter_updates():
    m = _tmix()
    a = m._packed_lora()
    assert m._packed_lora() is a  # unchanged parameters: the cached stack
    with torch.no_grad():
        m.g2.add_(1.0)  # an in-place update (an optimiser step) bumps the version
    b = m._packed_lora()
    assert b is not a
    assert torch.equal(b[1][3, : m.g2.shape[0]], m.g2.detach())
