"""BASELINE configs[4] shapes as parity cases (need a B200): the L24 D1024 model with
LoRA-MoE (E=8, top-2, rank 16) in every ChannelMix against the CPU restatement of
rwkv_mlx/model.py + moe.py, and the WKV-7 backward micro-batch (B=4, T=1024, H=16,
fp16) against the float64 oracle.  Tolerances relative to RMS as in the other tests
(2e-3: TF32 chunked kernels with fp32 state)."""

import numpy as np
import pytest
import torch

from oracle import model_oracle as mo
from oracle import wkv7_oracle as wo
from tests.inputs import rel_rms, wkv_inputs

pytestmark = pytest.mark.gpu


def test_config5_model_with_lora_moe_in_every_layer():
    from rwkv_mlx_b200.model import RWKV, RWKVConfig, init_weights

    cfg = RWKVConfig(n_layer=24, n_embd=1024, vocab_size=65568, moe_num_experts=8, moe_top_k=2, moe_lora_rank=16)
    torch.manual_seed(0)
    m = RWKV(cfg).cuda()
    init_weights(m, seed=5)
    g = torch.Generator(device="cuda").manual_seed(6)
    with torch.no_grad():  # the init leaves several matrices at zero: perturb every parameter
        for name, p in m.named_parameters():
            p.add_(torch.randn(p.shape, generator=g, device="cuda") * (0.02 if p.dim() > 1 else 0.01))
    idx = torch.randint(0, cfg.vocab_size, (1, 24), device="cuda", generator=g)
    with torch.no_grad():
        logits, aux = m(idx)
    sd = {k: v.detach().double().cpu() for k, v in m.state_dict().items()}
    ref, aux_r = mo.forward(sd, cfg, idx.cpu(), wkv="exact", dtype=torch.float64)
    assert rel_rms(logits.double().cpu().numpy(), ref.numpy()) < 2e-3
    assert abs(float(aux) - aux_r) < 1e-4 * max(1.0, abs(aux_r))


def test_config5_wkv_backward_micro_batch():
    from rwkv_mlx_b200 import wkv7

    B, T, H = 4, 1024, 16
    inp = wkv_inputs(B, T, H, seed=55)
    dt = torch.float16
    d, h = {}, {}
    for n, x in inp.items():
        t = torch.tensor(np.ascontiguousarray(x.reshape(B, T, -1)), dtype=dt, device="cuda")
        d[n], h[n] = t, t.double().cpu().numpy().reshape(x.shape)
    y, s, sa = wkv7.wkv7_forward(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"])
    grads = wkv7.wkv7_backward(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], d["dy"], s, sa)
    torch.cuda.synchronize()
    ge = wo.wkv7_backward_exact(h["r"], h["w"], h["k"], h["v"], h["a"], h["b"], h["dy"])
    for name, g, e in zip(["dr", "dw", "dk", "dv", "da", "db"], grads, ge[:6]):
        err = rel_rms(g.double().cpu().numpy(), e.reshape(B, T, -1))
        assert err < 2e-3, f"{name}: {err}"
