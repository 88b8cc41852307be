"""The RWKV-v7 model shell on the B200 kernels vs the CPU restatement of
rwkv_mlx/model.py (GPT mode, RNN mode, prefill->decode hand-over).  Needs a GPU.

GPT mode runs the chunked WKV-7 kernel (TF32 operands): 2e-3 relative-to-RMS on
the logits.  RNN mode runs the fp32 step kernel: 1e-4."""

import numpy as np
import pytest
import torch

from oracle import model_oracle as mo
from tests.inputs import rel_rms

pytestmark = pytest.mark.gpu


def _tiny(moe=False, groupnorm="mlx", full=False, n_embd=128):
    from rwkv_mlx_b200.model import RWKV, RWKVConfig, init_weights

    kw = dict(n_layer=2, n_embd=n_embd, vocab_size=512, dim_ffn=256, groupnorm=groupnorm)
    if moe:
        kw.update(moe_num_experts=4, moe_top_k=2, moe_lora_rank=8)
    if full:
        kw.update(moe_num_experts=4, moe_top_k=2, moe_mode="full")
    cfg = RWKVConfig(**kw)
    torch.manual_seed(0)
    m = RWKV(cfg).cuda()
    init_weights(m, seed=1)
    g = torch.Generator(device="cuda").manual_seed(2)
    with torch.no_grad():
        # the init leaves several matrices at zero; perturb everything so every path is exercised
        for name, p in m.named_parameters():
            p.add_(torch.randn(p.shape, generator=g, device="cuda") * (0.05 if p.dim() > 1 else 0.02))
        m.emb.weight.mul_(1000.0)
    return cfg, m


def _sd(m):
    return {k: v.detach().double().cpu() for k, v in m.state_dict().items()}


@pytest.mark.parametrize("groupnorm", ["mlx", "per_head"])
def test_gpt_forward_matches_cpu_restatement(groupnorm):
    cfg, m = _tiny(groupnorm=groupnorm)
    idx = torch.randint(0, cfg.vocab_size, (2, 40), device="cuda")
    with torch.no_grad():
        logits, aux = m(idx)
    ref, aux_r = mo.forward(_sd(m), cfg, idx.cpu(), wkv="exact", dtype=torch.float64)
    assert rel_rms(logits.double().cpu().numpy(), ref.numpy()) < 2e-3
    assert float(aux) == 0.0 and aux_r == 0.0


def test_gpt_forward_with_lora_moe_matches_cpu_restatement():
    cfg, m = _tiny(moe=True)
    idx = torch.randint(0, cfg.vocab_size, (2, 32), device="cuda")
    with torch.no_grad():
        logits, aux = m(idx)
    ref, aux_r = mo.forward(_sd(m), cfg, idx.cpu(), wkv="exact", dtype=torch.float64)
    assert rel_rms(logits.double().cpu().numpy(), ref.numpy()) < 2e-3
    assert abs(float(aux) - aux_r) < 1e-4 * max(1.0, abs(aux_r))


def test_gpt_forward_with_full_expert_moe_matches_cpu_restatement():
    cfg, m = _tiny(full=True)
    idx = torch.randint(0, cfg.vocab_size, (2, 32), device="cuda")
    with torch.no_grad():
        logits, aux = m(idx)
    ref, aux_r = mo.forward(_sd(m), cfg, idx.cpu(), wkv="exact", dtype=torch.float64)
    assert rel_rms(logits.double().cpu().numpy(), ref.numpy()) < 2e-3
    assert abs(float(aux) - aux_r) < 1e-4 * max(1.0, abs(aux_r))


def test_rnn_mode_matches_cpu_restatement():
    cfg, m = _tiny()
    st_g = m.init_state()
    st_c = mo.init_state(cfg)
    sd = _sd(m)
    for tok in [5, 77, 300, 2, 511]:
        with torch.no_grad():
            lg, st_g = m.forward_rnn(tok, st_g)
        lc, st_c = mo.forward_rnn(sd, cfg, tok, st_c)
        assert rel_rms(lg.double().cpu().numpy(), lc.numpy()) < 1e-4


@pytest.mark.parametrize("moe", ["none", "lora", "full"])
def test_prefill_state_then_decode_equals_gpt_forward(moe):
    """Prefill 24 tokens in GPT mode with state output, decode 6 more in RNN mode
    (batched): logits equal a GPT-mode pass over all 30 tokens."""
    cfg, m = _tiny(moe=moe == "lora", full=moe == "full")
    idx = torch.randint(0, cfg.vocab_size, (3, 30), device="cuda")
    with torch.no_grad():
        full, _ = m(idx)
        _, _, states = m.forward_with_state(idx[:, :24])
        outs = []
        for t in range(24, 30):
            outs.append(m.forward_rnn_batch(idx[:, t], states))
    dec = torch.stack(outs, 1)
    assert rel_rms(dec.double().cpu().numpy(), full[:, 24:].double().cpu().numpy()) < 2e-3


def test_fp16_model_close_to_fp32():
    from rwkv_mlx_b200.model import cast_for_inference

    cfg, m = _tiny()
    idx = torch.randint(0, cfg.vocab_size, (2, 64), device="cuda")
    with torch.no_grad():
        ref, _ = m(idx)
        cast_for_inference(m, torch.float16)
        assert m.blocks[0].att.w0.dtype == torch.float32
        out, _ = m(idx)
    assert rel_rms(out.double().cpu().numpy(), ref.double().cpu().numpy()) < 2e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_fused_path_matches_op_by_op_path(dtype):
    """The fused element-wise kernels give the same logits as the op-by-op torch path."""
    from rwkv_mlx_b200.model import cast_for_inference

    for moe in (False, True):
        cfg, m = _tiny(moe=moe)
        if dtype == torch.float16:
            cast_for_inference(m, torch.float16)
        idx = torch.randint(0, cfg.vocab_size, (2, 48), device="cuda")
        with torch.no_grad():
            cfg.fused = True
            a, aux_a = m(idx)
            cfg.fused = False
            b, aux_b = m(idx)
            cfg.fused = True
        tol = 1e-4 if dtype == torch.float32 else 3e-3
        assert rel_rms(a.double().cpu().numpy(), b.double().cpu().numpy()) < tol, moe
        assert abs(float(aux_a) - float(aux_b)) < 1e-4 * max(1.0, abs(float(aux_b)))


@pytest.mark.parametrize("groupnorm", ["mlx", "per_head"])
def test_fused_path_with_an_odd_head_count(groupnorm):
    """C = 192 (3 heads): the fused kernels' per-warp staging and group statistics on a
    head count that is not a multiple of 2, against the op-by-op path and the oracle."""
    cfg, m = _tiny(groupnorm=groupnorm, n_embd=192)
    idx = torch.randint(0, cfg.vocab_size, (2, 40), device="cuda")
    with torch.no_grad():
        cfg.fused = True
        a, _ = m(idx)
        cfg.fused = False
        b, _ = m(idx)
        cfg.fused = True
    assert rel_rms(a.double().cpu().numpy(), b.double().cpu().numpy()) < 1e-4
    ref, _ = mo.forward(_sd(m), cfg, idx.cpu(), wkv="exact", dtype=torch.float64)
    assert rel_rms(a.double().cpu().numpy(), ref.numpy()) < 2e-3


def test_fused_per_head_groupnorm_and_state_output():
    cfg, m = _tiny(groupnorm="per_head")
    idx = torch.randint(0, cfg.vocab_size, (2, 40), device="cuda")
    with torch.no_grad():
        la, _, sa = m.forward_with_state(idx)
        cfg.fused = False
        lb, _, sb = m.forward_with_state(idx)
        cfg.fused = True
    assert rel_rms(la.cpu().numpy(), lb.cpu().numpy()) < 1e-4
    for x, y in zip(sa, sb):
        for key in x:
            assert rel_rms(x[key].float().cpu().numpy(), y[key].float().cpu().numpy()) < 1e-4, key


def test_decode_graph_matches_eager_decode():
    from rwkv_mlx_b200.model import DecodeGraph

    cfg, m = _tiny()
    idx = torch.randint(0, cfg.vocab_size, (4, 20), device="cuda")
    with torch.no_grad():
        _, _, st_a = m.forward_with_state(idx)
        _, _, st_b = m.forward_with_state(idx)
        tok = idx[:, -1].clone()
        eager = []
        t = tok.clone()
        for _ in range(5):
            t = m.forward_rnn_batch(t, st_a).argmax(-1)
            eager.append(t.clone())
    g = DecodeGraph(m, st_b, tok)
    graphed = [g.step().clone() for _ in range(5)]
    for a, b in zip(eager, graphed):
        assert torch.equal(a, b)
    # an in-place weight update after the capture: the graph refuses to replay stale copies
    with torch.no_grad():
        m.blocks[0].att.key.weight.mul_(1.0)
    with pytest.raises(RuntimeError, match="DecodeGraph"):
        g.step()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_fused_rnn_step_matches_op_by_op(dtype):
    """RNN-mode batched step on the fused kernels (lerp with the stored previous token,
    TimeMix mid/post, relu^2, add+LayerNorm) equals the op-by-op path, states included."""
    from rwkv_mlx_b200.model import cast_for_inference

    for moe in (False, True):
        cfg, m = _tiny(moe=moe)
        if dtype == torch.float16:
            cast_for_inference(m, torch.float16)
        idx = torch.randint(0, cfg.vocab_size, (3, 20), device="cuda")
        with torch.no_grad():
            _, _, st_a = m.forward_with_state(idx)
            _, _, st_b = m.forward_with_state(idx)
            tok = idx[:, -1]
            for _ in range(4):
                cfg.fused = True
                la = m.forward_rnn_batch(tok, st_a)
                cfg.fused = False
                lb = m.forward_rnn_batch(tok, st_b)
                cfg.fused = True
                tol = 1e-4 if dtype == torch.float32 else 3e-3
                assert rel_rms(la.double().cpu().numpy(), lb.double().cpu().numpy()) < tol, moe
                tok = lb.argmax(-1)
        for x, y in zip(st_a, st_b):
            for key in x:
                assert rel_rms(x[key].float().cpu().numpy(), y[key].float().cpu().numpy()) < 1e-2, key


@pytest.mark.parametrize("dt,T", [(torch.float16, 1), (torch.float32, 1), (torch.bfloat16, 7)])
def test_lerp_writes_the_next_shift_state(dt, T):
    """rwkv_lerp_prev_state: the mixes as rwkv_lerp_prev computes them, and each sequence's
    last row stored as the next state (in place over the old state when T == 1)."""
    from rwkv_mlx_b200 import fused as fz

    rows, C = 21 * T, 768
    g = torch.Generator(device="cuda").manual_seed(T)
    x = torch.randn(rows, C, device="cuda", generator=g).to(dt)
    mix = torch.rand(6, C, device="cuda", generator=g).to(dt)
    state = torch.randn(rows // T, C, device="cuda", generator=g).to(dt)
    ref = fz.lerp(x, mix, T, prev=state.clone())
    dest = state if T == 1 else torch.empty_like(state)
    out = fz.lerp(x, mix, T, prev=state, prev_out=dest)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert torch.equal(dest, x.view(rows // T, T, C)[:, -1])


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
def test_lora_act_matches_torch(dt):
    """One-launch tanh (slice 1) / sigmoid (slice 3) of the stacked LoRA hidden."""
    from rwkv_mlx_b200 import fused as fz

    h = (3 * torch.randn(4, 300, 128, device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))).to(dt)
    ref = h.clone()
    ref[1] = torch.tanh(ref[1].float()).to(dt)
    ref[3] = torch.sigmoid(ref[3].float()).to(dt)
    fz.lora_act_(h)
    torch.cuda.synchronize()
    assert torch.equal(h[0], ref[0]) and torch.equal(h[2], ref[2])
    tol = {torch.float16: 1e-3, torch.bfloat16: 8e-3, torch.float32: 1e-6}[dt]
    assert (h.float() - ref.float()).abs().max().item() <= tol


@pytest.mark.parametrize("dt,V", [(torch.float16, 65536), (torch.bfloat16, 1000), (torch.float32, 777)])
def test_argmax_rows_matches_torch(dt, V):
    """Row argmax for greedy decoding: first index of the maximum, ties included."""
    from rwkv_mlx_b200 import fused as fz

    g = torch.Generator(device="cuda").manual_seed(V)
    x = torch.randn(37, V, device="cuda", generator=g).to(dt)
    x[5, :] = 1.0  # all tied: index 0
    x[6, V // 3] = x[6, 2 * V // 3] = x[6].max() + 1  # two tied maxima: the first
    got = fz.argmax_rows(x)
    torch.cuda.synchronize()
    assert torch.equal(got, x.argmax(-1))
    assert got[5].item() == 0 and got[6].item() == V // 3


@pytest.mark.parametrize("dt,C,with_delta", [(torch.float16, 768, True), (torch.bfloat16, 64, False),
                                             (torch.float32, 2048, True), (torch.float16, 4096, True)])
def test_add_layernorm_matches_torch(dt, C, with_delta):
    """Residual add + LayerNorm (registers for C <= 256 vectors, three passes beyond)."""
    from rwkv_mlx_b200 import fused as fz

    g = torch.Generator(device="cuda").manual_seed(C)
    x = torch.randn(333, C, device="cuda", generator=g).to(dt)
    d = torch.randn(333, C, device="cuda", generator=g).to(dt) if with_delta else None
    w = (1 + 0.1 * torch.randn(C, device="cuda", generator=g)).to(dt)
    b = (0.1 * torch.randn(C, device="cuda", generator=g)).to(dt)
    xs, y = fz.add_layernorm(x, d, w, b, 1e-5)
    torch.cuda.synchronize()
    ref_x = (x + d) if with_delta else x
    assert torch.equal(xs, ref_x)
    ref_y = torch.nn.functional.layer_norm(ref_x.float(), (C,), w.float(), b.float(), 1e-5)
    tol = {torch.float16: 4e-3, torch.bfloat16: 3e-2, torch.float32: 1e-5}[dt]
    assert (y.float() - ref_y).abs().max().item() < tol


def test_prefill_graph_matches_eager_forward():
    """model.PrefillGraph (the GPT-mode forward captured as a CUDA graph) gives the eager
    forward's logits for new inputs copied into it, and refuses stale weights."""
    from rwkv_mlx_b200.model import PrefillGraph

    for moe in (False, True):
        cfg, m = _tiny(moe=moe)
        g = PrefillGraph(m, 2, 48)
        for seed in (0, 1):
            idx = torch.randint(0, cfg.vocab_size, (2, 48), device="cuda",
                                generator=torch.Generator(device="cuda").manual_seed(seed))
            with torch.no_grad():
                ref, ref_aux = m(idx)
            got, aux = g(idx.cpu().pin_memory())
            torch.cuda.synchronize()
            assert rel_rms(got.float().cpu().numpy(), ref.float().cpu().numpy()) < 1e-5
            assert abs(float(aux) - float(ref_aux)) < 1e-6 * max(1.0, abs(float(ref_aux)))
        with torch.no_grad():
            m.head.weight.mul_(1.0)
        with pytest.raises(RuntimeError, match="PrefillGraph"):
            g()


def test_channel_mix_fused_key_gemm_matches_op_by_op():
    """At >= 24576 rows the fused ChannelMix runs key + squared ReLU as one tcgen05 GEMM;
    its output matches the op-by-op torch path (key product rounded to fp16, relu, square,
    value product)."""
    from rwkv_mlx_b200 import model as md

    cfg = md.RWKVConfig(n_layer=2, n_embd=768, dim_ffn=3072)
    torch.manual_seed(3)
    cm = md.RWKV_CMix_x070(cfg, 1).cuda()
    with torch.no_grad():
        cm.x_k.uniform_(0, 1)
        cm.key.weight.normal_(0, 768 ** -0.5)
        cm.value.weight.normal_(0, 3072 ** -0.5)
    cm = cm.half()
    B, T = 6, 4096
    assert B * T >= md._FUSED_KEY_MIN_ROWS
    x = torch.randn(B, T, 768, device="cuda").half()
    with torch.no_grad():
        fused = cm(x)
        cfg.fused = False
        try:
            ref = cm(x)
        finally:
            cfg.fused = True
    torch.cuda.synchronize()
    assert rel_rms(fused.double().cpu().numpy(), ref.double().cpu().numpy()) < 3e-3

