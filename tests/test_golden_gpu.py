"""The B200 path reproduces golden vectors computed by the reference's own code
(tests/golden/make_golden.py).  Tolerance 2e-3 relative to RMS (north star) unless
stated; routing compared as expert sets (the reference's slot order is unspecified)."""

import numpy as np
import pytest
import torch

from tests.golden.golden import golden, model_params, tiny_config, wkv_c1_inputs
from tests.inputs import rel_rms

pytestmark = pytest.mark.gpu


def _dev(x, dt=torch.float32):
    return torch.tensor(np.ascontiguousarray(x), dtype=dt, device="cuda")


def _bt(x):
    return x.reshape(x.shape[0], x.shape[1], -1)


def test_wkv_config1_matches_reference():
    from rwkv_mlx_b200 import wkv7

    G = golden()
    d = wkv_c1_inputs()
    args = [_dev(_bt(d[n])) for n in "rwkvab"]
    y, s, sa = wkv7.wkv7_forward(*args)
    grads = wkv7.wkv7_backward(*args, _dev(_bt(d["dy"])), s, sa)
    torch.cuda.synchronize()
    assert rel_rms(y.cpu().numpy(), G["wkv_c1_y"]) < 2e-3
    assert rel_rms(sa.cpu().numpy(), G["wkv_c1_sa"]) < 2e-3
    for n, g in zip(["dr", "dw", "dk", "dv", "da", "db"], grads):
        assert rel_rms(g.cpu().numpy(), G["wkv_c1_" + n]) < 2e-3, n


def test_wkv_fp16_matches_reference_kernel():
    from rwkv_mlx_b200 import wkv7

    G = golden()
    args = [_dev(G["wkv_h_in_" + n], torch.float16) for n in "rwkvab"]
    y, s, sa = wkv7.wkv7_forward(*args)
    grads = wkv7.wkv7_backward(*args, _dev(G["wkv_h_in_dy"], torch.float16), s, sa)
    torch.cuda.synchronize()
    assert rel_rms(y.double().cpu().numpy(), G["wkv_h_y"].astype(np.float64)) < 2e-3
    assert rel_rms(s.cpu().numpy(), G["wkv_h_s"]) < 2e-3
    for n, g in zip(["dr", "dw", "dk", "dv", "da", "db"], grads):
        assert rel_rms(g.double().cpu().numpy(), G["wkv_h_" + n].astype(np.float64)) < 3e-3, n


def _model(prefix, seed, moe=False, full=False):
    from rwkv_mlx_b200.model import RWKV, RWKVConfig

    cfg = RWKVConfig(**tiny_config(moe, full))
    m = RWKV(cfg).cuda()
    P = model_params(prefix, seed)
    sd = m.state_dict()
    assert set(P) == set(sd), set(P) ^ set(sd)  # same parameter names as the reference
    m.load_state_dict({k: torch.tensor(v).view(sd[k].shape) for k, v in P.items()})
    return cfg, m.eval()


def test_model_gpt_and_rnn_modes_match_reference():
    G = golden()
    cfg, m = _model("model", 2)
    with torch.no_grad():
        logits, aux = m(_dev(G["model_idx"], torch.long))
        assert rel_rms(logits.cpu().numpy(), G["model_logits"]) < 2e-3
        st = m.init_state()
        for i, tok in enumerate(G["model_rnn_tokens"]):
            lg, st = m.forward_rnn(int(tok), st)
            assert rel_rms(lg.cpu().numpy(), G["model_rnn_logits"][i]) < 1e-4
    for i in range(len(st)):
        assert rel_rms(st[i].cpu().numpy(), G[f"model_rnn_state_{i}"]) < 1e-4


def test_time_mixing_rnn_step_matches_reference():
    G = golden()
    cfg, m = _model("model", 2)
    att = m.blocks[1].att
    S = _dev(G["rnn_S"]).view(1, 2, 64, 64).contiguous()
    with torch.no_grad():
        out, _, S, _ = att.forward_rnn(_dev(G["rnn_x"]).view(1, -1), _dev(G["rnn_xprev"]).view(1, -1),
                                       _dev(G["rnn_vfirst"]).view(1, -1), S)
    assert rel_rms(out.cpu().numpy().reshape(-1), G["rnn_out"]) < 1e-4
    assert rel_rms(S.cpu().numpy().reshape(2, 64, 64), G["rnn_Snew"]) < 1e-5


def test_router_and_lora_moe_match_reference():
    from rwkv_mlx_b200.model import RWKV_CMix_x070, RWKVConfig
    from rwkv_mlx_b200.moe import LoRAMoE_CMix, Router

    G = golden()
    router = Router(64, 8, 2).cuda()
    with torch.no_grad():
        router.gate.weight.copy_(_dev(G["router_w"]))
        inds, scores, aux, z = router(_dev(G["router_x"]))
    inds, scores = inds.cpu().numpy().reshape(-1, 2), scores.cpu().numpy().reshape(-1, 2)
    ref_inds, ref_sc = G["router_inds"].reshape(-1, 2), G["router_scores"].reshape(-1, 2)
    for t in range(inds.shape[0]):
        assert set(inds[t]) == set(ref_inds[t])
        for slot in range(2):
            assert abs(scores[t, slot] - ref_sc[t][list(ref_inds[t]).index(inds[t, slot])]) < 1e-5
    assert abs(float(aux) - float(G["router_aux"])) < 1e-5
    assert abs(float(z) - float(G["router_z"])) < 1e-4

    base = RWKV_CMix_x070(RWKVConfig(n_layer=2, n_embd=64, dim_ffn=128), 1).cuda()
    moe = LoRAMoE_CMix(base, 8, 16, 2).cuda()
    with torch.no_grad():
        base.x_k.copy_(_dev(G["moe_xk"]))
        base.key.weight.copy_(_dev(G["moe_key"]))
        base.value.weight.copy_(_dev(G["moe_value"]))
        moe.lora_A.copy_(_dev(G["moe_A"]))
        moe.lora_B.copy_(_dev(G["moe_B"]))
        moe.router.gate.weight.copy_(_dev(G["moe_gate"]))
        out, aux, z = moe(_dev(G["moe_x"]))
        ortho = moe.orthogonal_loss()
    assert rel_rms(out.cpu().numpy(), G["moe_out"]) < 1e-4
    assert abs(float(aux) - float(G["moe_aux"])) < 1e-5 and abs(float(z) - float(G["moe_z"])) < 1e-4
    assert abs(float(ortho) - float(G["moe_ortho"])) < 1e-4 * float(G["moe_ortho"])


def test_model_with_lora_moe_matches_reference():
    G = golden()
    cfg, m = _model("modelmoe", 4, moe=True)
    with torch.no_grad():
        logits, aux = m(_dev(G["modelmoe_idx"], torch.long))
    assert rel_rms(logits.cpu().numpy(), G["modelmoe_logits"]) < 2e-3
    assert abs(float(aux) - float(G["modelmoe_aux"])) < 1e-4 * max(1.0, abs(float(G["modelmoe_aux"])))


def test_full_expert_moe_matches_reference():
    """MoE_CMix (moe.py:170-242) on the reference module's own output."""
    from rwkv_mlx_b200.model import RWKVConfig
    from rwkv_mlx_b200.moe import MoE_CMix

    G = golden()
    fm = MoE_CMix(RWKVConfig(n_layer=2, n_embd=64, dim_ffn=128), 1, 4, 2).cuda()
    with torch.no_grad():
        fm.x_k.copy_(_dev(G["fullmoe_xk"]))
        fm.expert_key.copy_(_dev(G["fullmoe_key"]))
        fm.expert_val.copy_(_dev(G["fullmoe_val"]))
        fm.router.gate.weight.copy_(_dev(G["fullmoe_gate"]))
        out, aux, z = fm(_dev(G["fullmoe_x"]))
        ortho = fm.orthogonal_loss()
    assert rel_rms(out.cpu().numpy(), G["fullmoe_out"]) < 1e-4
    assert abs(float(aux) - float(G["fullmoe_aux"])) < 1e-5 and abs(float(z) - float(G["fullmoe_z"])) < 1e-4
    assert float(ortho) == 0.0


def test_model_with_full_expert_moe_matches_reference():
    G = golden()
    cfg, m = _model("modelfull", 5, full=True)
    with torch.no_grad():
        logits, aux = m(_dev(G["modelfull_idx"], torch.long))
    assert rel_rms(logits.cpu().numpy(), G["modelfull_logits"]) < 2e-3
    assert abs(float(aux) - float(G["modelfull_aux"])) < 1e-4 * max(1.0, abs(float(G["modelfull_aux"])))


def test_converted_pytorch_checkpoint_runs_like_the_reference(tmp_path):
    """A PyTorch-layout RWKV-7 state dict (1-D mixing vectors, no layer-0 v0/v1/v2) of
    the golden model goes through the converter and the loader; the loaded model gives
    the reference model's logits."""
    from rwkv_mlx_b200 import checkpoint as ck
    from tests.golden.params import pth_state_dict, spec_from_arrays

    G = golden()
    sd = pth_state_dict(spec_from_arrays(G["model_spec_names"], G["model_spec_shapes"]), seed=2)
    torch.save(sd, tmp_path / "m.pth")
    ck.convert_pth(tmp_path / "m.pth", tmp_path / "out", "float32")
    m = ck.load_model(tmp_path / "out", device="cuda", dtype=torch.float32).eval()
    with torch.no_grad():
        logits, _ = m(_dev(G["model_idx"], torch.long))
    assert rel_rms(logits.cpu().numpy(), G["model_logits"]) < 2e-3


def test_reference_signature_rnn_functions_match_reference():
    """_time_mixing_rnn(layer_id, H, N, x, x_prev, v_first, state, att) and
    _channel_mixing_rnn(x, x_prev, ffn) with the reference's signatures and unbatched
    shapes (model.py:441-506); the caller's state is left unchanged, as with MLX arrays."""
    from rwkv_mlx_b200.model import _channel_mixing_rnn, _time_mixing_rnn

    G = golden()
    cfg, m = _model("model", 2)
    att, ffn = m.blocks[1].att, m.blocks[1].ffn
    S = _dev(G["rnn_S"])
    S_before = S.clone()
    with torch.no_grad():
        out, x_ret, S_new, vf = _time_mixing_rnn(1, cfg.n_head, cfg.head_size, _dev(G["rnn_x"]),
                                                 _dev(G["rnn_xprev"]), _dev(G["rnn_vfirst"]), S, att)
        cout, cx = _channel_mixing_rnn(_dev(G["cmix_rnn_x"]), _dev(G["cmix_rnn_xprev"]), ffn)
    assert out.shape == (128,) and S_new.shape == (cfg.n_head, 64, 64) and vf.shape == (128,)
    assert torch.equal(S, S_before)
    assert torch.equal(x_ret, _dev(G["rnn_x"]))
    assert rel_rms(out.cpu().numpy(), G["rnn_out"]) < 1e-4
    assert rel_rms(S_new.cpu().numpy(), G["rnn_Snew"]) < 1e-5
    assert torch.equal(vf, _dev(G["rnn_vfirst"]))  # layer 1 keeps v_first
    assert rel_rms(cout.cpu().numpy(), G["cmix_rnn_out"]) < 1e-4
    assert torch.equal(cx, _dev(G["cmix_rnn_x"]))


def test_router_config4_scale_matches_reference():
    """Router(768, 8, 2) on 4096 fp16 tokens: expert sets bit-exact with the reference's
    own router, scores to fp16 rounding, aux and z to fp32 rounding."""
    from rwkv_mlx_b200.moe import Router
    from tests.inputs import router_x

    G = golden()
    router = Router(768, 8, 2).cuda()
    with torch.no_grad():
        router.gate.weight.copy_(_dev(G["router4k_w"]))
        x = torch.tensor(router_x(4096, 768, seed=22), device="cuda").view(1, 4096, 768)
        inds, scores, aux, z = router(x)
    inds = inds.cpu().numpy().reshape(-1, 2).astype(np.int64)
    scores = scores.float().cpu().numpy().reshape(-1, 2)
    ref_i = G["router4k_inds"].reshape(-1, 2).astype(np.int64)
    ref_s = G["router4k_scores"].reshape(-1, 2).astype(np.float32)
    assert (np.sort(inds, -1) == np.sort(ref_i, -1)).all()
    for slot in range(2):
        j = np.where(ref_i[:, 0] == inds[:, slot], 0, 1)
        assert np.abs(scores[:, slot] - ref_s[np.arange(len(j)), j]).max() <= 1e-3
    assert abs(float(aux) - float(G["router4k_aux"])) < 1e-5
    assert abs(float(z) - float(G["router4k_z"])) < 1e-4 * max(1.0, float(G["router4k_z"]))
