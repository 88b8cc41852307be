"""The CPU oracles reproduce golden vectors computed by the reference's own code
(rwkv_mlx model.py / moe.py / wkv7_metal.py, see tests/golden/make_golden.py)."""

import numpy as np
import torch

from oracle import model_oracle, moe_oracle, wkv7_oracle
from rwkv_mlx_b200.model import RWKVConfig
from tests.golden.golden import golden, model_params, tiny_config, wkv_c1_inputs
from tests.inputs import rel_rms


def _bt(x):
    return x.reshape(x.shape[0], x.shape[1], -1)


def test_wkv_config1_forward_and_backward():
    G = golden()
    d = wkv_c1_inputs()
    args = [d[n].astype(np.float32).astype(np.float64) for n in "rwkvab"]
    y, sa, _, _ = wkv7_oracle.wkv7_forward_exact(*args)
    assert rel_rms(_bt(y), G["wkv_c1_y"]) < 1e-6
    assert rel_rms(sa, G["wkv_c1_sa"]) < 1e-6
    g = wkv7_oracle.wkv7_backward_exact(*args, d["dy"].astype(np.float32).astype(np.float64))
    for n, e in zip(["dr", "dw", "dk", "dv", "da", "db"], g[:6]):
        assert rel_rms(_bt(e), G["wkv_c1_" + n]) < 1e-4, n  # the reference divides by the decay


def test_wkv_fp16_kernel():
    G = golden()
    args = [G["wkv_h_in_" + n].astype(np.float64).reshape(1, 48, 2, 64) for n in "rwkvab"]
    y, sa, _, st = wkv7_oracle.wkv7_forward_exact(*args, keep_states=True)
    assert rel_rms(_bt(y), G["wkv_h_y"].astype(np.float64)) < 1e-3
    assert rel_rms(sa, G["wkv_h_sa"]) < 1e-5
    assert rel_rms(wkv7_oracle.checkpoints_from_states(st, 16).reshape(-1), G["wkv_h_s"]) < 1e-5


def test_router_and_lora_moe():
    G = golden()
    lg = moe_oracle.gate_logits(G["router_x"].reshape(-1, 64), G["router_w"])
    inds, scores, aux, z, _ = moe_oracle.router(None, None, 2, logits=lg)
    ref_inds = G["router_inds"].reshape(-1, 2)
    ref_sc = G["router_scores"].reshape(-1, 2)
    for t in range(inds.shape[0]):  # argpartition's slot order is unspecified: compare as sets
        assert set(inds[t]) == set(ref_inds[t])
        for slot in range(2):
            e = inds[t, slot]
            assert abs(scores[t, slot] - ref_sc[t][list(ref_inds[t]).index(e)]) < 1e-5
    assert abs(aux - float(G["router_aux"])) < 1e-5 and abs(z - float(G["router_z"])) < 1e-4

    x = G["moe_x"].astype(np.float64)
    base = moe_oracle.cmix(x, G["moe_xk"], G["moe_key"], G["moe_value"])
    lg = moe_oracle.gate_logits(x.reshape(-1, 64), G["moe_gate"])
    inds, scores, aux, z, _ = moe_oracle.router(None, None, 2, logits=lg)
    out = base + moe_oracle.lora_moe_delta(x, G["moe_A"], G["moe_B"], inds.reshape(2, 24, 2), scores.reshape(2, 24, 2))
    assert rel_rms(out, G["moe_out"]) < 1e-5
    assert abs(aux - float(G["moe_aux"])) < 1e-5 and abs(z - float(G["moe_z"])) < 1e-4
    assert abs(moe_oracle.orthogonal_loss(G["moe_A"]) - float(G["moe_ortho"])) < 1e-4 * float(G["moe_ortho"])


def _sd(P):
    return {k: torch.tensor(v, dtype=torch.float64) for k, v in P.items()}


def test_model_gpt_and_rnn_modes():
    G = golden()
    cfg = RWKVConfig(**tiny_config())
    P = _sd(model_params("model", seed=2))
    logits, aux = model_oracle.forward(P, cfg, torch.tensor(G["model_idx"]).long(), wkv="exact", dtype=torch.float64)
    assert rel_rms(logits.numpy(), G["model_logits"]) < 1e-5
    st = model_oracle.init_state(cfg)
    for i, tok in enumerate(G["model_rnn_tokens"]):
        lg, st = model_oracle.forward_rnn(P, cfg, int(tok), st)
        assert rel_rms(lg.numpy(), G["model_rnn_logits"][i]) < 1e-5
    for i in range(len(st)):
        assert rel_rms(st[i].numpy(), G[f"model_rnn_state_{i}"]) < 1e-5


def test_model_groupnorm_grouping_is_mlx_strided():
    """Per-head grouping gives different logits: the fixture pins MLX's strided groups."""
    G = golden()
    cfg = RWKVConfig(**tiny_config(), groupnorm="per_head")
    P = _sd(model_params("model", seed=2))
    logits, _ = model_oracle.forward(P, cfg, torch.tensor(G["model_idx"]).long(), wkv="exact", dtype=torch.float64)
    assert rel_rms(logits.numpy(), G["model_logits"]) > 1e-2


def test_model_with_lora_moe():
    G = golden()
    cfg = RWKVConfig(**tiny_config(moe=True))
    P = _sd(model_params("modelmoe", seed=4))
    logits, aux = model_oracle.forward(P, cfg, torch.tensor(G["modelmoe_idx"]).long(), wkv="exact",
                                       dtype=torch.float64)
    assert rel_rms(logits.numpy(), G["modelmoe_logits"]) < 1e-5
    assert abs(aux - float(G["modelmoe_aux"])) < 1e-5 * max(1.0, abs(aux))


def test_full_expert_moe():
    """MoE_CMix (moe.py:226-242): the dense expert loop of the oracle against the
    reference module's own output."""
    G = golden()
    x = G["fullmoe_x"].astype(np.float64)
    lg = moe_oracle.gate_logits(x.reshape(-1, 64), G["fullmoe_gate"])
    inds, scores, aux, z, _ = moe_oracle.router(None, None, 2, logits=lg)
    out = moe_oracle.full_moe(x, G["fullmoe_xk"], G["fullmoe_key"], G["fullmoe_val"], inds.reshape(2, 24, 2),
                              scores.reshape(2, 24, 2))
    assert rel_rms(out, G["fullmoe_out"]) < 1e-5
    assert abs(aux - float(G["fullmoe_aux"])) < 1e-5 and abs(z - float(G["fullmoe_z"])) < 1e-4


def test_model_with_full_expert_moe():
    G = golden()
    cfg = RWKVConfig(**tiny_config(full=True))
    P = _sd(model_params("modelfull", seed=5))
    logits, aux = model_oracle.forward(P, cfg, torch.tensor(G["modelfull_idx"]).long(), wkv="exact",
                                       dtype=torch.float64)
    assert rel_rms(logits.numpy(), G["modelfull_logits"]) < 1e-5
    assert abs(aux - float(G["modelfull_aux"])) < 1e-5 * max(1.0, abs(aux))


def test_l2_wrap_losses():
    """train.py:317-362 restated in torch float64 against the reference functions."""
    from oracle import loss_oracle

    G = golden()
    lg = torch.tensor(G["loss_logits"], dtype=torch.float64)
    tg = torch.tensor(G["loss_targets"])
    mk = torch.tensor(G["loss_mask"], dtype=torch.float64)
    assert abs(float(loss_oracle.l2_wrap_loss(lg, tg)) - float(G["loss_l2wrap"])) < 1e-5
    assert abs(float(loss_oracle.l2_wrap_loss_masked(lg, tg, mk)) - float(G["loss_l2wrap_masked"])) < 1e-5


def test_router_at_config4_scale_matches_reference():
    """4096 fp16 tokens, E=8, top-2 (moe.py:51-86): the oracle's own float64 logits route
    every token to the same expert set as the reference's float32 router; the scores,
    aux and z agree to float32 rounding."""
    import hashlib

    from tests.inputs import router_x

    G = golden()
    x = router_x(4096, 768, seed=22)
    assert np.array_equal(np.frombuffer(hashlib.sha256(x.tobytes()).digest(), np.uint8), G["router4k_x_sha256"])
    inds, scores, aux, z, _ = moe_oracle.router(x, G["router4k_w"], 2)
    ref_i = G["router4k_inds"].reshape(-1, 2)
    ref_s = G["router4k_scores"].reshape(-1, 2).astype(np.float64)
    assert (np.sort(inds, -1) == np.sort(ref_i.astype(np.int64), -1)).all()
    for slot in range(2):  # reference slot order is unspecified: match scores by expert
        j = np.where(ref_i[:, 0] == inds[:, slot], 0, 1)
        assert np.abs(scores[:, slot] - ref_s[np.arange(len(j)), j]).max() < 1e-3  # fp16 scores
    assert abs(aux - float(G["router4k_aux"])) < 1e-5
    assert abs(z - float(G["router4k_z"])) < 1e-4 * max(1.0, z)


def test_channel_mixing_rnn_step():
    """_channel_mixing_rnn (model.py:498-506) of the tiny model's layer 1."""
    G = golden()
    P = model_params("model", seed=2)
    x, xp = G["cmix_rnn_x"].astype(np.float64), G["cmix_rnn_xprev"].astype(np.float64)
    xk = P["blocks.1.ffn.x_k"].reshape(-1).astype(np.float64)
    kw, vw = P["blocks.1.ffn.key.weight"].astype(np.float64), P["blocks.1.ffn.value.weight"].astype(np.float64)
    k = np.maximum(kw @ (x + (xp - x) * xk), 0) ** 2
    assert rel_rms(vw @ k, G["cmix_rnn_out"]) < 1e-5
