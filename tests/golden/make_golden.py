"""Generate golden vectors by running the reference's own Python code.

Run where the reference checkout is available, at ``$RWKV_MLX_REFERENCE`` or (the
default) in a directory named ``reference`` beside this repository:

    python tests/golden/make_golden.py

It imports rwkv_mlx/model.py, rwkv_mlx/moe.py and rwkv_mlx/kernels/wkv7_metal.py
unmodified, with the numpy-backed MLX stand-in of tests/golden/mlx_shim on the path;
`mx.fast.metal_kernel` there compiles the reference's Metal kernel bodies as C++
(oracle/metal_cpu.py).  Outputs: tests/golden/reference_golden.npz.

Cases (all seeded):
  wkv_c1_*   BASELINE config 1 (B=1, T=256, H=4, fp32): wkv7_metal_forward y, sa and
             wkv7_metal_backward's six gradients; inputs are tests/inputs.wkv_inputs(1, 256, 4,
             seed=0) (their SHA-256 is stored and checked before use).
  wkv_h_*    fp16 case (B=1, T=48, H=2): forward y, s, sa and backward gradients.
  rnn_*      _time_mixing_rnn on layer 1 of the tiny model.
  router_*   Router(64, 8, 2) on x (2, 16, 64).
  moe_*      LoRAMoE_CMix(base C=64 F=128, E=8, r=16, k=2) forward + orthogonal_loss.
  model_*    RWKV L2 D128 (vocab 256, ffn 256): GPT-mode logits (B=2, T=32) and six
             RNN-mode steps; modelmoe_* the same model with LoRA-MoE in every layer,
             modelfull_* with full-expert MoE_CMix in every layer.
  fullmoe_*  MoE_CMix(C=64, F=128, E=4, k=2) forward.
  loss_*     l2_wrap_loss and l2_wrap_loss_masked (train.py:317-362).
  cmix_rnn_* _channel_mixing_rnn on layer 1 of the tiny model.
  router4k_* Router(768, 8, 2) on 4096 fp16 tokens (x regenerated from a seed by
             tests/inputs.router_x, its SHA-256 stored), as BASELINE configs[3]'s router
             sees them (without the harness's logit bias: the reference router has none).
  conv_*     convert_pytorch_to_mlx (convert.py:16-141) on a PyTorch-layout state dict of
             the tiny model: names, shapes, dtypes and SHA-256 of every converted tensor,
             and the inferred config.
             Model parameters are drawn by tests/golden/params.py from the stored
             (name, shape) spec and seed; their SHA-256 is stored.
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
REF = Path(os.environ.get("RWKV_MLX_REFERENCE", str(ROOT.parent / "reference")))
sys.path.insert(0, str(HERE / "mlx_shim"))
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(REF))


def walk(obj, prefix, out, nn):
    for k, v in vars(obj).items():
        if isinstance(v, np.ndarray):
            out[prefix + k] = v
        elif isinstance(v, nn.Module):
            walk(v, prefix + k + ".", out, nn)
        elif isinstance(v, list):
            for i, m in enumerate(v):
                if isinstance(m, nn.Module):
                    walk(m, f"{prefix}{k}.{i}.", out, nn)


def set_params(model, params):
    for name, val in params.items():
        obj = model
        parts = name.split(".")
        for p in parts[:-1]:
            obj = obj[int(p)] if isinstance(obj, list) else getattr(obj, p)
        old = getattr(obj, parts[-1])
        assert old.shape == val.shape, (name, old.shape, val.shape)
        setattr(obj, parts[-1], val.astype(np.float32))


def ref_mx_load(path):
    import mlx.core as mx

    return mx.load(path)


def spec_of(model, nn):
    names = {}
    walk(model, "", names, nn)
    return [(n, v.shape) for n, v in names.items()]


def main():
    from tests.golden.params import params_sha256, random_params, spec_arrays
    from tests.inputs import wkv_inputs

    import mlx.nn as nn
    from rwkv_mlx import model as ref_model
    from rwkv_mlx import moe as ref_moe
    import importlib

    wkv7_metal = importlib.import_module("rwkv_mlx.kernels.wkv7_metal")

    G = {}
    # ---- WKV-7, config 1 ----
    d = wkv_inputs(1, 256, 4, seed=0)
    h = hashlib.sha256()
    for n in "rwkvab":
        h.update(np.ascontiguousarray(d[n], np.float64).tobytes())
    h.update(np.ascontiguousarray(d["dy"], np.float64).tobytes())
    G["wkv_c1_input_sha256"] = np.frombuffer(h.digest(), np.uint8)
    bt = lambda x, dt: np.ascontiguousarray(x.reshape(x.shape[0], x.shape[1], -1), dt)
    args = [bt(d[n], np.float32) for n in "rwkvab"]
    y, s, sa = wkv7_metal.wkv7_metal_forward(*args)
    grads = wkv7_metal.wkv7_metal_backward(*args, bt(d["dy"], np.float32), s, sa)
    G["wkv_c1_y"], G["wkv_c1_sa"] = y, sa
    for n, gv in zip(["dr", "dw", "dk", "dv", "da", "db"], grads):
        G["wkv_c1_" + n] = gv
    # ---- WKV-7, fp16 ----
    d = wkv_inputs(1, 48, 2, seed=1)
    args = [bt(d[n], np.float16) for n in "rwkvab"]
    y, s, sa = wkv7_metal.wkv7_metal_forward(*args)
    grads = wkv7_metal.wkv7_metal_backward(*args, bt(d["dy"], np.float16), s, sa)
    for n, x in zip("rwkvab", args):
        G["wkv_h_in_" + n] = x
    G["wkv_h_in_dy"] = bt(d["dy"], np.float16)
    G["wkv_h_y"], G["wkv_h_s"], G["wkv_h_sa"] = y, s, sa
    for n, gv in zip(["dr", "dw", "dk", "dv", "da", "db"], grads):
        G["wkv_h_" + n] = gv

    # ---- tiny model (plain) ----
    cfg = ref_model.RWKVConfig(n_layer=2, n_embd=128, vocab_size=256, dim_ffn=256)
    m = ref_model.RWKV(cfg)
    spec = spec_of(m, nn)
    P = random_params(spec, seed=2)
    set_params(m, P)
    G["model_spec_names"], G["model_spec_shapes"] = spec_arrays(spec)
    G["model_params_sha256"] = params_sha256(P)
    rng = np.random.default_rng(3)
    idx = rng.integers(0, 256, (2, 32)).astype(np.int32)
    logits, aux = m(idx)
    G["model_idx"], G["model_logits"], G["model_aux"] = idx, logits, np.array(aux)
    state = m.init_state()
    toks = rng.integers(0, 256, 6)
    outs = []
    for t in toks:
        lg, state = m.forward_rnn(int(t), state)
        outs.append(lg)
    G["model_rnn_tokens"], G["model_rnn_logits"] = toks.astype(np.int32), np.stack(outs)
    for i, st in enumerate(state):
        G[f"model_rnn_state_{i}"] = st

    # ---- _time_mixing_rnn on layer 1 ----
    att = m.blocks[1].att
    H, N = cfg.n_head, cfg.head_size
    x = rng.standard_normal(128).astype(np.float32)
    xp = rng.standard_normal(128).astype(np.float32)
    vf = rng.standard_normal(128).astype(np.float32)
    S = (0.3 * rng.standard_normal((H, N, N))).astype(np.float32)
    out, xo, So, vfo = ref_model._time_mixing_rnn(1, H, N, x, xp, vf, S.copy(), att)
    G.update(rnn_x=x, rnn_xprev=xp, rnn_vfirst=vf, rnn_S=S, rnn_out=out, rnn_Snew=So)

    # ---- Router and LoRA-MoE ----
    router = ref_moe.Router(64, 8, 2)
    router.gate.weight = (rng.standard_normal((8, 64)) * 0.3).astype(np.float32)
    xr = rng.standard_normal((2, 16, 64)).astype(np.float32)
    inds, scores, aux, z = router(xr)
    G.update(router_w=router.gate.weight, router_x=xr, router_inds=inds, router_scores=scores,
             router_aux=np.array(aux), router_z=np.array(z))
    base = ref_model.RWKV_CMix_x070(ref_model.RWKVConfig(n_layer=2, n_embd=64, dim_ffn=128), 1)
    base.x_k = rng.uniform(0, 1, (1, 1, 64)).astype(np.float32)
    base.key.weight = (rng.standard_normal((128, 64)) / 8).astype(np.float32)
    base.value.weight = (rng.standard_normal((64, 128)) / 11).astype(np.float32)
    moe = ref_moe.LoRAMoE_CMix(base, n_experts=8, lora_rank=16, top_k=2)
    moe.lora_A = rng.normal(0, 0.02 * 5, (8, 64, 16)).astype(np.float32)
    moe.lora_B = rng.normal(0, 0.02 * 5, (8, 16, 64)).astype(np.float32)
    moe.router.gate.weight = (rng.standard_normal((8, 64)) * 0.3).astype(np.float32)
    xm = rng.standard_normal((2, 24, 64)).astype(np.float32)
    out, aux, z = moe(xm)
    G.update(moe_xk=base.x_k, moe_key=base.key.weight, moe_value=base.value.weight, moe_A=moe.lora_A,
             moe_B=moe.lora_B, moe_gate=moe.router.gate.weight, moe_x=xm, moe_out=out,
             moe_aux=np.array(aux), moe_z=np.array(z), moe_ortho=np.array(moe.orthogonal_loss()))

    # ---- tiny model with LoRA-MoE in every layer ----
    cfg2 = ref_model.RWKVConfig(n_layer=2, n_embd=128, vocab_size=256, dim_ffn=256, moe_num_experts=4,
                                moe_top_k=2, moe_lora_rank=8)
    m2 = ref_model.RWKV(cfg2)
    spec2 = spec_of(m2, nn)
    P2 = random_params(spec2, seed=4)
    set_params(m2, P2)
    G["modelmoe_spec_names"], G["modelmoe_spec_shapes"] = spec_arrays(spec2)
    G["modelmoe_params_sha256"] = params_sha256(P2)
    idx2 = rng.integers(0, 256, (2, 24)).astype(np.int32)
    logits2, aux2 = m2(idx2)
    G["modelmoe_idx"], G["modelmoe_logits"], G["modelmoe_aux"] = idx2, logits2, np.array(aux2)

    # ---- full-expert MoE_CMix (moe.py:170-242) ----
    fcfg = ref_model.RWKVConfig(n_layer=2, n_embd=64, dim_ffn=128)
    fm = ref_moe.MoE_CMix(fcfg, 1, n_experts=4, top_k=2)
    fm.x_k = rng.uniform(0, 1, (4, 1, 1, 64)).astype(np.float32)
    fm.expert_key = (rng.standard_normal((4, 128, 64)) / 8).astype(np.float32)
    fm.expert_val = (rng.standard_normal((4, 64, 128)) / 11).astype(np.float32)
    fm.router.gate.weight = (rng.standard_normal((4, 64)) * 0.3).astype(np.float32)
    xf = rng.standard_normal((2, 24, 64)).astype(np.float32)
    outf, auxf, zf = fm(xf)
    G.update(fullmoe_xk=fm.x_k, fullmoe_key=fm.expert_key, fullmoe_val=fm.expert_val,
             fullmoe_gate=fm.router.gate.weight, fullmoe_x=xf, fullmoe_out=outf,
             fullmoe_aux=np.array(auxf), fullmoe_z=np.array(zf))

    # ---- tiny model with full-expert MoE in every layer ----
    cfg3 = ref_model.RWKVConfig(n_layer=2, n_embd=128, vocab_size=256, dim_ffn=256, moe_num_experts=4,
                                moe_top_k=2, moe_mode="full")
    m3 = ref_model.RWKV(cfg3)
    spec3 = spec_of(m3, nn)
    P3 = random_params(spec3, seed=5)
    set_params(m3, P3)
    G["modelfull_spec_names"], G["modelfull_spec_shapes"] = spec_arrays(spec3)
    G["modelfull_params_sha256"] = params_sha256(P3)
    idx3 = rng.integers(0, 256, (2, 24)).astype(np.int32)
    logits3, aux3 = m3(idx3)
    G["modelfull_idx"], G["modelfull_logits"], G["modelfull_aux"] = idx3, logits3, np.array(aux3)

    # ---- loss: l2_wrap_loss / l2_wrap_loss_masked (train.py:317-362) ----
    from rwkv_mlx import train as ref_train

    lg = (3 * rng.standard_normal((2, 12, 50))).astype(np.float32)
    tg = rng.integers(0, 50, (2, 12)).astype(np.int32)
    mk = (rng.uniform(0, 1, (2, 12)) < 0.6).astype(np.float32)
    G.update(loss_logits=lg, loss_targets=tg, loss_mask=mk,
             loss_l2wrap=np.array(ref_train.l2_wrap_loss(lg, tg)),
             loss_l2wrap_masked=np.array(ref_train.l2_wrap_loss_masked(lg, tg, mk)))

    # ---- checkpoint conversion: convert_pytorch_to_mlx (convert.py:16-141) on a
    # PyTorch-layout state dict (1-D mixing vectors, no layer-0 v0/v1/v2) ----
    import json
    import tempfile

    import torch

    from rwkv_mlx import convert as ref_convert
    from tests.golden.params import pth_state_dict

    sd = pth_state_dict(spec, seed=6)
    with tempfile.TemporaryDirectory() as td:
        torch.save(sd, f"{td}/m.pth")
        conf = ref_convert.convert_pytorch_to_mlx(f"{td}/m.pth", f"{td}/out", "float16")
        conv = ref_mx_load(f"{td}/out/model.safetensors")
    names = sorted(conv)
    G["conv_names"] = np.array(names)
    G["conv_shapes"] = np.array([list(conv[n].shape) + [-1] * (4 - conv[n].ndim) for n in names], np.int64)
    G["conv_dtypes"] = np.array([str(conv[n].dtype) for n in names])
    G["conv_sha256"] = np.stack([np.frombuffer(hashlib.sha256(np.ascontiguousarray(conv[n]).tobytes()).digest(),
                                               np.uint8) for n in names])
    G["conv_config"] = np.array(json.dumps(conf, sort_keys=True))

    # ---- cases added later use their own generator (earlier draws stay unchanged) ----
    from tests.inputs import router_x

    rng2 = np.random.default_rng(21)
    ffn = m.blocks[1].ffn
    xc = rng2.standard_normal(128).astype(np.float32)
    xcp = rng2.standard_normal(128).astype(np.float32)
    outc, xco = ref_model._channel_mixing_rnn(xc, xcp, ffn)
    G.update(cmix_rnn_x=xc, cmix_rnn_xprev=xcp, cmix_rnn_out=outc)

    r4 = ref_moe.Router(768, 8, 2)
    r4.gate.weight = (rng2.standard_normal((8, 768)) / np.sqrt(768)).astype(np.float32)
    x4 = router_x(4096, 768, seed=22)  # fp16
    G["router4k_x_sha256"] = np.frombuffer(hashlib.sha256(x4.tobytes()).digest(), np.uint8)
    i4, s4, a4, z4 = r4(x4.reshape(1, 4096, 768))
    G.update(router4k_w=r4.gate.weight, router4k_inds=i4, router4k_scores=s4, router4k_aux=np.array(a4),
             router4k_z=np.array(z4))

    out_path = HERE / "reference_golden.npz"
    np.savez_compressed(out_path, **{k: np.asarray(v) for k, v in G.items()})
    print(f"wrote {out_path} ({out_path.stat().st_size / 1e6:.2f} MB, {len(G)} arrays)")


if __name__ == "__main__":
    main()
