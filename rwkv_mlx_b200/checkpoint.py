"""Checkpoint formats of the reference, for loading real RWKV-7 weights.

Reference (rwkv_mlx):
  * ``convert.py:16-141``  ``convert_pytorch_to_mlx``: a PyTorch RWKV-7 ``.pth`` state
    dict -> flat safetensors + ``config.json``: every tensor squeezed, ``att.w0`` and
    ``ln_x.*`` kept fp32, the rest in the target dtype, 1-D mixing vectors / biases
    reshaped to (1, 1, C), zero ``blocks.0.att.v0 / v1 / v2`` added (layer 0 has no
    value-residual LoRA in PyTorch checkpoints), config inferred from the shapes
                                              -> :func:`infer_config`, :func:`convert_state_dict`,
                                                 :func:`convert_pth`
  * ``convert.py:146-172`` ``load_mlx_weights``     -> :func:`load_safetensors`
  * ``train.py:625-640``   checkpoint save: flat parameter names (``blocks.3.att.w1``
    ...) in one safetensors file and a ``config.json``   -> :func:`save_safetensors`

The flat names and shapes are the reference model's own parameter paths, which this
package's ``RWKV`` module reproduces, so one file serves both.  Host-side code only
(file formats); the tensors land on the model's device.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from .model import RWKV, RWKVConfig

RESHAPE_1D = {"x_r", "x_w", "x_k", "x_v", "x_a", "x_g", "w0", "a0", "v0", "k_k", "k_a"}
_DTYPES = {"float16": torch.float16, "float32": torch.float32, "bfloat16": torch.bfloat16}


def infer_config(sd: dict) -> dict:
    """Model sizes from the shapes of a PyTorch RWKV-7 state dict (convert.py:40-75)."""
    vocab_size, n_embd = sd["emb.weight"].shape
    n_layer = 1 + max(int(k.split(".")[1]) for k in sd if k.startswith("blocks.") and k.endswith(".ln1.weight"))
    head_size = sd["blocks.0.att.r_k"].shape[1] if "blocks.0.att.r_k" in sd else 64
    dim_ffn = sd["blocks.0.ffn.key.weight"].shape[0] if "blocks.0.ffn.key.weight" in sd else 0

    def lora(name):
        return sd[name].shape[1] if name in sd else 0

    return {"n_layer": int(n_layer), "n_embd": int(n_embd), "vocab_size": int(vocab_size),
            "head_size": int(head_size), "dim_ffn": int(dim_ffn),
            "d_decay_lora": int(lora("blocks.0.att.w1")), "d_aaa_lora": int(lora("blocks.0.att.a1")),
            "d_mv_lora": int(lora("blocks.1.att.v1")), "d_gate_lora": int(lora("blocks.0.att.g1"))}


def convert_state_dict(sd: dict, dtype: str = "float16", config: dict | None = None) -> dict:
    """The tensors ``convert_pytorch_to_mlx`` writes (convert.py:80-141), as CPU tensors."""
    target = _DTYPES[dtype]
    config = config or infer_config(sd)
    out = {}
    for name, t in sd.items():
        t = t.detach().squeeze().float().cpu()
        if name.endswith("att.w0") or "ln_x.weight" in name or "ln_x.bias" in name:
            t = t.to(torch.float32)  # decay bias and GroupNorm parameters stay fp32
        else:
            t = t.to(target)
        if name.split(".")[-1] in RESHAPE_1D and t.dim() == 1:
            t = t.reshape(1, 1, -1)
        out[name] = t.contiguous()
    C = config.get("n_embd", 768)
    d_mv = config.get("d_mv_lora", 0) or max(32, int(round((1.7 * C ** 0.5) / 32) * 32))
    if "blocks.0.att.v0" not in out:  # unused by layer 0; present so the module loads
        out["blocks.0.att.v0"] = torch.zeros(1, 1, C)
        out["blocks.0.att.v1"] = torch.zeros(C, d_mv)
        out["blocks.0.att.v2"] = torch.zeros(d_mv, C)
    return out


def config_from_dict(d: dict, **overrides) -> RWKVConfig:
    fields = RWKVConfig.__dataclass_fields__
    kw = {k: v for k, v in d.items() if k in fields}
    kw.update(overrides)
    return RWKVConfig(**kw)


def convert_pth(pth_path, output_dir, dtype: str = "float16") -> dict:
    """``convert_pytorch_to_mlx``: read a ``.pth``, write ``model.safetensors`` and
    ``config.json`` into ``output_dir``; returns the inferred config."""
    from safetensors.torch import save_file

    sd = torch.load(pth_path, map_location="cpu", weights_only=True)
    config = infer_config(sd)
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    save_file(convert_state_dict(sd, dtype, config), str(out / "model.safetensors"))
    (out / "config.json").write_text(json.dumps(config, indent=2))
    return config


def load_safetensors(model: RWKV, weight_dir) -> RWKV:
    """``load_mlx_weights``: copy ``weight_dir/model.safetensors`` into ``model`` by
    parameter name (each tensor cast to the parameter's dtype and device)."""
    from safetensors.torch import load_file

    flat = load_file(str(Path(weight_dir) / "model.safetensors"))
    params = dict(model.named_parameters())
    missing = sorted(set(params) - set(flat))
    unexpected = sorted(set(flat) - set(params))
    if missing or unexpected:
        raise KeyError(f"checkpoint does not match the model: missing {missing[:5]}, unexpected {unexpected[:5]}")
    with torch.no_grad():
        for name, p in params.items():
            t = flat[name]
            if tuple(t.shape) != tuple(p.shape):
                raise ValueError(f"{name}: checkpoint shape {tuple(t.shape)} != parameter shape {tuple(p.shape)}")
            p.copy_(t.to(device=p.device, dtype=p.dtype))
    return model


def load_model(weight_dir, device="cuda", dtype=torch.float16, **overrides) -> RWKV:
    """Build an ``RWKV`` from ``weight_dir/config.json`` and load its safetensors; the
    parameters take ``dtype`` except ``w0`` (fp32), as the reference keeps it."""
    from .model import cast_for_inference

    d = json.loads((Path(weight_dir) / "config.json").read_text())
    model = RWKV(config_from_dict(d, **overrides))
    model = cast_for_inference(model, dtype).to(device)
    return load_safetensors(model, weight_dir)


def save_safetensors(model: RWKV, output_dir, name: str = "model.safetensors") -> Path:
    """Checkpoint in the reference's layout (train.py:625-640): every parameter under
    its flat name in one safetensors file, plus ``config.json`` with the model sizes."""
    from safetensors.torch import save_file

    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    flat = {n: p.detach().contiguous().cpu() for n, p in model.named_parameters()}
    save_file(flat, str(out / name))
    c = model.config
    conf = {"n_layer": c.n_layer, "n_embd": c.n_embd, "vocab_size": c.vocab_size, "head_size": c.head_size,
            "ctx_len": c.ctx_len, "dim_ffn": c.dim_ffn, "d_decay_lora": c.lora_dim("decay"),
            "d_aaa_lora": c.lora_dim("aaa"), "d_mv_lora": c.lora_dim("mv"), "d_gate_lora": c.lora_dim("gate")}
    if c.moe_num_experts:
        conf.update(moe_num_experts=c.moe_num_experts, moe_top_k=c.moe_top_k, moe_mode=c.moe_mode,
                    moe_lora_rank=c.moe_lora_rank, moe_layers=list(c.moe_layers))
    (out / "config.json").write_text(json.dumps(conf, indent=2))
    return out / name
