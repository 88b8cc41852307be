"""Checkpoint formats (rwkv_mlx/convert.py, train.py:625-640): the converter reproduces
the reference converter's output tensor for tensor (golden vectors made by running
convert_pytorch_to_mlx itself, tests/golden/make_golden.py), and safetensors files
round-trip through the model.  Host-side, no GPU."""

import hashlib
import json

import numpy as np
import torch

from rwkv_mlx_b200 import checkpoint as ck
from rwkv_mlx_b200.model import RWKV, RWKVConfig, init_weights
from tests.golden.golden import golden
from tests.golden.params import pth_state_dict, spec_from_arrays


def _pth():
    G = golden()
    return pth_state_dict(spec_from_arrays(G["model_spec_names"], G["model_spec_shapes"]), seed=6)


def test_convert_matches_reference_converter():
    G = golden()
    sd = _pth()
    conf = ck.infer_config(sd)
    assert conf == json.loads(str(G["conv_config"]))
    out = ck.convert_state_dict(sd, "float16", conf)
    assert sorted(out) == list(G["conv_names"])
    for i, n in enumerate(G["conv_names"]):
        t = out[str(n)]
        shape = [s for s in G["conv_shapes"][i] if s >= 0]
        assert list(t.shape) == shape, n
        assert str(t.dtype).replace("torch.", "") == str(G["conv_dtypes"][i]), n
        digest = hashlib.sha256(np.ascontiguousarray(t.numpy()).tobytes()).digest()
        assert np.array_equal(np.frombuffer(digest, np.uint8), G["conv_sha256"][i]), n


def test_convert_files_then_load_model(tmp_path):
    sd = _pth()
    torch.save(sd, tmp_path / "m.pth")
    conf = ck.convert_pth(tmp_path / "m.pth", tmp_path / "out", "float32")
    m = ck.load_model(tmp_path / "out", device="cpu", dtype=torch.float32)
    assert m.config.n_layer == conf["n_layer"] and m.config.dim_ffn == conf["dim_ffn"]
    params = dict(m.named_parameters())
    for n, t in sd.items():
        assert torch.equal(params[n].detach().reshape(-1), t.float().reshape(-1)), n
    assert float(params["blocks.0.att.v1"].detach().abs().sum()) == 0.0


def test_save_and_load_round_trip(tmp_path):
    cfg = RWKVConfig(n_layer=2, n_embd=128, vocab_size=300, dim_ffn=256, moe_num_experts=4, moe_top_k=2,
                     moe_mode="full", moe_layers=(1,))
    a = RWKV(cfg)
    init_weights(a, seed=3)
    ck.save_safetensors(a, tmp_path)
    conf = json.loads((tmp_path / "config.json").read_text())
    b = ck.load_model(tmp_path, device="cpu", dtype=torch.float32)
    assert conf["moe_mode"] == "full" and b.blocks[1].is_moe and not b.blocks[0].is_moe
    for (na, pa), (nb, pb) in zip(a.named_parameters(), b.named_parameters()):
        assert na == nb and torch.equal(pa.detach(), pb.detach()), na


def test_load_rejects_mismatched_checkpoint(tmp_path):
    a = RWKV(RWKVConfig(n_layer=2, n_embd=128, vocab_size=300, dim_ffn=256))
    ck.save_safetensors(a, tmp_path)
    b = RWKV(RWKVConfig(n_layer=2, n_embd=128, vocab_size=300, dim_ffn=384))
    try:
        ck.load_safetensors(b, tmp_path)
    except ValueError as e:
        assert "ffn.key.weight" in str(e)
    else:
        raise AssertionError("a shape mismatch must raise")
