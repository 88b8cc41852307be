"""Load tests/golden/reference_golden.npz (made by make_golden.py from the reference's
own code) and rebuild the model parameters it was generated with."""

import hashlib
from functools import lru_cache
from pathlib import Path

import numpy as np

from tests.golden.params import params_sha256, random_params, spec_from_arrays
from tests.inputs import wkv_inputs

PATH = Path(__file__).resolve().parent / "reference_golden.npz"


@lru_cache(maxsize=1)
def golden():
    return dict(np.load(PATH))


def wkv_c1_inputs():
    """Config-1 inputs, regenerated and checked against the stored hash."""
    G = golden()
    d = wkv_inputs(1, 256, 4, seed=0)
    h = hashlib.sha256()
    for n in "rwkvab":
        h.update(np.ascontiguousarray(d[n], np.float64).tobytes())
    h.update(np.ascontiguousarray(d["dy"], np.float64).tobytes())
    assert np.array_equal(np.frombuffer(h.digest(), np.uint8), G["wkv_c1_input_sha256"]), \
        "regenerated config-1 inputs differ from the ones the fixture was made with"
    return d


def model_params(prefix, seed):
    G = golden()
    P = random_params(spec_from_arrays(G[prefix + "_spec_names"], G[prefix + "_spec_shapes"]), seed)
    assert np.array_equal(params_sha256(P), G[prefix + "_params_sha256"]), "regenerated parameters differ"
    return P


def tiny_config(moe=False, full=False):
    kw = dict(n_layer=2, n_embd=128, vocab_size=256, dim_ffn=256)
    if moe:
        kw.update(moe_num_experts=4, moe_top_k=2, moe_lora_rank=8)
    if full:
        kw.update(moe_num_experts=4, moe_top_k=2, moe_mode="full")
    return kw
