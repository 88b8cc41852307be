"""The C-ABI library loads, exports every entry point of include/rwkv_b200.h, and
rejects bad arguments before touching the GPU (CPU-only checks)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "rwkv_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(rwkv_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from rwkv_mlx_b200 import _native

    return _native.load()


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ["rwkv_wkv7_forward", "rwkv_wkv7_backward", "rwkv_wkv7_step", "rwkv_moe_router",
              "rwkv_moe_permute", "rwkv_moe_lora_down", "rwkv_moe_lora_combine", "rwkv_moe_ortho_loss"]:
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    from rwkv_mlx_b200 import _native

    assert set(declared_functions()) <= set(_native.SIGNATURES)


def test_abi_version(lib):
    assert lib.rwkv_abi_version() >= 1


def test_argument_validation_without_gpu(lib):
    P = None
    # head size != 64 is rejected first (RWKV_ERR_HEAD_SIZE = 3)
    assert lib.rwkv_wkv7_forward(*([P] * 11), 1, 16, 1, 32, 1, 1, 16, P) == 3
    # bad dtype (RWKV_ERR_DTYPE = 2)
    assert lib.rwkv_wkv7_forward(*([P] * 11), 1, 16, 1, 64, 9, 9, 16, P) == 2
    # empty shape (RWKV_ERR_SHAPE = 1)
    assert lib.rwkv_wkv7_forward(*([P] * 11), 0, 16, 1, 64, 1, 1, 16, P) == 1
    # NULL inputs (RWKV_ERR_ARG = 6)
    assert lib.rwkv_wkv7_forward(*([P] * 11), 1, 16, 1, 64, 1, 1, 16, P) == 6
    assert lib.rwkv_wkv7_step(*([P] * 8), 1, 1, 64, 1, 1, 0, P) == 6
    assert lib.rwkv_moe_router(*([P] * 9), 0, 16, 768, 40, 2, 1, P) == 1  # E > 32
    assert lib.rwkv_moe_permute(*([P] * 5), 0, 0, 2, 8, P) == 1


def test_workspace_queries(lib):
    assert lib.rwkv_moe_router_workspace_size(65536, 8) > 0
    assert lib.rwkv_moe_permute_workspace_size(131072, 8) >= 2 * 64 * 8 * 4
    assert lib.rwkv_moe_router_workspace_size(0, 8) == 0
    assert lib.rwkv_wkv7_backward_launch_count(1, 16, 1, 32) == 0  # head size 32: invalid sizes


def test_python_api_refuses_cpu_tensors():
    import torch

    from rwkv_mlx_b200 import _native, wkv7

    x = torch.zeros(1, 16, 64)
    with pytest.raises(_native.RwkvNativeError):
        wkv7.wkv7(x, x, x, x, x, x)
