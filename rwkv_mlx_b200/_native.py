"""ctypes binding of the C-ABI library ``_lib/librwkv_b200.so`` (include/rwkv_b200.h).

The library is the only compute path: if it is missing, or no CUDA device is
present, the public functions raise instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "librwkv_b200.so"

STATUS = {
    0: "ok",
    1: "bad shape",
    2: "unsupported dtype",
    3: "unsupported head size (must be 64)",
    4: "CUDA error",
    5: "misaligned pointer",
    6: "invalid argument",
    7: "workspace too small",
}

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); must match include/rwkv_b200.h
SIGNATURES = {
    "rwkv_last_error": (ctypes.c_char_p, []),
    "rwkv_abi_version": (_I, []),
    "rwkv_device_error": (_I, [_I]),
    "rwkv_set_wkv_impl": (_I, [_I]),
    "rwkv_wkv7_forward": (_I, [_P] * 11 + [_I] * 7 + [_P]),
    "rwkv_wkv7_forward_workspace_size": (_SZ, [_I] * 5),
    "rwkv_wkv7_forward_ws": (_I, [_P] * 11 + [_I] * 7 + [_P, _SZ, _P]),
    "rwkv_set_wkv_segments": (_I, [_I]),
    "rwkv_wkv7_backward_launch_count": (_I, [_I, _I, _I, _I]),
    "rwkv_debug_force_wait_timeout": (_I, [_I]),
    "rwkv_debug_set_device_error": (_I, [_I]),
    "rwkv_wkv7_backward": (_I, [_P] * 17 + [_I] * 7 + [_P]),
    "rwkv_wkv7_backward_workspace_size": (_SZ, [_I] * 4),
    "rwkv_wkv7_backward_ws": (_I, [_P] * 17 + [_I] * 7 + [_P, _SZ, _P]),
    "rwkv_wkv7_step": (_I, [_P] * 8 + [_I] * 6 + [_P]),
    "rwkv_moe_router_workspace_size": (_SZ, [_I, _I]),
    "rwkv_moe_router": (_I, [_P] * 9 + [_SZ] + [_I] * 5 + [_P]),
    "rwkv_moe_router_noalloc_scratch_bytes": (_SZ, []),
    "rwkv_moe_router_noalloc": (_I, [_P] * 8 + [_I] * 5 + [_P]),
    "rwkv_moe_permute_workspace_size": (_SZ, [_I, _I]),
    "rwkv_moe_permute": (_I, [_P] * 5 + [_SZ] + [_I] * 3 + [_P]),
    "rwkv_moe_lora_down": (_I, [_P] * 5 + [_I] * 6 + [_P]),
    "rwkv_moe_lora_combine": (_I, [_P] * 7 + [_I] * 6 + [_P]),
    "rwkv_moe_lora_apply_supported": (_I, [_I] * 5),
    "rwkv_moe_lora_apply": (_I, [_P] * 7 + [_I] * 6 + [_P]),
    "rwkv_moe_set_apply_impl": (_I, [_I]),
    "rwkv_moe_lora_apply_routed_supported": (_I, [_I] * 5),
    "rwkv_moe_lora_apply_routed_workspace_size": (_SZ, [_I] * 3),
    "rwkv_moe_lora_apply_routed": (_I, [_P] * 11 + [_SZ, _P] + [_I] * 6 + [_P]),
    "rwkv_moe_ortho_loss": (_I, [_P] * 2 + [_I] * 4 + [_P]),
    "rwkv_moe_gather_rows": (_I, [_P] * 3 + [_I] * 4 + [_P]),
    "rwkv_moe_lora_up": (_I, [_P] * 5 + [_I] * 5 + [_P]),
    "rwkv_moe_combine_rows": (_I, [_P] * 5 + [_I] * 4 + [_P]),
    "rwkv_moe_expert_mix_rows": (_I, [_P] * 6 + [_I] * 6 + [_P]),
    "rwkv_grouped_gemm": (_I, [_P] * 4 + [_I] * 4 + [ctypes.c_longlong, _I, _I, _P]),
    "rwkv_head_ce_workspace_size": (_SZ, [_I, _I]),
    "rwkv_head_ce_stats": (_I, [_P] * 4 + [_I] * 3 + [_P, _SZ, _I, _P]),
    "rwkv_head_ce_grad": (_I, [_P] * 7 + [ctypes.c_float, _I, _P, ctypes.c_longlong] + [_I] * 5 + [_P]),
    "rwkv_ce_chunk": (_I, [_P, ctypes.c_longlong, _P, _P] + [_I] * 5 + [_P]),
    "rwkv_ce_finalize": (_I, [_P, _P, ctypes.c_float, _P, _I, _P]),
    "rwkv_ce_chunk_grad": (_I, [_P, ctypes.c_longlong] + [_P] * 5 + [ctypes.c_float, _I, _P, ctypes.c_longlong]
                           + [_I] * 4 + [_P]),
    "rwkv_lerp": (_I, [_P] * 3 + [_I, ctypes.c_longlong, _I, _I, _I, _P]),
    "rwkv_lerp_prev": (_I, [_P] * 4 + [_I, ctypes.c_longlong, _I, _I, _I, _P]),
    "rwkv_lerp_prev_state": (_I, [_P] * 5 + [_I, ctypes.c_longlong, _I, _I, _I, _P]),
    "rwkv_tmix_mid": (_I, [_P] * 16 + [ctypes.c_longlong, _I, _I, _I, _P]),
    "rwkv_tmix_post": (_I, [_P] * 9 + [ctypes.c_longlong, _I, _I, ctypes.c_float, _I, _I, _P]),
    "rwkv_relu_sq": (_I, [_P, ctypes.c_longlong, _I, _P]),
    "rwkv_lora_act": (_I, [_P, ctypes.c_longlong, _I, _P]),
    "rwkv_argmax_rows": (_I, [_P, ctypes.c_longlong, ctypes.c_longlong, _I, _P, _I, _P]),
    "rwkv_add_layernorm": (_I, [_P] * 6 + [ctypes.c_longlong, _I, ctypes.c_float, _I, _P]),
}

_lib = None


class RwkvNativeError(RuntimeError):
    pass


class RwkvDeviceError(RwkvNativeError):
    """A kernel gave up a bounded wait (its outputs were filled with NaN)."""


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load the library (no GPU needed to load it)."""
    global _lib
    if _lib is None or path is not None:
        p = Path(path or os.environ.get("RWKV_B200_LIB", LIB_PATH))
        if not p.exists():
            raise RwkvNativeError(
                f"{p} not found: build it with `python -m rwkv_mlx_b200.build` (there is no fallback)"
            )
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is not None:
            return lib
        _lib = lib
    return _lib


def lib() -> ctypes.CDLL:
    if not torch.cuda.is_available():
        raise RwkvNativeError("rwkv_mlx_b200 kernels need a CUDA device (no CPU fallback)")
    return load()


# Kernel launches issued through this binding (per C-ABI entry point: the number of
# kernels that entry point enqueues).  bench.py reads it to report gpu_launches.
KERNELS_PER_CALL = {
    "rwkv_wkv7_forward": 1, "rwkv_wkv7_backward": 1, "rwkv_wkv7_backward_ws": 2, "rwkv_wkv7_step": 1,
    "rwkv_moe_router": 2, "rwkv_moe_router_noalloc": 2, "rwkv_moe_permute": 3, "rwkv_moe_lora_down": 1,
    "rwkv_moe_lora_combine": 1, "rwkv_moe_lora_apply": 1, "rwkv_moe_lora_apply_routed": 3, "rwkv_moe_ortho_loss": 1, "rwkv_moe_gather_rows": 1,
    "rwkv_moe_lora_up": 1, "rwkv_moe_combine_rows": 1, "rwkv_lerp": 1, "rwkv_lerp_prev": 1, "rwkv_lerp_prev_state": 1, "rwkv_tmix_mid": 1,
    "rwkv_tmix_post": 1, "rwkv_relu_sq": 1, "rwkv_lora_act": 1, "rwkv_argmax_rows": 1, "rwkv_add_layernorm": 1, "rwkv_moe_expert_mix_rows": 1,
    "rwkv_ce_chunk": 1, "rwkv_ce_finalize": 1, "rwkv_ce_chunk_grad": 1,
    "rwkv_grouped_gemm": 1, "rwkv_head_ce_stats": 2, "rwkv_head_ce_grad": 1,
}
launch_count = 0


def check(rc: int, what: str, kernels: int | None = None) -> None:
    global launch_count
    if rc == 0:
        launch_count += KERNELS_PER_CALL.get(what, 0) if kernels is None else kernels
    if rc != 0:
        msg = STATUS.get(rc, f"status {rc}")
        if rc == 4:
            msg += ": " + (load().rwkv_last_error() or b"").decode()
        raise RwkvNativeError(f"{what} failed: {msg}")


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(t: torch.Tensor) -> int:
    return dtype_code_of(t.dtype)


def dtype_code_of(dt: torch.dtype) -> int:
    if dt not in DTYPE_CODE:
        raise RwkvNativeError(f"unsupported dtype {dt}")
    return DTYPE_CODE[dt]


def check_device_error(clear: bool = True) -> None:
    """Raise :class:`RwkvDeviceError` if a kernel of this library gave up a bounded wait
    since the last check (reads the device error word: a host synchronisation).  The
    aborting kernel also fills its outputs with NaN, so results never look valid."""
    v = lib().rwkv_device_error(1 if clear else 0)
    if v < 0:
        raise RwkvNativeError("rwkv_device_error failed: " + (load().rwkv_last_error() or b"").decode())
    if v:
        raise RwkvDeviceError(f"a kernel gave up a bounded wait (device error word {v}); its outputs are NaN")
