"""B200-native (sm_100a) WKV-7 recurrence and LoRA-MoE ChannelMix for RWKV-v7.

Drop-in replacements for the hot paths of RWKV-MLX (rwkv_mlx/kernels/wkv7_metal.py,
rwkv_mlx/model.py, rwkv_mlx/moe.py) on hand-written CUDA kernels behind the C ABI
declared in include/rwkv_b200.h.  Submodules: ``wkv7`` (WKV-7 operators),
``moe`` (Router / LoRAMoE_CMix), ``model`` (the RWKV-v7 model shell), ``ep``
(expert-parallel dispatch / combine).
"""

from . import wkv7  # noqa: F401
from ._native import RwkvDeviceError, RwkvNativeError, check_device_error  # noqa: F401
from .wkv7 import wkv7_backward, wkv7_forward, wkv7_recurrent, wkv7_step, wkv7_with_state  # noqa: F401

__all__ = ["wkv7", "wkv7_forward", "wkv7_backward", "wkv7_recurrent", "wkv7_step", "wkv7_with_state",
           "check_device_error", "RwkvDeviceError", "RwkvNativeError"]
