"""titan_b200 — a B200-native (sm_100a) quantised mixture-of-experts block.

The hot path of Titan's MoE layer: router softmax + top-k, the int8-activation
x int4-affine-weight expert gather for gate_up, SwiGLU, the int4 down
projection, and the unsort + weighted top-k sum plus the sigmoid-gated shared
expert.  Host code is Python/PyTorch; the compute is hand-written CUDA for
sm_100a behind the C ABI of include/titan_moe.h (libtitan_moe.so).

    from titan_b200 import SparseMoeBlock, ops, patch
    patch.install()                      # int8 prefill overlay
    y = block(x)                         # one C-ABI call per layer
"""
from . import ops, patch
from ._lib import (CudaError, DeviceTimeout, ExtensionMissing, InvalidArgument, NcclError,
                   TmoeError, Unsupported, WorkspaceError)
from .moe_block import SharedExpert, SparseMoeBlock
from .switch_layers import QuantizedSwitchLinear, SwiGLU, SwitchGLU

__all__ = ["ops", "patch", "SparseMoeBlock", "SharedExpert", "SwitchGLU", "SwiGLU",
           "QuantizedSwitchLinear", "TmoeError", "InvalidArgument", "Unsupported", "CudaError",
           "NcclError", "DeviceTimeout", "WorkspaceError", "ExtensionMissing"]
