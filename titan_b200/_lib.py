"""ctypes binding of libtitan_moe.so (include/titan_moe.h).

The library is the product: there is no CPU or eager fallback.  If the
shared object is missing or was built for another ABI the first call raises
:class:`ExtensionMissing`; a failing entry point raises the typed error that
matches its status code.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtitan_moe.so")
ABI_VERSION = 4


class TmoeError(RuntimeError):
    """Base class for errors reported by the C ABI."""

    code = -1


class InvalidArgument(TmoeError, ValueError):
    code = 1


class Unsupported(TmoeError, NotImplementedError):
    code = 2


class CudaError(TmoeError):
    code = 3


class NcclError(TmoeError):
    code = 4


class DeviceTimeout(TmoeError):
    code = 5


class WorkspaceError(TmoeError):
    code = 6


class ExtensionMissing(RuntimeError):
    """The compiled CUDA library is not present or not loadable."""


_ERRORS = {c.code: c for c in (InvalidArgument, Unsupported, CudaError, NcclError, DeviceTimeout,
                                WorkspaceError)}

P = C.c_void_p
I32 = C.c_int
I64 = C.c_int64
SZ = C.c_size_t


class Layer(C.Structure):
    """struct tmoe_layer."""

    _fields_ = [("hidden", I32), ("num_experts", I32), ("top_k", I32), ("moe_inter", I32),
                ("shared_inter", I32)] + [
        (n, P) for n in (
            "router_w", "gate_up_w", "gate_up_s", "gate_up_b", "down_w", "down_s", "down_b",
            "gate_up_st", "gate_up_bt", "down_st", "down_bt",
            "shared_gate_up_w", "shared_gate_up_s", "shared_gate_up_b",
            "shared_down_w", "shared_down_s", "shared_down_b",
            "shared_gate_up_st", "shared_gate_up_bt", "shared_down_st", "shared_down_bt",
            "shared_gate_w", "gate_up_rs", "down_rs", "shared_gate_up_rs", "shared_down_rs")]


class Options(C.Structure):
    """struct tmoe_options."""

    _fields_ = [("min_tokens", I32), ("down_int8", I32), ("wsum_mode", I32), ("int8_prefill", I32),
                ("gemm_kernel", I32), ("decode_kernel", I32)]


STAGE_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_char_p)

_SIGS = {
    "tmoe_abi_version": ([], I32),
    "tmoe_set_stage_hook": ([STAGE_FN, P], None),
    "tmoe_device_status": ([], I32),
    "tmoe_last_error": ([], C.c_char_p),
    "tmoe_affine_quantize": ([P, I64, I32, P, P, P, P], I32),
    "tmoe_prepare_tables": ([P, P, I32, I32, I32, P, P, P], I32),
    "tmoe_qsum": ([P, I32, I32, I32, P, P], I32),
    "tmoe_quantize_activations": ([P, I32, I32, P, P, P, P], I32),
    "tmoe_router_topk": ([P, P, I32, I32, I32, I32, P, P, P, P, P], I32),
    "tmoe_route_workspace_size": ([I32, I32], SZ),
    "tmoe_route_sort": ([P, I32, I32, P, SZ, P, P, P, P, P, P, I32, P], I32),
    "tmoe_gather_qmm_int8_workspace_size": ([I32, I32, I32, I32], SZ),
    "tmoe_gather_qmm_int8": ([P, P, P, P, P, I32, I32, I32, I32, P, SZ, P, P], I32),
    "tmoe_static_scratch_bytes": ([], SZ),
    "tmoe_gather_qmm_int8_static": ([P, P, P, P, P, I32, I32, I32, I32, P, P], I32),
    "tmoe_gather_qmm_bf16_workspace_size": ([I32, I32, I32, I32], SZ),
    "tmoe_gather_qmm_bf16": ([P, P, P, P, P, P, P, I32, I32, I32, I32, P, SZ, P, P], I32),
    "tmoe_decode_workspace_size": ([I32, I32, I32, I32, I32], SZ),
    "tmoe_gate_up_silu": ([P, P, P, P, P, I32, I32, I32, I32, I32, P, SZ, P, P], I32),
    "tmoe_down_wsum": ([P, P, P, P, P, P, I32, I32, I32, I32, I32, P, SZ, P, P], I32),
    "tmoe_swiglu": ([P, I32, I32, P, P], I32),
    "tmoe_weighted_sum": ([P, P, P, I32, I32, I32, I32, P, P], I32),
    "tmoe_moe_workspace_size": ([C.POINTER(Layer), I32, C.POINTER(Options)], SZ),
    "tmoe_moe_forward": ([C.POINTER(Layer), P, I32, C.POINTER(Options), P, SZ, P, P, P, P], I32),
    "tmoe_moe_experts_workspace_size": ([C.POINTER(Layer), I32, I32, C.POINTER(Options)], SZ),
    "tmoe_moe_experts": ([C.POINTER(Layer), P, I32, P, P, I32, C.POINTER(Options), P, SZ, P, P],
                         I32),
    "tmoe_moe_experts_slots": ([C.POINTER(Layer), P, I32, P, C.POINTER(Options), P, SZ, P, P],
                               I32),
    "tmoe_moe_combine": ([P, P, P, I32, I32, I32, I32, P, P, P, P], I32),
    "tmoe_moe_local_workspace_size": ([C.POINTER(Layer), I32, C.POINTER(Options)], SZ),
    "tmoe_moe_local": ([C.POINTER(Layer), P, I32, C.POINTER(Options), P, SZ, P, P, P, P, P], I32),
    "tmoe_ep_buffer_bytes": ([I32, I32, I32, I32, I32, P], SZ),
    "tmoe_ep_alloc": ([SZ, P], I32),
    "tmoe_ep_free": ([P], I32),
    "tmoe_ipc_handle": ([P, P], I32),
    "tmoe_ipc_open": ([P, P], I32),
    "tmoe_ipc_close": ([P], I32),
    "tmoe_ep_dispatch": ([P, P, I32, I32, I32, I32, I32, I32, P, P, I32, I32, P, P], I32),
    "tmoe_ep_slots": ([P, P, P, I32, I32, I32, I32, I32, P, P, P, P], I32),
    "tmoe_ep_wait": ([P, P, I32, I32, I32, P, P], I32),
    "tmoe_ep_post": ([I32, P, I32, I32, P, P, I32, P], I32),
    "tmoe_prepare_row_scale": ([P, P, I32, I32, I32, P, P], I32),
    "tmoe_rmsnorm": ([P, P, I32, I32, C.c_float, P, P], I32),
    "tmoe_residual_inject": ([P, P, P, I32, I32, I32, P, P], I32),
    "tmoe_moe_sublayer_workspace_size": ([P, I32, P], SZ),
    "tmoe_moe_sublayer": ([P, P, C.c_float, P, I32, P, P, I32, P, P, SZ, P, P], I32),
    "tmoe_ep_post_return": ([P, I32, I32, P, P, I32, P], I32),
    "tmoe_ep_guard": ([P, I32, P, I64, P], I32),
}

EXPORTED = tuple(_SIGS)

_lib = None
_lock = threading.Lock()


def load() -> C.CDLL:
    """Load (once) and type the C ABI.  Raises ExtensionMissing if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ExtensionMissing(
                f"{LIB_PATH} is not built; run `python -m titan_b200.build` (nvcc, sm_100a)")
        try:
            lib = C.CDLL(LIB_PATH)
        except OSError as exc:
            raise ExtensionMissing(f"cannot load {LIB_PATH}: {exc}") from exc
        for name, (args, res) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        v = lib.tmoe_abi_version()
        if v != ABI_VERSION:
            raise ExtensionMissing(f"{LIB_PATH} has ABI {v}, expected {ABI_VERSION}; rebuild it")
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().tmoe_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str = "") -> None:
    if rc == 0:
        return
    cls = _ERRORS.get(rc, TmoeError)
    raise cls(f"{what}: {last_error()}" if what else last_error())


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


_hook_ref = None


def set_stage_hook(fn) -> None:
    """Install fn(name: str) to be called before every kernel launch of the
    library on this thread (None removes it)."""
    global _hook_ref
    if fn is None:
        _hook_ref = None
        load().tmoe_set_stage_hook(STAGE_FN(), None)
        return
    _hook_ref = STAGE_FN(lambda _ctx, name: fn(name.decode()))
    load().tmoe_set_stage_hook(_hook_ref, None)
