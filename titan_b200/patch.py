"""Runtime overlay: route the sorted routed-expert prefill gathers through the
int8 x int4 grouped GEMM.  Mirrors engine/patches/moe-int8/patch.py:

  * ``ops.gather_qmm`` (the stock op, as ``mx.gather_qmm`` there) is wrapped;
    the previous implementation is captured and keeps every call this kernel
    does not claim;
  * ``SwitchGLU.forward`` is wrapped only to record the token count of the call
    in progress, so the ``min_tokens`` floor is expressed in tokens;
  * a claimed call that fails raises (there is no silent fallback for shapes
    the kernel claims).

Configuration follows the reference's environment names, overridable by
keyword: OMLX_MOE_INT8_PREFILL (enable), OMLX_MOE_INT8_MIN_TOKENS (512),
OMLX_MOE_INT8_MIN_ROWS (4096), OMLX_MOE_INT8_SKIP_DOWN (gate_up only).
Memory: each routed weight tensor gets transposed [E, G, N] scale and bias
tables, two arrays the size of its scales (``warmup``/``clear_cache``).
"""
from __future__ import annotations

import logging
import os

from . import _lib, ops

logger = logging.getLogger(__name__)

_original_gather_qmm = None
_original_switchglu_forward = None
_ctx = {"tokens": None}
_stats = {"routed": 0, "fallback": 0}
_cfg = {"enabled": None, "min_tokens": None, "min_rows": None, "skip_down": None}


def _env_flag(name: str, default: str) -> bool:
    return os.environ.get(name, default) == "1"


def _enabled() -> bool:
    v = _cfg["enabled"]
    return _env_flag("OMLX_MOE_INT8_PREFILL", "0") if v is None else bool(v)


def _min_tokens() -> int:
    v = _cfg["min_tokens"]
    return int(os.environ.get("OMLX_MOE_INT8_MIN_TOKENS", "512")) if v is None else int(v)


def _min_rows() -> int:
    v = _cfg["min_rows"]
    return int(os.environ.get("OMLX_MOE_INT8_MIN_ROWS", "4096")) if v is None else int(v)


def _skip_down() -> bool:
    v = _cfg["skip_down"]
    return _env_flag("OMLX_MOE_INT8_SKIP_DOWN", "0") if v is None else bool(v)


def _arg(args, kwargs, pos, name, default=None):
    if len(args) > pos:
        return args[pos]
    return kwargs.get(name, default)


def _should_route(x, w, args, kwargs) -> bool:
    """engine/patches/moe-int8/patch.py:78-102."""
    if not _enabled() or not kwargs.get("sorted_indices"):
        return False
    scales = _arg(args, kwargs, 0, "scales")
    biases = _arg(args, kwargs, 1, "biases")
    lhs = _arg(args, kwargs, 2, "lhs_indices")
    rhs = _arg(args, kwargs, 3, "rhs_indices")
    transpose = _arg(args, kwargs, 4, "transpose", True)
    group_size = _arg(args, kwargs, 5, "group_size", 64)
    bits = _arg(args, kwargs, 6, "bits", 4)
    mode = _arg(args, kwargs, 7, "mode", "affine")
    if lhs is not None or mode != "affine":
        return False
    if _skip_down() and x.shape[-1] <= 1024:
        return False
    tokens = _ctx.get("tokens")
    if tokens is not None:
        if tokens < _min_tokens():
            return False
    elif x.dim() < 1 or x.shape[0] < _min_rows():
        return False
    return ops.supported_int8(x, w, scales, biases, rhs, transpose, group_size, bits)


def _gather_qmm(x, w, *args, **kwargs):
    if _should_route(x, w, args, kwargs):
        scales = _arg(args, kwargs, 0, "scales")
        biases = _arg(args, kwargs, 1, "biases")
        out = ops.gather_qmm_int8(x, w, scales, biases, _arg(args, kwargs, 3, "rhs_indices"),
                                  ops.cached_tables(w, scales, biases),
                                  group_size=_arg(args, kwargs, 5, "group_size", 64),
                                  bits=_arg(args, kwargs, 6, "bits", 4))
        _stats["routed"] += 1
        return out
    _stats["fallback"] += 1
    return _original_gather_qmm(x, w, *args, **kwargs)


_gather_qmm._titan_moe_int8 = True


def _switchglu_forward(self, x, indices, *a, **kw):
    prev = _ctx.get("tokens")
    try:
        _ctx["tokens"] = int(indices.numel() // indices.shape[-1]) if indices.dim() else None
    except Exception:  # noqa: BLE001 - token count is advisory
        _ctx["tokens"] = None
    try:
        return _original_switchglu_forward(self, x, indices, *a, **kw)
    finally:
        _ctx["tokens"] = prev


def install(*, enabled: bool | None = True, min_tokens: int | None = None,
            min_rows: int | None = None, skip_down: bool | None = None) -> bool:
    """Idempotent.  Returns True when this call installed the hooks.
    Keyword values override the OMLX_MOE_INT8_* environment variables."""
    global _original_gather_qmm, _original_switchglu_forward
    given = dict(enabled=enabled, min_tokens=min_tokens, min_rows=min_rows, skip_down=skip_down)
    _cfg.update({k: v for k, v in given.items() if v is not None})
    if getattr(ops.gather_qmm, "_titan_moe_int8", False):
        return False
    _original_gather_qmm = ops.gather_qmm
    ops.gather_qmm = _gather_qmm
    from .switch_layers import SwitchGLU
    if not getattr(SwitchGLU, "_titan_moe_int8", False):
        _original_switchglu_forward = SwitchGLU.forward
        SwitchGLU.forward = _switchglu_forward
        SwitchGLU._titan_moe_int8 = True
    logger.info("titan_b200 int8 prefill overlay installed (enabled=%s)", _enabled())
    return True


def uninstall() -> None:
    global _original_gather_qmm, _original_switchglu_forward
    if _original_gather_qmm is not None:
        ops.gather_qmm = _original_gather_qmm
        _original_gather_qmm = None
    if _original_switchglu_forward is not None:
        from .switch_layers import SwitchGLU
        SwitchGLU.forward = _original_switchglu_forward
        SwitchGLU._titan_moe_int8 = False
        _original_switchglu_forward = None
    _cfg.update(enabled=None, min_tokens=None, min_rows=None, skip_down=None)


def installed() -> bool:
    return bool(getattr(ops.gather_qmm, "_titan_moe_int8", False))


def clear_cache() -> None:
    ops.clear_tables()


def stats() -> dict:
    return dict(_stats)


def reset_stats() -> None:
    _stats.update(routed=0, fallback=0)


def warmup(model) -> int:
    """Pre-build the tables of every routed projection the overlay would take
    (patch.py:179-198).  Returns the number of tensors prepared."""
    from .switch_layers import QuantizedSwitchLinear
    n = total = 0
    for _, m in model.named_modules():
        if not isinstance(m, QuantizedSwitchLinear):
            continue
        if m.scales.shape[1] % 128:
            continue
        if _skip_down() and m.input_dims <= 1024:
            continue
        total += ops.cached_tables(m.weight, m.scales, m.biases).nbytes
        n += 1
    logger.info("titan_b200 int8 prefill: %d expert tensors prepared, %.2f GB of tables", n,
                total / 1e9)
    return n


def block_options() -> _lib.Options:
    """Options of the fused block forward matching the current overlay state:
    installed and enabled -> int8 gate_up at T >= min_tokens (int8 down unless
    skip_down); otherwise the stock bf16 grouped GEMMs above min_tokens."""
    o = _lib.Options()
    on = installed() and _enabled()
    o.min_tokens = _min_tokens()
    o.int8_prefill = 1 if on else 0
    o.down_int8 = 0 if (not on or _skip_down()) else 1
    o.wsum_mode = 0
    return o
