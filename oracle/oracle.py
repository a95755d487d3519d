"""TEST INFRASTRUCTURE ONLY: Python binding of the CPU oracle (moe_oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg (and its
``--impl reference`` arm) may import this module, and only as the checker or
the timed CPU baseline.  Nothing in titan_b200/ imports it.

Parity status: unpinned at the value level against MLX (see the header of
moe_oracle.c for what the reference's own tests pin and how).

bf16 tensors are carried as numpy uint16 bit patterns; packed int4 weights as
uint32 [rows, K/8] with element 8w+j in bits 4j..4j+3 (low nibble first).
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field

import numpy as np

from . import build as _build

_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        path = _build.build()
        L = C.CDLL(path)
        P = C.c_void_p
        i32, i64 = C.c_int, C.c_int64
        sig = {
            "orc_threads": ([], i32),
            "orc_set_threads": ([i32], None),
            "orc_exp": ([C.c_float], C.c_float),
            "orc_sigmoid": ([C.c_float], C.c_float),
            "orc_f32_to_bf16": ([P, P, i64], None),
            "orc_router": ([P, P, i32, i32, i32, i32, P, P, P, P], None),
            "orc_sort_routes": ([P, i32, i32, P, P, P], None),
            "orc_quantize_act": ([P, i32, i32, P, P, P, P], None),
            "orc_qsum": ([P, i32, i32, i32, P], None),
            "orc_prepare_tables": ([P, P, i32, i32, i32, P, P], None),
            "orc_affine_quantize": ([P, i64, i32, P, P, P], None),
            "orc_dequant": ([P, P, P, i64, i32, P], None),
            "orc_gather_qmm_int8": ([P, P, P, P, P, i32, i32, i32, i32, P], None),
            "orc_gather_qmm_exact": ([P, P, P, P, P, i32, i32, i32, P, P], None),
            "orc_swiglu": ([P, i32, i32, P], None),
            "orc_weighted_sum": ([P, P, P, i32, i32, i32, i32, P], None),
            "orc_moe_prefill": ([P, P, i32, P, P, P], None),
            "orc_set_parts_out": ([P, P, P], None),
            "orc_moe_decode": ([P, P, P, P, P], None),
            "orc_rmsnorm": ([P, P, i32, i32, C.c_float, P], None),
            "orc_inject": ([P, P, P, i32, i32, i32, P], None),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _LIB = L
    return _LIB


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


# --------------------------------------------------------------- bf16 helpers

def f32_to_bf16(a) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit pattern (uint16)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    r = np.where(nan, (u >> 16) | 0x40, r)
    return r.astype(np.uint16)


def bf16_to_f32(h) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    return (h.astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------ thin wrappers

def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def threads() -> int:
    return int(lib().orc_threads())


def exp(x: float) -> float:
    return float(lib().orc_exp(float(x)))


def router(x, wr, k):
    T, H = x.shape
    E = wr.shape[0]
    idx = np.zeros((T, k), np.int32)
    sc = np.zeros((T, k), np.uint16)
    lg = np.zeros((T, E), np.uint16)
    pb = np.zeros((T, E), np.uint16)
    lib().orc_router(_p(x), _p(wr), T, H, E, k, _p(idx), _p(sc), _p(lg), _p(pb))
    return idx, sc, lg, pb


def sort_routes(idx_flat, E):
    R = idx_flat.size
    idx_flat = np.ascontiguousarray(idx_flat.reshape(-1), dtype=np.int32)
    order = np.zeros(R, np.int32)
    inv = np.zeros(R, np.int32)
    off = np.zeros(E + 1, np.int32)
    lib().orc_sort_routes(_p(idx_flat), R, E, _p(order), _p(inv), _p(off))
    return order, inv, off


def quantize_act(x):
    R, K = x.shape
    G = K // 64
    xs = np.zeros((R, K), np.int8)
    xsc = np.zeros((R, G), np.float32)
    xrs = np.zeros((R, G), np.float32)
    xav = np.zeros((R, G), np.float32)
    lib().orc_quantize_act(_p(x), R, K, _p(xs), _p(xsc), _p(xrs), _p(xav))
    return xs, xsc, xrs, xav


def qsum(wq):
    E, N, KW = wq.shape
    K = KW * 8
    out = np.zeros((E, K // 64, N), np.uint16)
    lib().orc_qsum(_p(wq), E, N, K, _p(out))
    return out


def prepare_tables(scales, biases):
    E, N, G = scales.shape
    st = np.zeros((E, G, N), np.uint16)
    bt = np.zeros((E, G, N), np.uint16)
    lib().orc_prepare_tables(_p(scales), _p(biases), E, N, G, _p(st), _p(bt))
    return st, bt


def affine_quantize(w):
    """MLX-style affine int4 g64 quantiser on an fp32 array [..., K]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    *lead, K = w.shape
    rows = int(np.prod(lead)) if lead else 1
    wq = np.zeros((rows, K // 8), np.uint32)
    s = np.zeros((rows, K // 64), np.uint16)
    b = np.zeros((rows, K // 64), np.uint16)
    lib().orc_affine_quantize(_p(w), rows, K, _p(wq), _p(s), _p(b))
    return (wq.reshape(*lead, K // 8), s.reshape(*lead, K // 64), b.reshape(*lead, K // 64))


def dequant(wq, scales, biases):
    *lead, KW = wq.shape
    K = KW * 8
    rows = int(np.prod(lead))
    out = np.zeros((rows, K), np.float32)
    lib().orc_dequant(_p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(scales)),
                      _p(np.ascontiguousarray(biases)), rows, K, _p(out))
    return out.reshape(*lead, K)


def gather_qmm_int8(x, wq, scales, biases, rhs, order=0):
    R, K = x.shape
    E, N, _ = wq.shape
    y = np.zeros((R, N), np.uint16)
    lib().orc_gather_qmm_int8(_p(x), _p(wq), _p(scales), _p(biases),
                              _p(np.ascontiguousarray(rhs, dtype=np.int32)), R, N, K, order, _p(y))
    return y


def gather_qmm_exact(x, wq, scales, biases, rhs=None, f32=False):
    R, K = x.shape
    N = wq.shape[-2]
    rhs_c = None if rhs is None else np.ascontiguousarray(rhs, dtype=np.int32)
    if f32:
        y = np.zeros((R, N), np.float32)
        lib().orc_gather_qmm_exact(_p(x), _p(wq), _p(scales), _p(biases), _p(rhs_c), R, N, K,
                                   None, _p(y))
    else:
        y = np.zeros((R, N), np.uint16)
        lib().orc_gather_qmm_exact(_p(x), _p(wq), _p(scales), _p(biases), _p(rhs_c), R, N, K,
                                   _p(y), None)
    return y


def swiglu(gu):
    R, I2 = gu.shape
    h = np.zeros((R, I2 // 2), np.uint16)
    lib().orc_swiglu(_p(gu), R, I2 // 2, _p(h))
    return h


def weighted_sum(ys, inv, scores, mode=0):
    T, k = scores.shape
    D = ys.shape[-1]
    out = np.zeros((T, D), np.uint16)
    inv_c = None if inv is None else np.ascontiguousarray(inv, dtype=np.int32)
    lib().orc_weighted_sum(_p(ys), _p(inv_c), _p(scores), T, k, D, mode, _p(out))
    return out


# --------------------------------------------------------- whole-block oracle

class _Desc(C.Structure):
    _fields_ = [("T", C.c_int), ("H", C.c_int), ("E", C.c_int), ("k", C.c_int),
                ("I", C.c_int), ("Is", C.c_int)] + [
        (n, C.c_void_p) for n in ("wr", "gu_w", "gu_s", "gu_b", "dn_w", "dn_s", "dn_b",
                                  "sgu_w", "sgu_s", "sgu_b", "sdn_w", "sdn_s", "sdn_b", "wg")]


@dataclass
class Layer:
    """One MoE layer's weights in MLX layout (numpy, bf16 as uint16)."""
    H: int
    E: int
    k: int
    I: int
    Is: int
    wr: np.ndarray                    # [E, H] bf16
    gu_w: np.ndarray                  # [E, 2I, H/8] u32 (gate rows first)
    gu_s: np.ndarray                  # [E, 2I, H/64] bf16
    gu_b: np.ndarray
    dn_w: np.ndarray                  # [E, H, I/8] u32
    dn_s: np.ndarray                  # [E, H, I/64] bf16
    dn_b: np.ndarray
    sgu_w: np.ndarray | None = None   # [1, 2Is, H/8]
    sgu_s: np.ndarray | None = None
    sgu_b: np.ndarray | None = None
    sdn_w: np.ndarray | None = None   # [1, H, Is/8]
    sdn_s: np.ndarray | None = None
    sdn_b: np.ndarray | None = None
    wg: np.ndarray | None = None      # [H] bf16
    _keep: list = field(default_factory=list, repr=False)

    def desc(self, T: int) -> _Desc:
        d = _Desc()
        d.T, d.H, d.E, d.k, d.I = T, self.H, self.E, self.k, self.I
        d.Is = self.Is if self.sgu_w is not None else 0
        for n in ("wr", "gu_w", "gu_s", "gu_b", "dn_w", "dn_s", "dn_b",
                  "sgu_w", "sgu_s", "sgu_b", "sdn_w", "sdn_s", "sdn_b", "wg"):
            a = getattr(self, n)
            setattr(d, n, None if a is None else a.ctypes.data)
        return d


def make_layer(H, E, k, I, Is=0, seed=0, w_std=0.02, router_std=0.02) -> Layer:
    """Seeded synthetic layer with the benchmark workloads' distributions: router bf16
    N(0, router_std); expert weights fp32 N(0, w_std) quantised affine int4 g64
    with bf16 scales/biases; shared expert the same; shared gate bf16 N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    wr = f32_to_bf16(rng.standard_normal((E, H), dtype=np.float32) * router_std)

    def qlin(rows, K):
        w = rng.standard_normal((rows, K), dtype=np.float32) * w_std
        return affine_quantize(w)

    gw, gs, gb = [], [], []
    dw, ds, db = [], [], []
    for _ in range(E):
        a = qlin(2 * I, H)
        gw.append(a[0]); gs.append(a[1]); gb.append(a[2])
        b = qlin(H, I)
        dw.append(b[0]); ds.append(b[1]); db.append(b[2])
    L = Layer(H, E, k, I, Is, wr, np.stack(gw), np.stack(gs), np.stack(gb),
              np.stack(dw), np.stack(ds), np.stack(db))
    if Is:
        a = qlin(2 * Is, H)
        b = qlin(H, Is)
        L.sgu_w, L.sgu_s, L.sgu_b = a[0][None], a[1][None], a[2][None]
        L.sdn_w, L.sdn_s, L.sdn_b = b[0][None], b[1][None], b[2][None]
        L.wg = f32_to_bf16(rng.standard_normal((H,), dtype=np.float32) * 0.02)
    return L


def make_x(T, H, seed=0, scale=1.0):
    rng = np.random.default_rng(seed + 1_000_003)
    return f32_to_bf16(rng.standard_normal((T, H), dtype=np.float32) * scale)


def moe_prefill(layer: Layer, x, int8_mode=3, parts=False):
    """int8_mode: 0 stock bf16, 1 int8 gate_up only, 3 int8 gate_up and down
    (+4: re-centred FMA order).  parts=True also returns the rounding
    operands of the output: (routed, shared_term, term_max) — the routed sum
    and the gated shared term of the final bf16 add, and the largest bf16
    product score_j * Y_j of each output's weighted sum."""
    T = x.shape[0]
    d = layer.desc(T)
    y = np.zeros((T, layer.H), np.uint16)
    idx = np.zeros((T, layer.k), np.int32)
    sc = np.zeros((T, layer.k), np.uint16)
    routed = np.zeros((T, layer.H), np.uint16) if parts else None
    shared = np.zeros((T, layer.H), np.uint16) if parts else None
    tmax = np.zeros((T, layer.H), np.uint16) if parts else None
    lib().orc_set_parts_out(_p(routed), _p(shared), _p(tmax))
    try:
        lib().orc_moe_prefill(C.byref(d), _p(np.ascontiguousarray(x)), int(int8_mode),
                              _p(idx), _p(sc), _p(y))
    finally:
        lib().orc_set_parts_out(None, None, None)
    if parts:
        return y, idx, sc, (routed, shared, tmax)
    return y, idx, sc


def moe_decode(layer: Layer, x):
    T = x.shape[0]
    d = layer.desc(T)
    y = np.zeros((T, layer.H), np.uint16)
    idx = np.zeros((T, layer.k), np.int32)
    sc = np.zeros((T, layer.k), np.uint16)
    lib().orc_moe_decode(C.byref(d), _p(np.ascontiguousarray(x)), _p(idx), _p(sc), _p(y))
    return y, idx, sc


def rmsnorm(x, w, eps=1e-6):
    """RMSNorm of bf16 rows x [T, H] with weight w [H] (canonical order)."""
    T, H = x.shape
    out = np.zeros((T, H), np.uint16)
    lib().orc_rmsnorm(_p(np.ascontiguousarray(x)), _p(np.ascontiguousarray(w)), T, H,
                      float(eps), _p(out))
    return out


def inject(branch, residual, weights=None):
    """Residual write-back: n = 0 (weights None) bf16(branch + residual) [T, H];
    else the hyper-connection inject into residual [T, n, H] with weights [T, n]."""
    T, H = branch.shape
    n = 0 if weights is None else weights.shape[1]
    out = np.zeros(residual.shape, np.uint16)
    lib().orc_inject(_p(np.ascontiguousarray(branch)), _p(np.ascontiguousarray(residual)),
                     _p(None if weights is None else np.ascontiguousarray(weights)), T, H, n,
                     _p(out))
    return out
