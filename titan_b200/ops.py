"""Operator surface of the quantised MoE block on torch CUDA tensors.

Each function mirrors a reference operator and calls the C ABI of
libtitan_moe.so; torch provides device memory and the current stream only.

  gather_qmm            mx.gather_qmm (stock: bf16 activations, exact int4
                        dequant, fp32 accumulate) — the op that
                        ``titan_b200.patch.install()`` swaps
  gather_qmm_int8       engine/patches/moe-int8/kernel.py:482-501 and
                        titan/kernels/moe_gather_int8.py:393-425
  quantize              mx.quantize(w, 64, 4, "affine")
  build_tables          titan/kernels/moe_gather_int8.py:227-248
  quantize_activations  titan/kernels/moe_gather_int8.py:168-182
  router_topk           qwen3_5_moe/language.py:65-71 (canonical router)
  route_sort            switch_layers.py:13-25 + moe_gather_ws.py:176-202
  weighted_sum          titan/kernels/moe_weighted_sum.py:142-195
  gate_up_silu/down_wsum  engine/patches/decode-fusion/fused_kernels.py:194-229

Packed int4 weights are int32 (or uint32) tensors [E, N, K/8] holding MLX's
uint32 words; bf16 tensors are torch.bfloat16.
"""
from __future__ import annotations

import math
import weakref
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import InvalidArgument, Unsupported

GROUP = 64
BITS = 4

__all__ = ["GROUP", "BITS", "Int8Tables", "gather_qmm", "gather_qmm_int8", "quantize",
           "build_tables", "prepare_tables", "qsum", "quantize_activations", "router_topk",
           "route_sort", "weighted_sum", "swiglu", "gate_up_silu", "down_wsum", "workspace",
           "stream_ptr"]


# ------------------------------------------------------------------ plumbing

def _p(t):
    return None if t is None else t.data_ptr()


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_WS: dict = {}


def workspace(nbytes: int, device, tag: str = "") -> torch.Tensor:
    """A grow-only device byte buffer per (device, stream, tag).  The C ABI
    never allocates; the host owns this memory.  Calls on one stream are
    ordered, so reusing the buffer across calls is safe.  New buffers start
    zero-filled: tmoe_moe_forward keeps self-resetting counters at the head of
    its workspace."""
    device = torch.device(device)
    key = (device.index, torch.cuda.current_stream(device).cuda_stream, tag)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def clear_workspaces() -> None:
    _WS.clear()


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise InvalidArgument("titan_b200 ops take CUDA tensors (there is no CPU path)")


def _as_words(w: torch.Tensor) -> torch.Tensor:
    if w.dtype not in (torch.int32, torch.uint32):
        raise InvalidArgument(f"packed weights must be int32/uint32, got {w.dtype}")
    return w.contiguous()


def _bf16(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        raise InvalidArgument(f"{name} must be bfloat16, got {t.dtype}")
    return t.contiguous()


def _check_quant(transpose, group_size, bits, mode):
    if not transpose or group_size != GROUP or bits != BITS or mode != "affine":
        raise Unsupported(
            f"titan_b200 implements affine 4-bit group-64 transposed gathers only "
            f"(transpose={transpose}, group_size={group_size}, bits={bits}, mode={mode})")


# ------------------------------------------------------------- weight prep

def quantize(w: torch.Tensor, group_size: int = GROUP, bits: int = BITS, mode: str = "affine"):
    """mx.quantize on the GPU: fp32 [..., K] -> (int32 words [..., K/8],
    bf16 scales [..., K/64], bf16 biases [..., K/64])."""
    _check_quant(True, group_size, bits, mode)
    _need_cuda(w)
    w = w.float().contiguous()
    *lead, K = w.shape
    rows = math.prod(lead) if lead else 1
    wq = torch.empty(*lead, K // 8, dtype=torch.int32, device=w.device)
    s = torch.empty(*lead, K // GROUP, dtype=torch.bfloat16, device=w.device)
    b = torch.empty_like(s)
    _lib.call("tmoe_affine_quantize", _p(w), rows, K, _p(wq), _p(s), _p(b), stream_ptr(w.device))
    return wq, s, b


def prepare_tables(scales: torch.Tensor, biases: torch.Tensor):
    """[E, N, G] -> transposed [E, G, N] scale and bias tables."""
    scales = _bf16(scales, "scales")
    biases = _bf16(biases, "biases")
    squeeze = scales.dim() == 2
    if squeeze:
        scales, biases = scales[None], biases[None]
    E, N, G = scales.shape
    st = torch.empty(E, G, N, dtype=torch.bfloat16, device=scales.device)
    bt = torch.empty_like(st)
    _lib.call("tmoe_prepare_tables", _p(scales), _p(biases), E, N, G * GROUP, _p(st), _p(bt),
              stream_ptr(scales.device))
    return (st[0], bt[0]) if squeeze else (st, bt)


def qsum(w: torch.Tensor) -> torch.Tensor:
    """Reference nibble sums [E, G, N] uint16 (as int16 bits -> returned int32)."""
    w = _as_words(w)
    E, N, KW = w.shape
    out = torch.empty(E, KW * 8 // GROUP, N, dtype=torch.int16, device=w.device)
    _lib.call("tmoe_qsum", _p(w), E, N, KW * 8, _p(out), stream_ptr(w.device))
    return out.to(torch.int32) & 0xFFFF


@dataclass(frozen=True)
class Int8Tables:
    """Per-weight-tensor tables of the int8 path, owned by the caller
    (titan/kernels/moe_gather_int8.py:205-224).  The B200 kernel re-centres
    the nibbles in registers, so no qsum table is needed."""

    scales_t: torch.Tensor   # [E, G, N] bf16
    biases_t: torch.Tensor   # [E, G, N] bf16 (raw biases; b + 8s is folded in-kernel)
    row_scale: torch.Tensor  # [E, N] fp32 power-of-two row normalisers (swap-AB GEMM)

    @property
    def nbytes(self) -> int:
        return self.scales_t.numel() * 2 + self.biases_t.numel() * 2 + self.row_scale.numel() * 4


def row_scale(scales: torch.Tensor, biases: torch.Tensor) -> torch.Tensor:
    """[E, N, G] scales / biases -> [E, N] fp32 row normalisers 2^Ew of the
    swap-AB grouped GEMM (tmoe_prepare_row_scale)."""
    scales = _bf16(scales, "scales")
    biases = _bf16(biases, "biases")
    squeeze = scales.dim() == 2
    if squeeze:
        scales, biases = scales[None], biases[None]
    E, N, G = scales.shape
    rs = torch.empty(E, N, dtype=torch.float32, device=scales.device)
    _lib.call("tmoe_prepare_row_scale", _p(scales), _p(biases), E, N, G * GROUP, _p(rs),
              stream_ptr(scales.device))
    return rs[0] if squeeze else rs


def build_tables(wq, scales, biases) -> Int8Tables:
    st, bt = prepare_tables(scales, biases)
    return Int8Tables(st, bt, row_scale(scales, biases))


_TABLES: dict = {}


def cached_tables(wq, scales, biases) -> Int8Tables:
    """Tables memoised per weight tensor (engine/patches/moe-int8/kernel.py:
    449-459 keys its cache on the weight's identity the same way).  A Python
    id is reused once its object is freed, so each entry also holds weak
    references to the weight and scale tensors it was built from and is
    rebuilt unless both are still the very objects passed in; the scale and
    bias versions make an in-place update rebuild it too."""
    key = (id(wq), tuple(wq.shape), scales.data_ptr())
    hit = _TABLES.get(key)
    ver = (scales._version, biases._version)
    if hit is None or hit[0] != ver or hit[2]() is not wq or hit[3]() is not scales:
        hit = (ver, build_tables(wq, scales, biases), weakref.ref(wq), weakref.ref(scales))
        _TABLES[key] = hit
    return hit[1]


def clear_tables() -> None:
    _TABLES.clear()


def tables_nbytes() -> int:
    return sum(h[1].nbytes for h in _TABLES.values())


# --------------------------------------------------------------- activations

def quantize_activations(x: torch.Tensor):
    """Per (row, 64-group) int8 quantiser: (codes xu-128 int8 [R,K],
    scales fp32 [R,G], exact group sums fp32 [R,G])."""
    _need_cuda(x)
    x = _bf16(x, "x")
    R, K = x.shape
    xq = torch.empty(R, K, dtype=torch.int8, device=x.device)
    xsc = torch.empty(R, K // GROUP, dtype=torch.float32, device=x.device)
    xrs = torch.empty_like(xsc)
    _lib.call("tmoe_quantize_activations", _p(x), R, K, _p(xq), _p(xsc), _p(xrs),
              stream_ptr(x.device))
    return xq, xsc, xrs


# -------------------------------------------------------------------- router

def router_topk(x: torch.Tensor, router_w: torch.Tensor, k: int, return_probs: bool = False):
    """Canonical router: (idx int32 [T,k], scores bf16 [T,k][, logits, probs])."""
    _need_cuda(x, router_w)
    x = _bf16(x, "x")
    router_w = _bf16(router_w, "router weight")
    T, H = x.shape
    E = router_w.shape[0]
    logits = torch.empty(T, E, dtype=torch.bfloat16, device=x.device)
    idx = torch.empty(T, k, dtype=torch.int32, device=x.device)
    sc = torch.empty(T, k, dtype=torch.bfloat16, device=x.device)
    probs = torch.empty(T, E, dtype=torch.bfloat16, device=x.device) if return_probs else None
    _lib.call("tmoe_router_topk", _p(x), _p(router_w), T, H, E, k, _p(logits), _p(idx), _p(sc),
              _p(probs), stream_ptr(x.device))
    if return_probs:
        return idx, sc, logits, probs
    return idx, sc


# -------------------------------------------------------------- routing plan

def route_sort(indices: torch.Tensor, num_experts: int, with_tiles: bool = False):
    """Stable expert sort of flat ids: (order, inv_order, offsets[, tile_row,
    tile_exp, ntiles]).  order[r] = flat index of sorted row r."""
    _need_cuda(indices)
    idx = indices.reshape(-1).to(torch.int32).contiguous()
    R = idx.numel()
    dev = idx.device
    order = torch.empty(R, dtype=torch.int32, device=dev)
    inv = torch.empty(R, dtype=torch.int32, device=dev)
    off = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    maxt = (R + 127) // 128 + num_experts
    tr = te = nt = None
    if with_tiles:
        tr = torch.zeros(maxt, dtype=torch.int32, device=dev)
        te = torch.zeros(maxt, dtype=torch.int32, device=dev)
        nt = torch.zeros(1, dtype=torch.int32, device=dev)
    nb = _lib.load().tmoe_route_workspace_size(R, num_experts)
    ws = workspace(nb, dev, "route")
    _lib.call("tmoe_route_sort", _p(idx), R, num_experts, _p(ws), ws.numel(), _p(order), _p(inv),
              _p(off), _p(tr), _p(te), _p(nt), maxt if with_tiles else 0, stream_ptr(dev))
    if with_tiles:
        return order, inv, off, tr, te, nt
    return order, inv, off


# ------------------------------------------------------------------- gathers

def _broadcast_rows(x: torch.Tensor, rhs: torch.Tensor):
    """x [..., 1, K] and rhs [...] -> flat x rows [R, K], flat rhs [R] and the
    output batch shape (MLX gather_qmm broadcasting of the batch dims)."""
    if x.dim() < 2 or x.shape[-2] != 1:
        raise Unsupported(f"gather_qmm expects x [..., 1, K] (M = 1), got {tuple(x.shape)}")
    batch = torch.broadcast_shapes(tuple(x.shape[:-2]), tuple(rhs.shape))
    K = x.shape[-1]
    xb = x.expand(*batch, 1, K).reshape(-1, K).contiguous()
    rb = rhs.expand(*batch).reshape(-1).to(torch.int32).contiguous()
    return xb, rb, batch


def gather_qmm(x, w, scales, biases=None, lhs_indices=None, rhs_indices=None, transpose=True,
               group_size=GROUP, bits=BITS, mode="affine", sorted_indices=False, *, tables=None):
    """Stock mx.gather_qmm: y[b] = x[b] @ dequant(w[rhs[b]])^T with bf16
    activations and exact int4 dequantisation, fp32 accumulation, bf16 out."""
    _check_quant(transpose, group_size, bits, mode)
    if lhs_indices is not None:
        raise Unsupported("lhs_indices is not supported (the MoE block never passes it)")
    if biases is None or rhs_indices is None:
        raise Unsupported("affine gather needs biases and rhs_indices")
    _need_cuda(x, w, scales, biases, rhs_indices)
    x = _bf16(x, "x")
    w = _as_words(w)
    scales = _bf16(scales, "scales")
    biases = _bf16(biases, "biases")
    E, N, KW = w.shape
    K = KW * 8
    xr, rr, batch = _broadcast_rows(x, rhs_indices)
    R = xr.shape[0]
    y = torch.empty(R, N, dtype=torch.bfloat16, device=x.device)
    st = bt = None
    if R > 256:
        if tables is None:
            tables = build_tables(w, scales, biases)
        st, bt = tables.scales_t, tables.biases_t
    nb = _lib.load().tmoe_gather_qmm_bf16_workspace_size(R, E, N, K)
    ws = workspace(nb, x.device, "gather")
    _lib.call("tmoe_gather_qmm_bf16", _p(xr), _p(w), _p(scales), _p(biases), _p(st), _p(bt),
              _p(rr), R, E, N, K, _p(ws), ws.numel(), _p(y), stream_ptr(x.device))
    return y.reshape(*batch, 1, N)


def gather_qmm_int8(x, w, scales, biases, rhs_indices, tables: Int8Tables | None = None, *,
                    group_size=GROUP, bits=BITS):
    """int8 x int4 sorted gather (the overlay's op).  x [R, 1, K] bf16 sorted
    by expert, rhs_indices [R]; returns [R, 1, N] bf16."""
    _check_quant(True, group_size, bits, "affine")
    _need_cuda(x, w, rhs_indices)
    x = _bf16(x, "x")
    w = _as_words(w)
    E, N, KW = w.shape
    K = KW * 8
    if x.shape[-1] != K:
        raise InvalidArgument(f"x has K={x.shape[-1]}, weights K={K}")
    xr = x.reshape(-1, K).contiguous()
    rr = rhs_indices.reshape(-1).to(torch.int32).contiguous()
    R = xr.shape[0]
    if rr.numel() != R:
        raise InvalidArgument("rhs_indices must have one id per row of x")
    if tables is None:
        tables = build_tables(w, scales, biases)
    y = torch.empty(R, N, dtype=torch.bfloat16, device=x.device)
    nb = _lib.load().tmoe_gather_qmm_int8_workspace_size(R, E, N, K)
    ws = workspace(nb, x.device, "gather")
    _lib.call("tmoe_gather_qmm_int8", _p(xr), _p(w), _p(tables.scales_t), _p(tables.biases_t),
              _p(rr), R, E, N, K, _p(ws), ws.numel(), _p(y), stream_ptr(x.device))
    return y.reshape(R, 1, N)


def supported_int8(x, w, scales, biases, rhs_indices, transpose=True, group_size=GROUP,
                   bits=BITS) -> bool:
    """The routing predicate of engine/patches/moe-int8/kernel.py:466-479 for
    this kernel: affine 4-bit g64, bf16 [R, 1, K], K % 64 == 0, N % 128 == 0."""
    if not (transpose and group_size == GROUP and bits == BITS):
        return False
    if biases is None or w is None or rhs_indices is None:
        return False
    if w.dim() != 3 or scales.dim() != 3 or rhs_indices.dim() != 1:
        return False
    if x.dtype != torch.bfloat16 or x.dim() != 3 or x.shape[1] != 1:
        return False
    if x.shape[0] != rhs_indices.shape[0] or x.shape[-1] % GROUP:
        return False
    return scales.shape[1] % 128 == 0


# ----------------------------------------------------------- elementwise / sums

def swiglu(x_up: torch.Tensor, x_gate: torch.Tensor) -> torch.Tensor:
    """SwiGLU with bf16 rounding after each op (activations.py:9-11), via the
    library's kernel: returns silu(gate) * up."""
    _need_cuda(x_up, x_gate)
    up = _bf16(x_up, "x_up").reshape(-1, x_up.shape[-1])
    gate = _bf16(x_gate, "x_gate").reshape(-1, x_gate.shape[-1])
    gu = torch.cat([gate, up], dim=-1).contiguous()
    R, I2 = gu.shape
    h = torch.empty(R, I2 // 2, dtype=torch.bfloat16, device=gu.device)
    _lib.call("tmoe_swiglu", _p(gu), R, I2 // 2, _p(h), stream_ptr(gu.device))
    return h.reshape(x_up.shape)


def weighted_sum(xs: torch.Tensor, inv_order, scores: torch.Tensor, out_shape, mode="clone"):
    """Unsort + routed weighted sum (moe_weighted_sum.py:142-195)."""
    modes = {"clone": 0, "fast": 1}
    if mode not in modes:
        raise Unsupported(f"weighted_sum mode {mode!r} (have {sorted(modes)})")
    _need_cuda(xs, scores)
    D = out_shape[-1]
    rows = math.prod(out_shape[:-1])
    k = scores.shape[-1]
    ys = _bf16(xs, "xs").reshape(rows * k, D).contiguous()
    sc = scores.reshape(rows * k).to(torch.bfloat16).contiguous()
    inv = None if inv_order is None else inv_order.reshape(-1).to(torch.int32).contiguous()
    out = torch.empty(*out_shape, dtype=torch.bfloat16, device=xs.device)
    _lib.call("tmoe_weighted_sum", _p(ys), _p(inv), _p(sc), rows, k, D, modes[mode], _p(out),
              stream_ptr(xs.device))
    return out


def gate_up_silu(x, weight, scales, biases, idx, group_size=GROUP):
    """decode-fusion gate_up_silu: x [T, K] bf16, fused gate_up [E, 2I, K/8],
    idx [T, k] -> h [T, k, I] fp32."""
    _check_quant(True, group_size, BITS, "affine")
    _need_cuda(x, weight, idx)
    x = _bf16(x, "x")
    w = _as_words(weight)
    T, K = x.shape
    E, I2, _ = w.shape
    k = idx.shape[-1]
    idx = idx.to(torch.int32).contiguous()
    h = torch.empty(T, k, I2 // 2, dtype=torch.float32, device=x.device)
    nb = _lib.load().tmoe_decode_workspace_size(T, k, E, K, I2 // 2)
    ws = workspace(nb, x.device, "decode")
    _lib.call("tmoe_gate_up_silu", _p(x), _p(w), _p(_bf16(scales, "scales")),
              _p(_bf16(biases, "biases")), _p(idx), T, k, E, K, I2 // 2, _p(ws), ws.numel(), _p(h),
              stream_ptr(x.device))
    return h


def down_wsum(h, weight, scales, biases, idx, scores, group_size=GROUP):
    """decode-fusion down_wsum: h [T, k, I] fp32, down [E, D, I/8], idx,
    scores [T, k] fp32 -> y [T, D] bf16."""
    _check_quant(True, group_size, BITS, "affine")
    _need_cuda(h, weight, idx, scores)
    h = h.float().contiguous()
    w = _as_words(weight)
    T, k, I = h.shape
    E, D, _ = w.shape
    idx = idx.to(torch.int32).contiguous()
    sc = scores.float().contiguous()
    y = torch.empty(T, D, dtype=torch.bfloat16, device=h.device)
    nb = _lib.load().tmoe_decode_workspace_size(T, k, E, max(D, I), I)
    ws = workspace(nb, h.device, "decode")
    _lib.call("tmoe_down_wsum", _p(h), _p(w), _p(_bf16(scales, "scales")),
              _p(_bf16(biases, "biases")), _p(idx), _p(sc), T, k, E, I, D, _p(ws), ws.numel(), _p(y),
              stream_ptr(h.device))
    return y


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """nn.RMSNorm (qwen3_5_moe/language.py:103-107): bf16 rows x [..., H]."""
    _need_cuda(x, weight)
    H = x.shape[-1]
    xf = _bf16(x, "x").reshape(-1, H).contiguous()
    w = _bf16(weight, "weight").contiguous()
    out = torch.empty_like(xf)
    _lib.call("tmoe_rmsnorm", _p(xf), _p(w), xf.shape[0], H, float(eps), _p(out),
              stream_ptr(x.device))
    return out.reshape(x.shape)


def residual_inject(branch: torch.Tensor, residual: torch.Tensor,
                    weights: torch.Tensor | None = None) -> torch.Tensor:
    """The write-back of a branch: branch + residual, or with weights [T, n]
    the hyper-connection inject into residual [T, n, H]
    (qwen4_exp/language.py:3198-3218)."""
    _need_cuda(branch, residual)
    H = branch.shape[-1]
    b = _bf16(branch, "branch").reshape(-1, H).contiguous()
    r = _bf16(residual, "residual").contiguous()
    n = 0 if weights is None else weights.shape[-1]
    w = None if weights is None else _bf16(weights, "weights").reshape(-1, n).contiguous()
    out = torch.empty_like(r)
    _lib.call("tmoe_residual_inject", _p(b), _p(r), _p(w), b.shape[0], H, n, _p(out),
              stream_ptr(branch.device))
    return out
