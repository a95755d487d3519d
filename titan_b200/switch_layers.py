"""SwitchGLU and QuantizedSwitchLinear on torch CUDA tensors.

Mirrors titan/adapters/mlx/vendor/mlx_lm/models/switch_layers.py:13-245 with
the loader's fused [gate | up] layout (gate rows first, loader.py:440-470):

  * ``QuantizedSwitchLinear.forward`` calls ``ops.gather_qmm`` through the
    module attribute, so ``titan_b200.patch.install()`` swaps it exactly the
    way the reference overlay swaps ``mx.gather_qmm``;
  * ``SwitchGLU.forward`` sorts the routed rows by expert when
    ``indices.numel() >= 64`` (switch_layers.py:218), runs gate_up, SwiGLU and
    down, and unsorts.
"""
from __future__ import annotations

import math

import torch
from torch import nn

from . import ops
from ._lib import Unsupported


def _gather_sort(x, indices, num_experts):
    """switch_layers.py:13-18: rows in expert order, sorted ids, inverse."""
    M = indices.shape[-1]
    flat = indices.reshape(-1)
    order, inv, _ = ops.route_sort(flat, num_experts)
    order = order.long()
    xs = x.flatten(0, -3)[order // M]
    return xs, flat[order], inv.long()


def _scatter_unsort(x, inv_order, shape=None):
    """switch_layers.py:21-25."""
    x = x[inv_order]
    if shape is not None:
        x = x.unflatten(0, tuple(shape))
    return x


class QuantizedSwitchLinear(nn.Module):
    """Per-expert affine int4 (group 64) linear: weight [E, out, in/8] int32
    words, scales / biases [E, out, in/64] bf16."""

    def __init__(self, input_dims: int, output_dims: int, num_experts: int, bias: bool = False,
                 group_size: int = 64, bits: int = 4, mode: str = "affine", device=None,
                 init: bool = True, weight_std: float | None = None):
        """``init``: draw fp32 weights and quantise them on the GPU, a chunk
        of experts at a time — uniform(-1/sqrt(in), 1/sqrt(in)) as the
        reference's constructor (switch_layers.py:41-51), or N(0, weight_std)
        when given (the benchmark workloads use N(0, 0.02))."""
        super().__init__()
        if bias:
            raise Unsupported("QuantizedSwitchLinear with bias is not part of the MoE block")
        if (group_size, bits, mode) != (64, 4, "affine"):
            raise Unsupported("only affine int4 with group size 64 is implemented")
        self.group_size, self.bits, self.mode = group_size, bits, mode
        device = torch.device(device or "cuda")
        wq = torch.zeros(num_experts, output_dims, input_dims // 8, dtype=torch.int32, device=device)
        s = torch.zeros(num_experts, output_dims, input_dims // 64, dtype=torch.bfloat16, device=device)
        b = torch.zeros_like(s)
        if init:
            scale = math.sqrt(1.0 / input_dims)
            chunk = max(1, (1 << 27) // max(1, output_dims * input_dims))
            for e0 in range(0, num_experts, chunk):
                n = min(chunk, num_experts - e0)
                w = torch.empty(n, output_dims, input_dims, device=device)
                if weight_std is None:
                    w.uniform_(-scale, scale)
                else:
                    w.normal_(0.0, weight_std)
                wq[e0:e0 + n], s[e0:e0 + n], b[e0:e0 + n] = ops.quantize(w)
                del w
        self.register_buffer("weight", wq)
        self.register_buffer("scales", s)
        self.register_buffer("biases", b)

    @property
    def input_dims(self) -> int:
        return self.scales.shape[2] * self.group_size

    @property
    def output_dims(self) -> int:
        return self.weight.shape[1]

    @property
    def num_experts(self) -> int:
        return self.weight.shape[0]

    def forward(self, x, indices, sorted_indices: bool = False):
        return ops.gather_qmm(x, self.weight, self.scales, self.biases, rhs_indices=indices,
                              transpose=True, group_size=self.group_size, bits=self.bits,
                              mode=self.mode, sorted_indices=sorted_indices,
                              tables=ops.cached_tables(self.weight, self.scales, self.biases))


class SwiGLU(nn.Module):
    def forward(self, x, gate):
        return ops.swiglu(x, gate)


class SwitchGLU(nn.Module):
    def __init__(self, input_dims: int, hidden_dims: int, num_experts: int, activation=None,
                 bias: bool = False, device=None, init: bool = True,
                 weight_std: float | None = None):
        super().__init__()
        self.gate_up_proj = QuantizedSwitchLinear(input_dims, 2 * hidden_dims, num_experts, bias,
                                                  device=device, init=init, weight_std=weight_std)
        self.down_proj = QuantizedSwitchLinear(hidden_dims, input_dims, num_experts, bias,
                                               device=device, init=init, weight_std=weight_std)
        self.activation = activation or SwiGLU()

    def forward(self, x, indices):
        x = x.unsqueeze(-2).unsqueeze(-3)
        do_sort = indices.numel() >= 64
        idx, inv_order = indices, None
        if do_sort:
            x, idx, inv_order = _gather_sort(x, indices, self.gate_up_proj.num_experts)
        gate_up = self.gate_up_proj(x, idx, sorted_indices=do_sort)
        x_gate, x_up = gate_up.chunk(2, dim=-1)
        x = self.down_proj(self.activation(x_up, x_gate), idx, sorted_indices=do_sort)
        if do_sort:
            x = _scatter_unsort(x, inv_order, indices.shape)
        return x.squeeze(-2)
