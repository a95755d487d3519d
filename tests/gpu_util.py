"""numpy <-> torch CUDA conversion for the parity tests (bf16 as uint16 bits)."""
from __future__ import annotations

import numpy as np
import torch


def bf(a: np.ndarray, dev="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).to(dev).view(
        torch.bfloat16)


def words(a: np.ndarray, dev="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint32).view(np.int32)).to(dev)


def i32(a: np.ndarray, dev="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)


def f32t(a: np.ndarray, dev="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


def nbf(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def nwords(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().numpy().view(np.uint32)


def load_block(block, L) -> None:
    """Copy an oracle.Layer's weights into a titan_b200.SparseMoeBlock."""
    sm = block.switch_mlp
    block.gate_weight.copy_(bf(L.wr))
    sm.gate_up_proj.weight.copy_(words(L.gu_w))
    sm.gate_up_proj.scales.copy_(bf(L.gu_s))
    sm.gate_up_proj.biases.copy_(bf(L.gu_b))
    sm.down_proj.weight.copy_(words(L.dn_w))
    sm.down_proj.scales.copy_(bf(L.dn_s))
    sm.down_proj.biases.copy_(bf(L.dn_b))
    if L.sgu_w is not None:
        se = block.shared_expert
        se.gate_up_proj.weight.copy_(words(L.sgu_w))
        se.gate_up_proj.scales.copy_(bf(L.sgu_s))
        se.gate_up_proj.biases.copy_(bf(L.sgu_b))
        se.down_proj.weight.copy_(words(L.sdn_w))
        se.down_proj.scales.copy_(bf(L.sdn_s))
        se.down_proj.biases.copy_(bf(L.sdn_b))
        block.shared_expert_gate_weight.copy_(bf(L.wg[None, :]))
    block._layer = None
    block._tables = None


def layer_from_block(oracle, block):
    """The inverse: an oracle.Layer holding a block's (GPU-initialised) weights."""
    sm = block.switch_mlp
    L = oracle.Layer(block.hidden, block.num_experts, block.top_k, block.moe_inter,
                     block.shared_inter, nbf(block.gate_weight),
                     nwords(sm.gate_up_proj.weight), nbf(sm.gate_up_proj.scales),
                     nbf(sm.gate_up_proj.biases), nwords(sm.down_proj.weight),
                     nbf(sm.down_proj.scales), nbf(sm.down_proj.biases))
    if block.shared_expert is not None:
        se = block.shared_expert
        L.sgu_w, L.sgu_s, L.sgu_b = (nwords(se.gate_up_proj.weight), nbf(se.gate_up_proj.scales),
                                     nbf(se.gate_up_proj.biases))
        L.sdn_w, L.sdn_s, L.sdn_b = (nwords(se.down_proj.weight), nbf(se.down_proj.scales),
                                     nbf(se.down_proj.biases))
        L.wg = nbf(block.shared_expert_gate_weight)[0]
    return L
