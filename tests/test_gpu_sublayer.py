"""The steps either side of the MoE block: the post-attention RMSNorm and the
residual / hyper-connection write-back, alone and fused into the sub-layer
call, bit for bit against the CPU oracle's restatement
(qwen3_5_moe/language.py:103-107, 136-137; qwen4_exp/language.py:3198-3218,
3338-3343)."""
import numpy as np
import pytest
import torch

from gpu_util import bf, load_block, nbf
from helpers import f32


def test_oracle_rmsnorm_known_values(oracle):
    x = oracle.f32_to_bf16(np.array([[3.0, 4.0] * 32, [0.0] * 64], np.float32))
    w = oracle.f32_to_bf16(np.full(64, 2.0, np.float32))
    y = f32(oracle.rmsnorm(x, w, eps=0.0))
    r = 1.0 / np.sqrt(np.float32(12.5))
    assert np.allclose(y[0, :2], [3.0 * r * 2.0, 4.0 * r * 2.0], rtol=2 ** -8)
    y = f32(oracle.rmsnorm(x[1:], w, eps=1e-6))
    assert (y == 0).all()
    b = oracle.f32_to_bf16(np.ones((2, 8), np.float32))
    res = oracle.f32_to_bf16(np.full((2, 3, 8), 0.5, np.float32))
    wt = oracle.f32_to_bf16(np.array([[1.0, 2.0, 0.25]] * 2, np.float32))
    out = f32(oracle.inject(b, res, wt))
    assert np.allclose(out[:, :, 0], [[1.5, 2.5, 0.75]] * 2)


@pytest.mark.gpu
@pytest.mark.parametrize("H,scale", [(2048, 1.0), (3072, 30.0), (512, 1e-3)])
def test_rmsnorm_bitexact(cuda, oracle, H, scale):
    from titan_b200 import ops
    x = oracle.make_x(77, H, seed=H, scale=scale)
    w = oracle.f32_to_bf16(np.random.default_rng(H).normal(1.0, 0.1, H).astype(np.float32))
    got = ops.rmsnorm(bf(x), bf(w), eps=1e-6)
    assert np.array_equal(nbf(got), oracle.rmsnorm(x, w, eps=1e-6))


@pytest.mark.gpu
@pytest.mark.parametrize("n", [0, 4])
def test_residual_inject_bitexact(cuda, oracle, n):
    from titan_b200 import ops
    T, H = 33, 1024
    b = oracle.make_x(T, H, seed=1)
    res = oracle.make_x(T * max(n, 1), H, seed=2).reshape((T, n, H) if n else (T, H))
    wt = oracle.make_x(T, n, seed=3) if n else None
    got = ops.residual_inject(bf(b), bf(res), None if wt is None else bf(wt))
    assert np.array_equal(nbf(got), oracle.inject(b, res, wt))


@pytest.mark.gpu
@pytest.mark.parametrize("n", [0, 4])
def test_moe_sublayer_bitexact(cuda, oracle, n):
    """One call: norm, block (routed int8 experts, bit-exact in the
    re-centred order), write-back; equal to the oracle's composition."""
    from titan_b200 import SparseMoeBlock, _lib
    H = 1024
    L = oracle.make_layer(H=H, E=32, k=6, I=256, Is=0, seed=9)
    blk = SparseMoeBlock(H, 32, 6, 256, 0, device=cuda, init=False)
    load_block(blk, L)
    T = 150
    h = oracle.make_x(T, H, seed=9, scale=4.0)
    w = oracle.f32_to_bf16(np.random.default_rng(9).normal(1.0, 0.1, H).astype(np.float32))
    res = oracle.make_x(T * n, H, seed=10).reshape(T, n, H) if n else None
    wt = oracle.make_x(T, n, seed=11) if n else None
    o = _lib.Options()
    o.min_tokens, o.int8_prefill, o.down_int8, o.wsum_mode = 1, 1, 1, 0
    out = blk.forward_sublayer(bf(h), bf(w), eps=1e-6,
                               residual=None if res is None else bf(res),
                               inject_weights=None if wt is None else bf(wt), options=o)
    xn = oracle.rmsnorm(h, w, eps=1e-6)
    y, _, _ = oracle.moe_prefill(L, xn, int8_mode=3 | 4)
    ref = oracle.inject(y, h if n == 0 else res, wt)
    assert np.array_equal(nbf(out), ref)
