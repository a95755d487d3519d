"""The speculative-decode verify layout and the batched verify workload.

The reference's verify step (titan/adapters/mlx/vendor/mlx_vlm/models/
qwen3_5_moe/language.py:16-41) flattens x [B, T, D] to B*T tokens, runs the
experts through unsorted stock gathers, keeps the expert outputs token-major
and combines them with the weighted sum's no-permutation layout
(engine/patches/round3/small-items/REPORT.md:7-12).  Routing must be
bit-exact; outputs follow the stock path's bar.  The routing generator of
the batched verify workload (64 streams x 4 tokens, Zipf(1.2), 7 shared
experts per stream) prescribes every token's top-k set, so the router's
selection is checked bit for bit against it.
"""
import numpy as np
import pytest
import torch

from gpu_util import bf, layer_from_block, load_block, nbf
from helpers import assert_bf16_close, f32, rel_rms

import bench


def test_spec_tokens_prescribe_the_routing(oracle):
    """CPU: the generator's sets are the top-k of its one-hot router logits,
    with a clear gap at the boundary, and the tokens of a stream share at
    least 7 experts."""
    x, sets = bench.spec_tokens(8, 3, 256, 64, 10, seed=3)
    xf = oracle.f32_to_bf16(x.reshape(-1, 256))
    wr = np.zeros((64, 256), np.float32)
    wr[np.arange(64), np.arange(64)] = 1.0
    idx, sc, _, _ = oracle.router(xf, oracle.f32_to_bf16(wr), 10)
    assert np.array_equal(np.sort(idx, axis=1), sets)
    s = sets.reshape(8, 4, 10)
    for st in range(8):
        common = set(s[st, 0])
        for j in range(1, 4):
            common &= set(s[st, j])
        assert len(common) >= 7


@pytest.mark.gpu
def test_verify_layout_matches_oracle_and_modular(cuda, oracle):
    from titan_b200 import SparseMoeBlock
    L = oracle.make_layer(H=512, E=64, k=10, I=128, Is=256, seed=41)
    wr = np.zeros((64, 512), np.float32)
    wr[np.arange(64), np.arange(64)] = 1.0
    L.wr = oracle.f32_to_bf16(wr)
    blk = SparseMoeBlock(512, 64, 10, 128, 256, device=cuda, init=False)
    load_block(blk, L)
    x, sets = bench.spec_tokens(6, 3, 512, 64, 10, seed=5)
    xb = oracle.f32_to_bf16(x)
    y, idx, sc = blk.forward_verify(bf(xb), return_routing=True)
    assert y.shape == (6, 4, 512)
    assert np.array_equal(np.sort(idx.cpu().numpy(), axis=1), sets)
    flat = xb.reshape(24, 512)
    ry, ridx, rsc, ops = oracle.moe_prefill(L, flat, int8_mode=0, parts=True)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.array_equal(nbf(sc), rsc)
    yf = f32(nbf(y).reshape(24, 512))
    assert rel_rms(yf, f32(ry)) < 1e-2
    assert_bf16_close(nbf(y).reshape(24, 512), ry, what="verify layout", operands=ops,
                      operand_ulps=4)
    ym = blk.forward_verify_modular(bf(xb))
    assert rel_rms(f32(nbf(ym).reshape(24, 512)), f32(ry)) < 1e-2
    # the verify step is the block on the flattened tokens, bit for bit
    y2 = blk(bf(flat), options=blk.verify_options())
    assert torch.equal(y.reshape(24, 512).view(torch.int16), y2.view(torch.int16))


@pytest.mark.gpu
def test_batched_verify_full_shape(cuda, oracle):
    """The batched verify workload at the decode shape (H=2048, 512 experts +
    shared, I=512, top-10): 64 streams x 4 tokens, every token's top-k set
    as prescribed, scores bit-exact, and a subset of outputs against the
    oracle on those tokens."""
    from titan_b200 import SparseMoeBlock
    torch.manual_seed(2)
    blk = SparseMoeBlock(2048, 512, 10, 512, 512, device=cuda)
    bench.spec_router_(blk)
    L = layer_from_block(oracle, blk)
    x, sets = bench.spec_tokens(64, 3, 2048, 512, 10, seed=77)
    xb = oracle.f32_to_bf16(x)
    y, idx, sc = blk.forward_verify(bf(xb), return_routing=True)
    assert np.array_equal(np.sort(idx.cpu().numpy(), axis=1), sets)
    flat = xb.reshape(256, 2048)
    ridx, rsc, _, _ = oracle.router(flat, L.wr, 10)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.array_equal(nbf(sc), rsc)
    sub = np.r_[0:4, 128:132, 252:256]
    ry, _, _, ops = oracle.moe_prefill(L, np.ascontiguousarray(flat[sub]), int8_mode=0,
                                       parts=True)
    got = nbf(y).reshape(256, 2048)[sub]
    assert rel_rms(f32(got), f32(ry)) < 1e-2
    assert_bf16_close(got, ry, what="batched verify subset", operands=ops, operand_ulps=4)
