"""Committed regression vectors (tests/golden/moe_small.npz, written by
tests/golden/make_golden.py): the oracle must reproduce them bit for bit on
CPU, and the CUDA path must match them on the GPU (bit-exact where the
arithmetic is integer or fixed-order, within the north-star tolerance
elsewhere)."""
import os

import numpy as np
import pytest

from helpers import assert_bf16_close

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "moe_small.npz")


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


def _layer(oracle, g):
    H, E, k, I, Is = (int(v) for v in g["shape"])
    L = oracle.Layer(H, E, k, I, Is, g["w_wr"], g["w_gu_w"], g["w_gu_s"], g["w_gu_b"],
                     g["w_dn_w"], g["w_dn_s"], g["w_dn_b"])
    for n in ("sgu_w", "sgu_s", "sgu_b", "sdn_w", "sdn_s", "sdn_b", "wg"):
        setattr(L, n, g["w_" + n])
    return L


def test_oracle_reproduces_golden_router_and_gathers(oracle, golden):
    g = golden
    L = _layer(oracle, g)
    idx, sc, logits, probs = oracle.router(g["x"], L.wr, L.k)
    assert np.array_equal(idx, g["router_idx"])
    assert np.array_equal(sc, g["router_scores"])
    assert np.array_equal(logits, g["router_logits"])
    assert np.array_equal(probs, g["router_probs"])
    for order in (0, 1):
        got = oracle.gather_qmm_int8(g["gather_x"], L.gu_w, L.gu_s, L.gu_b, g["gather_ids"],
                                     order=order)
        assert np.array_equal(got, g[f"gather_int8_order{order}"])


@pytest.mark.parametrize("mode", [0, 1, 3, 7])
def test_oracle_reproduces_golden_block(oracle, golden, mode):
    g = golden
    L = _layer(oracle, g)
    y, idx, _ = oracle.moe_prefill(L, g["x"], int8_mode=mode)
    assert np.array_equal(idx, g["router_idx"])
    assert np.array_equal(y, g[f"prefill_mode{mode}"])


def test_oracle_reproduces_golden_decode(oracle, golden):
    g = golden
    L = _layer(oracle, g)
    T = g["decode_y"].shape[0]
    y, _, _ = oracle.moe_decode(L, g["x"][:T])
    assert np.array_equal(y, g["decode_y"])


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", [0, 2, 1], ids=["tcgen05_tile", "tcgen05_swapab", "mma_sync"])
def test_cuda_block_matches_golden(cuda, oracle, golden, kernel):
    from gpu_util import bf, load_block, nbf
    from titan_b200 import SparseMoeBlock, _lib
    g = golden
    L = _layer(oracle, g)
    blk = SparseMoeBlock(L.H, L.E, L.k, L.I, L.Is, device=cuda, init=False)
    load_block(blk, L)
    o = _lib.Options()
    o.min_tokens, o.int8_prefill, o.down_int8, o.wsum_mode, o.gemm_kernel = 1, 1, 1, 0, kernel
    y, idx, sc = blk(bf(g["x"]), options=o, return_routing=True)
    assert np.array_equal(idx.cpu().numpy(), g["router_idx"])
    assert np.array_equal(nbf(sc), g["router_scores"])
    ops = (g["mode3_routed"], g["mode3_shared"], g["mode3_termmax"])
    assert_bf16_close(nbf(y), g["prefill_mode3"], what="prefill int8 block", operands=ops,
                      operand_ulps=4)
    o.min_tokens = 512
    T = g["decode_y"].shape[0]
    yd = blk(bf(g["x"][:T]), options=o)
    assert_bf16_close(nbf(yd), g["decode_y"], what="decode block")


@pytest.mark.gpu
def test_cuda_int8_gather_matches_golden_bitexact(cuda, golden):
    from gpu_util import bf, i32, nbf, words
    from titan_b200 import ops
    g = golden
    R, K = g["gather_x"].shape
    got = ops.gather_qmm_int8(bf(g["gather_x"]).reshape(R, 1, K), words(g["w_gu_w"]),
                              bf(g["w_gu_s"]), bf(g["w_gu_b"]), i32(g["gather_ids"]))
    assert np.array_equal(nbf(got.reshape(R, -1)), g["gather_int8_order1"])
