"""Per-kernel parity of the CUDA path against the CPU oracle (run on a B200).

Bit-exact where the arithmetic is integer or follows the canonical order the
oracle fixes (weight quantiser, tables, activation quantiser, router logits,
probabilities, indices and scores, routing sort, SwiGLU, clone weighted sum,
the int8 gather in its re-centred order); within the north-star tolerance
(2 bf16 ULP or 1e-2 relative, whichever is looser) where tensor-core fp32
accumulation order differs (bf16-activation gathers, decode GEMVs).
"""
import numpy as np
import pytest
import torch

from gpu_util import bf, f32t, i32, nbf, nwords, words
from helpers import assert_bf16_close, f32, rel_rms

pytestmark = pytest.mark.gpu


def test_affine_quantize_bitexact(cuda, oracle):
    from titan_b200 import ops
    rng = np.random.default_rng(0)
    w = rng.standard_normal((96, 512), dtype=np.float32) * 0.02
    w[0] = 0.0
    w[1, :64] = 3.0
    wq, s, b = ops.quantize(torch.from_numpy(w).to(cuda))
    owq, os_, ob = oracle.affine_quantize(w)
    assert np.array_equal(nwords(wq), owq)
    assert np.array_equal(nbf(s), os_) and np.array_equal(nbf(b), ob)


def test_tables_and_qsum(cuda, oracle):
    from titan_b200 import ops
    L = oracle.make_layer(H=256, E=4, k=2, I=128, seed=1)
    st, bt = ops.prepare_tables(bf(L.gu_s), bf(L.gu_b))
    ost = L.gu_s.transpose(0, 2, 1)
    assert np.array_equal(nbf(st), ost)
    assert np.array_equal(nbf(bt), L.gu_b.transpose(0, 2, 1))
    qs = ops.qsum(words(L.gu_w)).cpu().numpy()
    assert np.array_equal(qs, oracle.qsum(L.gu_w).astype(np.int64))


@pytest.mark.parametrize("R,K", [(1, 64), (37, 2048), (1000, 3072)])
def test_quantize_activations_bitexact(cuda, oracle, R, K):
    from titan_b200 import ops
    x = oracle.make_x(R, K, seed=R)
    xq, xsc, xrs = ops.quantize_activations(bf(x))
    oxs, oxsc, oxrs, _ = oracle.quantize_act(x)
    assert np.array_equal(xq.cpu().numpy(), oxs)
    assert np.array_equal(xsc.cpu().numpy(), oxsc)
    assert np.array_equal(xrs.cpu().numpy(), oxrs)


@pytest.mark.parametrize("T,H,E,k", [(1, 2048, 512, 10), (3, 2048, 512, 10), (8, 2048, 512, 10),
                                     (32, 2048, 512, 10), (33, 256, 64, 4), (128, 2048, 64, 10),
                                     (300, 3072, 512, 10), (64, 512, 1024, 32)])
def test_router_bitexact(cuda, oracle, T, H, E, k):
    from titan_b200 import ops
    rng = np.random.default_rng(T * 7 + E)
    x = oracle.make_x(T, H, seed=T + H)
    wr = oracle.f32_to_bf16(rng.standard_normal((E, H), dtype=np.float32) * 0.02)
    idx, sc, lg, pb = ops.router_topk(bf(x), bf(wr), k, return_probs=True)
    oidx, osc, olg, opb = oracle.router(x, wr, k)
    assert np.array_equal(nbf(lg), olg), "logits"
    assert np.array_equal(nbf(pb), opb), "probabilities"
    assert np.array_equal(idx.cpu().numpy(), oidx), "indices"
    assert np.array_equal(nbf(sc), osc), "scores"


def test_router_ties_lowest_index(cuda, oracle):
    from titan_b200 import ops
    H, E, k = 64, 64, 4
    x = oracle.f32_to_bf16(np.ones((2, H), np.float32))
    w = np.zeros((E, H), np.float32)
    w[[5, 17, 40, 41, 63], :] = 1.0 / H
    wr = oracle.f32_to_bf16(w)
    idx, sc = ops.router_topk(bf(x), bf(wr), k)
    assert idx.cpu().numpy().tolist() == [[5, 17, 40, 41]] * 2


@pytest.mark.parametrize("R,E", [(1, 8), (10, 512), (320, 512), (2048, 64), (2049, 64),
                                 (40960, 512), (100000, 1024)])
def test_route_sort_matches_stable_argsort(cuda, oracle, R, E):
    from titan_b200 import ops
    rng = np.random.default_rng(R)
    p = 1.0 / np.arange(1, E + 1) ** 1.1          # Zipf-skewed, many empty experts
    ids = rng.choice(E, size=R, p=p / p.sum()).astype(np.int32)
    order, inv, off, tr, te, nt = ops.route_sort(i32(ids), E, with_tiles=True)
    oorder, oinv, ooff = oracle.sort_routes(ids, E)
    assert np.array_equal(order.cpu().numpy(), oorder)
    assert np.array_equal(inv.cpu().numpy(), oinv)
    assert np.array_equal(off.cpu().numpy(), ooff)
    # tile table: every expert's rows covered by tiles of 128 in order
    n = int(nt.item())
    cnt = np.diff(ooff)
    assert n == int(np.sum((cnt + 127) // 128))
    exp_rows = [(e, ooff[e] + r) for e in range(E) for r in range(0, cnt[e], 128)]
    got = list(zip(te.cpu().numpy()[:n].tolist(), tr.cpu().numpy()[:n].tolist()))
    assert got == exp_rows


def test_route_sort_one_expert_takes_all(cuda, oracle):
    from titan_b200 import ops
    ids = np.full(5000, 7, np.int32)
    order, inv, off = ops.route_sort(i32(ids), 16)
    assert np.array_equal(order.cpu().numpy(), np.arange(5000))
    assert off.cpu().numpy().tolist() == [0] * 8 + [5000] * 9


def test_swiglu_bitexact(cuda, oracle):
    from titan_b200 import ops
    rng = np.random.default_rng(3)
    gu = oracle.f32_to_bf16(rng.standard_normal((50, 256), dtype=np.float32) * 3)
    h = ops.swiglu(bf(gu[:, 128:]), bf(gu[:, :128]))
    assert np.array_equal(nbf(h), oracle.swiglu(gu))


@pytest.mark.parametrize("T,D,k,sorted_layout", [(1, 2048, 10, False), (9, 256, 10, True),
                                                 (13, 2560, 10, True), (128, 2048, 10, True),
                                                 (32, 512, 6, True), (32, 512, 8, False)])
@pytest.mark.parametrize("mode", ["clone", "fast"])
def test_weighted_sum_bitexact(cuda, oracle, T, D, k, sorted_layout, mode):
    from titan_b200 import ops
    rng = np.random.default_rng(T + D)
    ys = oracle.f32_to_bf16(rng.standard_normal((T * k, D), dtype=np.float32))
    sc = rng.uniform(size=(T, k)).astype(np.float32)
    sc = oracle.f32_to_bf16(sc / sc.sum(1, keepdims=True))
    inv = rng.permutation(T * k).astype(np.int32) if sorted_layout else None
    got = ops.weighted_sum(bf(ys), None if inv is None else i32(inv), bf(sc), (T, D), mode=mode)
    ref = oracle.weighted_sum(ys, inv, sc, mode={"clone": 0, "fast": 1}[mode])
    assert np.array_equal(nbf(got), ref)


def _gather_inputs(oracle, R, E, N, K, seed, zipf=True):
    rng = np.random.default_rng(seed)
    dense = rng.standard_normal((E, N, K), dtype=np.float32) * 0.02
    wq, s, b = oracle.affine_quantize(dense)
    if zipf:
        p = 1.0 / np.arange(1, E + 1)
        ids = np.sort(rng.choice(E, size=R, p=p / p.sum())).astype(np.int32)
    else:
        ids = np.sort(rng.integers(0, E, size=R)).astype(np.int32)
    x = oracle.make_x(R, K, seed=seed + 11)
    return x, wq, s, b, ids


@pytest.mark.parametrize("R,E,N,K", [(64, 8, 256, 256), (128, 8, 256, 512), (300, 16, 1024, 2048),
                                     (1280, 64, 1024, 2048), (777, 32, 3072, 768)])
def test_gather_qmm_int8_bitexact_recentred_order(cuda, oracle, R, E, N, K):
    """The kernel evaluates the reference's algebra in the re-centred order:
    bit-identical to the oracle in that order, and within one bf16 ULP of the
    reference's own FMA order."""
    from titan_b200 import ops
    x, wq, s, b, ids = _gather_inputs(oracle, R, E, N, K, seed=R)
    got = ops.gather_qmm_int8(bf(x).reshape(R, 1, K), words(wq), bf(s), bf(b), i32(ids))
    got = nbf(got.reshape(R, N))
    assert np.array_equal(got, oracle.gather_qmm_int8(x, wq, s, b, ids, order=1))
    ref0 = oracle.gather_qmm_int8(x, wq, s, b, ids, order=0)
    assert_bf16_close(got, ref0, ulps=1, rel=0, what="vs reference FMA order")
    stock = oracle.gather_qmm_exact(x, wq, s, b, ids)
    assert rel_rms(f32(got), f32(stock)) < 0.02


def test_gather_qmm_int8_unsorted_and_empty_experts(cuda, oracle):
    """Rows handed over in any order come back in the caller's order."""
    from titan_b200 import ops
    x, wq, s, b, ids = _gather_inputs(oracle, 500, 64, 256, 512, seed=9)
    perm = np.random.default_rng(0).permutation(500)
    got = nbf(ops.gather_qmm_int8(bf(x[perm]).reshape(500, 1, 512), words(wq), bf(s), bf(b),
                                  i32(ids[perm])).reshape(500, 256))
    ref = oracle.gather_qmm_int8(x, wq, s, b, ids, order=1)
    assert np.array_equal(got, ref[perm])


@pytest.mark.parametrize("R,E,N,K,sorted_", [(5, 8, 256, 256, False), (40, 64, 1024, 2048, False),
                                             (256, 16, 512, 512, True), (300, 16, 1024, 2048, True),
                                             (2000, 64, 1536, 3072, True)])
def test_gather_qmm_bf16_vs_exact(cuda, oracle, R, E, N, K, sorted_):
    from titan_b200 import ops
    x, wq, s, b, ids = _gather_inputs(oracle, R, E, N, K, seed=R + 1, zipf=sorted_)
    if not sorted_:
        ids = np.random.default_rng(1).permutation(ids).astype(np.int32)
    got = ops.gather_qmm(bf(x).reshape(R, 1, K), words(wq), bf(s), bf(b), rhs_indices=i32(ids),
                         sorted_indices=sorted_)
    ref = oracle.gather_qmm_exact(x, wq, s, b, ids)
    assert_bf16_close(nbf(got.reshape(R, N)), ref, what="bf16 gather")


def test_gather_qmm_broadcast_decode_layout(cuda, oracle):
    """SwitchGLU's unsorted decode call: x [T,1,1,K] with indices [T,k]."""
    from titan_b200 import ops
    T, k, E, N, K = 3, 10, 64, 1024, 2048
    x, wq, s, b, _ = _gather_inputs(oracle, T, E, N, K, seed=4)
    ids = np.random.default_rng(2).integers(0, E, size=(T, k)).astype(np.int32)
    got = ops.gather_qmm(bf(x).reshape(T, 1, 1, K), words(wq), bf(s), bf(b), rhs_indices=i32(ids))
    assert tuple(got.shape) == (T, k, 1, N)
    ref = oracle.gather_qmm_exact(np.repeat(x, k, axis=0), wq, s, b, ids.reshape(-1))
    assert_bf16_close(nbf(got.reshape(T * k, N)), ref)


@pytest.mark.parametrize("T,E,H,I", [(1, 64, 2048, 512), (2, 512, 2048, 512), (8, 64, 3072, 768),
                                     (32, 128, 2048, 512)])
def test_decode_fused_ops_vs_fp32_golden(cuda, oracle, T, E, H, I):
    """decode-fusion gate_up_silu / down_wsum against the fp32 golden of
    decode-fusion/test_exact.py:31-50 (here in double)."""
    from titan_b200 import ops
    L = oracle.make_layer(H=H, E=E, k=10 if E >= 10 else 2, I=I, seed=T)
    x = oracle.make_x(T, H, seed=T)
    k = L.k
    idx, sc, _, _ = oracle.router(x, L.wr, k)
    h = ops.gate_up_silu(bf(x), words(L.gu_w), bf(L.gu_s), bf(L.gu_b), i32(idx))
    # golden h
    gu = oracle.gather_qmm_exact(np.repeat(x, k, axis=0), L.gu_w, L.gu_s, L.gu_b, idx.reshape(-1),
                                 f32=True).astype(np.float64)
    g, u = gu[:, :I], gu[:, I:]
    href = (g / (1 + np.exp(-g)) * u).reshape(T, k, I)
    hg = h.cpu().numpy()
    assert np.allclose(hg, href, rtol=1e-4, atol=1e-5 * np.abs(href).max())
    scf = f32(sc)
    y = ops.down_wsum(h, words(L.dn_w), bf(L.dn_s), bf(L.dn_b), i32(idx), f32t(scf))
    # golden y from the kernel's own h, in double
    deq = oracle.dequant(L.dn_w, L.dn_s, L.dn_b).astype(np.float64)     # [E, H, I]
    yref = np.zeros((T, H))
    for t in range(T):
        for j in range(k):
            yref[t] += scf[t, j] * (deq[idx[t, j]] @ hg[t, j].astype(np.float64))
    assert_bf16_close(nbf(y), oracle.f32_to_bf16(yref.astype(np.float32)), ulps=1, rel=0,
                      what="down_wsum")
