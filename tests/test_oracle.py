"""The CPU oracle pinned against what the reference's own tests establish.

The reference stores no golden tensors for this path (its tests draw from
mx.random under a seed, and MLX cannot run here), so the oracle is pinned by
restating each of the reference's structural tests and known answers:

  * nibble order / packing     tests/kernels/test_moe_gather_int8.py:104-115
  * dequant w = q*s + b        engine/patches/decode-fusion/test_exact.py:19-28
  * int8 error bar (rel-RMS < 0.02 vs the bf16 path, not growing with K,
    immune to large biases)    tests/kernels/test_moe_gather_int8.py:28,66-101
  * int8 algebra (re-centred nibble, exact integer correction)
                               engine/patches/moe-int8/REPORT.md:66-97
  * clone weighted sum = 8 bf16 partials      titan/kernels/moe_weighted_sum.py:51-98
  * router tie rule: lowest index             fused_kernels.py:295-307
  * stable sort                               switch_layers.py:13-18
plus independent numpy restatements of the canonical orders.
"""
import math

import numpy as np
import pytest

from helpers import f32, rel_rms, ulp_bf16


def test_exp_matches_math_exp(oracle):
    xs = np.concatenate([np.linspace(-87, 88, 4001), np.linspace(-1, 1, 2001)])
    for v in xs:
        got = oracle.exp(float(v))
        ref = math.exp(float(np.float32(v)))
        assert abs(got - ref) <= 3e-7 * ref, (v, got, ref)
    assert oracle.exp(-200.0) == 0.0
    assert math.isinf(oracle.exp(100.0))


def _host_nibbles(wq):
    packed = np.ascontiguousarray(wq).view(np.uint32)
    return np.stack([(packed >> (4 * t)) & 0xF for t in range(8)], axis=-1)


def test_qsum_matches_a_host_nibble_count(oracle):
    """tests/kernels/test_moe_gather_int8.py:104-115, restated."""
    rng = np.random.default_rng(0)
    w = rng.standard_normal((4, 128, 256), dtype=np.float32)
    wq, s, b = oracle.affine_quantize(w)
    got = oracle.qsum(wq).astype(np.int64)                     # [E, G, N]
    nib = _host_nibbles(wq)                                    # [E, N, K/8, 8]
    e, n, words, _ = nib.shape
    host = nib.reshape(e, n, words // 8, 64).sum(axis=-1)      # [E, N, G]
    assert np.array_equal(got, host.transpose(0, 2, 1))


def test_dequant_is_q_times_s_plus_b_low_nibble_first(oracle):
    """decode-fusion/test_exact.py:19-28 (deq32), restated in numpy."""
    rng = np.random.default_rng(1)
    w = rng.standard_normal((3, 64, 256), dtype=np.float32) * 0.02
    wq, s, b = oracle.affine_quantize(w)
    nib = _host_nibbles(wq).reshape(3, 64, 256).astype(np.float32)
    g = np.repeat(np.arange(256 // 64), 64)
    host = nib * f32(s)[:, :, g] + f32(b)[:, :, g]
    assert np.array_equal(oracle.dequant(wq, s, b), host)


def test_affine_quantiser_known_answer(oracle):
    """One hand-checked group: values 0..63 scaled so max-min = 15*0.1 -> the
    positive edge is the larger magnitude, scale = -(1.5)/15 rescaled to
    edge/q0, bias = edge, codes count down from 15."""
    v = (np.arange(64, dtype=np.float32) % 16) * np.float32(0.1)
    wq, s, b = oracle.affine_quantize(v[None, :])
    scale, bias = f32(s)[0, 0], f32(b)[0, 0]
    assert bias == f32(oracle.f32_to_bf16(np.float32(1.5)))
    assert scale < 0
    codes = _host_nibbles(wq).reshape(-1)
    assert codes.max() <= 15 and codes.min() >= 0
    deq = codes * scale + bias
    assert np.abs(deq - v).max() <= abs(scale) * 0.51 + 1e-6


def test_affine_quantiser_zero_is_exact_and_error_bounded(oracle):
    rng = np.random.default_rng(2)
    w = rng.standard_normal((64, 512), dtype=np.float32) * 0.02
    w[:, 3] = 0.0
    wq, s, b = oracle.affine_quantize(w)
    deq = oracle.dequant(wq, s, b)
    sc = np.repeat(np.abs(f32(s)), 64, axis=1)
    # bf16 rounding of the scale/bias adds a little on top of half a step
    assert np.all(np.abs(deq - w) <= 0.5 * sc * 1.05 + 16 * ulp_bf16(np.abs(w).max()))
    assert np.abs(deq[:, 3]).max() <= 2 * ulp_bf16(np.repeat(f32(b), 64, axis=1)[:, 3]).max()


# ------------------------------------------------------------------- router

def _np_router(x, wr, k):
    """Independent numpy restatement of the canonical router."""
    T, H = x.shape
    E = wr.shape[0]
    xf, wf = f32(x), f32(wr)
    idx = np.zeros((T, k), np.int64)
    sc = np.zeros((T, k), np.uint16)
    for t in range(T):
        lg = np.zeros(E, np.float32)
        for e in range(E):
            part = np.zeros(8, np.float32)
            for c in range(H // 8):
                for u in range(8):
                    kk = c * 8 + u
                    part[c % 8] = _fma32(xf[t, kk], wf[e, kk], part[c % 8])
            v = part[:4] + part[4:]
            w2 = v[:2] + v[2:]
            lg[e] = f32(np.array([_bf(w2[0] + w2[1])]))[0]
        m = lg.max()
        return_probs = None
        ex = np.array([_exp_canon(np.float32(l - m)) for l in lg], np.float32)
        lanes = np.zeros(32, np.float32)
        for e in range(E):
            lanes[e % 32] = np.float32(lanes[e % 32] + ex[e])
        for off in (16, 8, 4, 2, 1):
            lanes = np.array([np.float32(lanes[l] + lanes[l ^ off]) for l in range(32)], np.float32)
        inv = np.float32(np.float32(1.0) / lanes[0])
        pb = np.array([_bf(np.float32(a * inv)) for a in ex], np.uint16)
        order = sorted(range(E), key=lambda e: (-int(pb[e]), e))[:k]
        idx[t] = order
        ssum = np.float32(0)
        for e in order:
            ssum = np.float32(ssum + f32(np.array([pb[e]]))[0])
        sb = f32(np.array([_bf(ssum)]))[0]
        sc[t] = [_bf(np.float32(f32(np.array([pb[e]]))[0] / sb)) for e in order]
        del return_probs
    return idx, sc


def _fma32(a, b, c):
    """fp32 fma emulated in float64: the product of two fp32 values is exact
    in float64; the sum is rounded twice (float64 then fp32), which differs
    from a single rounding only at exact float32 midpoints."""
    return np.float32(float(np.float32(a)) * float(np.float32(b)) + float(np.float32(c)))


def _bf(v):
    u = np.array([v], np.float32).view(np.uint32)[0].astype(np.uint64)
    return np.uint16((u + 0x7FFF + ((u >> 16) & 1)) >> 16)


def _exp_canon(x):
    """numpy mirror of the canonical exp (fp32 ops through float64 fma)."""
    x = np.float32(x)
    if x < np.float32(-103.972084045410):
        return np.float32(0)
    n = np.float32(np.rint(np.float32(x * np.float32(1.44269504088896341))))
    fma = _fma32
    r = fma(-n, np.float32(0.693145751953125), x)
    r = fma(-n, np.float32(1.42860682030941723e-06), r)
    p = np.float32(1.98412698412698413e-4)
    for c in (1.38888888888888889e-3, 8.33333333333333333e-3, 4.16666666666666667e-2,
              1.66666666666666667e-1, 0.5, 1.0, 1.0):
        p = fma(p, r, np.float32(c))
    ni = int(n)
    n1 = int(ni / 2)
    n2 = ni - n1
    return np.float32(np.float32(p * np.float32(2.0 ** n1)) * np.float32(2.0 ** n2))


def test_router_matches_numpy_restatement(oracle):
    x = oracle.make_x(3, 128, seed=5)
    rng = np.random.default_rng(5)
    wr = oracle.f32_to_bf16(rng.standard_normal((64, 128), dtype=np.float32) * 0.02)
    idx, sc, _, _ = oracle.router(x, wr, 6)
    nidx, nsc = _np_router(x, wr, 6)
    assert np.array_equal(idx, nidx) and np.array_equal(sc, nsc)


def test_exp_numpy_mirror_bitexact(oracle):
    for v in np.linspace(-30, 5, 701).astype(np.float32):
        assert np.float32(oracle.exp(float(v))) == _exp_canon(v), v


def test_router_tie_rule_lowest_index(oracle):
    """Equal bf16 probabilities: the lowest expert index is selected first
    (fused_kernels.py:295-307); output is in selection order."""
    H, E, k = 64, 32, 4
    x = oracle.f32_to_bf16(np.ones((1, H), np.float32))
    w = np.zeros((E, H), np.float32)
    w[[3, 9, 20, 21, 30], :] = 1.0 / H       # five equal top logits
    w[[1], :] = 0.5 / H
    idx, sc, lg, pb = oracle.router(x, oracle.f32_to_bf16(w), k)
    assert idx[0].tolist() == [3, 9, 20, 21]
    assert len(set(sc[0].tolist())) == 1       # equal renormalised scores
    assert pb[0, 3] == pb[0, 30]


def test_router_scores_renormalised(oracle):
    x = oracle.make_x(8, 256, seed=1)
    rng = np.random.default_rng(1)
    wr = oracle.f32_to_bf16(rng.standard_normal((128, 256), dtype=np.float32) * 0.02)
    idx, sc, lg, pb = oracle.router(x, wr, 10)
    s = f32(sc).sum(axis=1)
    assert np.all(np.abs(s - 1) < 0.02)
    # selected probabilities are the top-k of the bf16 probabilities
    p = f32(pb)
    for t in range(8):
        kth = np.sort(p[t])[::-1][9]
        assert np.all(p[t, idx[t]] >= kth)
        assert np.all(np.diff(p[t, idx[t]]) <= 0)


def test_sort_routes_is_stable_argsort(oracle):
    rng = np.random.default_rng(3)
    ids = rng.integers(0, 50, size=4000).astype(np.int32)
    order, inv, off = oracle.sort_routes(ids, 50)
    assert np.array_equal(order, np.argsort(ids, kind="stable"))
    assert np.array_equal(inv[order], np.arange(4000))
    assert np.array_equal(off, np.concatenate([[0], np.cumsum(np.bincount(ids, minlength=50))]))


# ------------------------------------------------------- activation quantiser

def test_activation_quantiser(oracle):
    x = oracle.make_x(16, 512, seed=2)
    xs, xsc, xrs, xav = oracle.quantize_act(x)
    xf = f32(x).reshape(16, 8, 64)
    amax = np.abs(xf).max(axis=-1)
    assert np.array_equal(xsc, np.maximum(amax, 1e-30).astype(np.float32) / np.float32(127))
    assert xs.min() >= -128 and xs.max() <= 127
    rec = xs.reshape(16, 8, 64).astype(np.float32) * xsc[..., None]
    assert np.all(np.abs(rec - xf) <= xsc[..., None] * 0.5 * 1.0001)
    # group sum: canonical pair + butterfly order, equal to the exact sum to fp32 rounding
    assert np.allclose(xrs, xf.astype(np.float64).sum(-1), rtol=1e-6, atol=1e-6)
    # xav = 65536 - 8 * sum(xu)
    xu = xs.reshape(16, 8, 64).astype(np.int64) + 128
    assert np.array_equal(xav, (65536 - 8 * xu.sum(-1)).astype(np.float32))


def test_int8_recentred_identity(oracle):
    """sum (xu-128)(q-8) == D + av - 128*qsum, exactly (REPORT.md:66-97)."""
    rng = np.random.default_rng(4)
    xu = rng.integers(0, 256, size=(32, 64))
    q = rng.integers(0, 16, size=(48, 64))
    D = xu @ q.T
    av = 65536 - 8 * xu.sum(1)
    qs = q.sum(1)
    lhs = (xu - 128) @ (q - 8).T
    assert np.array_equal(lhs, D + av[:, None] - 128 * qs[None, :])


# --------------------------------------------------------- int8 gather bars

def _gather_case(oracle, rows, experts, n, k, seed=0, bias_shift=0.0):
    rng = np.random.default_rng(seed)
    dense = rng.standard_normal((experts, n, k), dtype=np.float32) + np.float32(bias_shift)
    wq, s, b = oracle.affine_quantize(dense)
    p = 1.0 / np.arange(1, experts + 1)
    ids = np.sort(rng.choice(experts, size=rows, p=p / p.sum())).astype(np.int32)
    x = oracle.make_x(rows, k, seed=seed + 7)
    ref = oracle.gather_qmm_exact(x, wq, s, b, ids)
    got = oracle.gather_qmm_int8(x, wq, s, b, ids)
    return got, ref, (x, wq, s, b, ids)


@pytest.mark.parametrize("rows,experts,n,k", [(64, 8, 256, 256), (128, 8, 256, 512)])
def test_int8_rel_rms_within_quantisation_floor(oracle, rows, experts, n, k):
    got, ref, _ = _gather_case(oracle, rows, experts, n, k)
    assert rel_rms(f32(got), f32(ref)) < 0.02


@pytest.mark.slow
def test_int8_rel_rms_real_shape(oracle):
    got, ref, _ = _gather_case(oracle, 512, 32, 1280, 2560)
    assert rel_rms(f32(got), f32(ref)) < 0.02


def test_int8_error_does_not_grow_with_k(oracle):
    errs = [rel_rms(*map(f32, _gather_case(oracle, 64, 8, 256, k)[:2])) for k in (256, 1024, 4096)]
    assert all(e < 0.02 for e in errs)
    assert errs[-1] < 3 * errs[0] + 1e-4, errs


def test_int8_large_biases_do_not_degrade_it(oracle):
    got, ref, _ = _gather_case(oracle, 64, 8, 256, 256, seed=3, bias_shift=20.0)
    assert rel_rms(f32(got), f32(ref)) < 0.02


def test_int8_reference_order_vs_recentred_order(oracle):
    """Both FMA orders evaluate the same real number; they differ only in fp32
    rounding, i.e. almost never in the bf16 result."""
    _, _, (x, wq, s, b, ids) = _gather_case(oracle, 64, 8, 256, 512, seed=6)
    a = oracle.gather_qmm_int8(x, wq, s, b, ids, order=0)
    c = oracle.gather_qmm_int8(x, wq, s, b, ids, order=1)
    d = np.abs(f32(a) - f32(c))
    assert np.all(d <= ulp_bf16(f32(a)) + 1e-12)
    assert (d > 0).mean() < 0.01


# --------------------------------------------------------------- weighted sum

def _np_wsum_clone(ys, inv, scores):
    T, k = scores.shape
    D = ys.shape[1]
    out = np.zeros((T, D), np.uint16)
    for t in range(T):
        acc = np.zeros((8, D), np.float32)
        for j in range(k):
            src = inv[t * k + j] if inv is not None else t * k + j
            prod = f32(oracle_bf(f32(scores[t, j:j + 1])[0] * f32(ys[src])))
            acc[j % 8] = f32(oracle_bf(acc[j % 8] + prod))
        a = acc[0]
        for j in range(1, 8):
            a = f32(oracle_bf(a + acc[j]))
        out[t] = oracle_bf(a)
    return out


def oracle_bf(v):
    u = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("T,D,k", [(1, 256, 10), (9, 256, 10), (13, 512, 10), (32, 512, 8)])
def test_weighted_sum_clone_matches_8_partial_model(oracle, T, D, k):
    rng = np.random.default_rng(T)
    ys = oracle.f32_to_bf16(rng.standard_normal((T * k, D), dtype=np.float32))
    sc = rng.uniform(size=(T, k)).astype(np.float32)
    sc = oracle.f32_to_bf16(sc / sc.sum(1, keepdims=True))
    inv = rng.permutation(T * k).astype(np.int32)
    got = oracle.weighted_sum(ys, inv, sc, mode=0)
    assert np.array_equal(got, _np_wsum_clone(ys, inv, sc))
    # fast mode: fp32 throughout, within one bf16 rounding of the exact sum
    fast = oracle.weighted_sum(ys, inv, sc, mode=1)
    exact = np.einsum("tj,tjd->td", f32(sc).astype(np.float64),
                      f32(ys)[inv].reshape(T, k, D).astype(np.float64))
    assert np.all(np.abs(f32(fast) - exact) <= ulp_bf16(exact) + 1e-6)


def test_weighted_sum_clone_known_answer(oracle):
    """A case where bf16 partial accumulation differs from fp32: ten equal
    products of 1/3 into slots 0..7, 0, 1."""
    one_third = oracle.f32_to_bf16(np.full((10, 8), 1.0 / 3.0, np.float32))
    sc = oracle.f32_to_bf16(np.ones((1, 10), np.float32))
    got = f32(oracle.weighted_sum(one_third, None, sc, mode=0))[0, 0]
    p = f32(oracle.f32_to_bf16(np.float32(1.0 / 3.0)))
    acc = [p] * 8
    acc[0] = f32(oracle_bf(np.float32(p + p)))
    acc[1] = acc[0]
    a = acc[0]
    for j in range(1, 8):
        a = f32(oracle_bf(np.float32(a + acc[j])))
    assert got == a


# --------------------------------------------------------------- whole block

def test_block_int8_close_to_fp32_semantics(oracle):
    L = oracle.make_layer(H=256, E=16, k=4, I=128, Is=128, seed=0)
    x = oracle.make_x(32, 256, seed=0)
    y8, i8, s8 = oracle.moe_prefill(L, x, int8_mode=3)
    y0, i0, s0 = oracle.moe_prefill(L, x, int8_mode=0)
    yd, idd, sd = oracle.moe_decode(L, x)
    assert np.array_equal(i8, idd) and np.array_equal(s8, sd) and np.array_equal(i0, i8)
    assert rel_rms(f32(y0), f32(yd)) < 0.01       # stock bf16 intermediates vs fp32
    assert rel_rms(f32(y8), f32(yd)) < 0.03       # int8 gate_up + down (REPORT: 1.41 %)
