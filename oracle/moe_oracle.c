/*
 * TEST INFRASTRUCTURE ONLY — CPU oracle for the quantised MoE block.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs may load this library, and only as the checker or
 * the timed CPU baseline.  The product (titan_b200) never links it.
 *
 * Parity status: UNPINNED at the value level against the reference.  The
 * reference computes this block through MLX 0.32.2 (mx.gather_qmm,
 * mx.quantize, mx.softmax(precise=True), mx.argpartition), which is neither
 * vendored under the reference tree nor installable here, and the reference
 * stores no golden tensors for this path (every test draws from mx.random).
 * What IS pinned, by the reference's own tests restated in tests/:
 *   - nibble order and packing (tests/kernels/test_moe_gather_int8.py:104-115)
 *   - the affine dequant w = q*s + b (engine/patches/decode-fusion/test_exact.py:19-28)
 *   - the 8-partial bf16 weighted-sum model, bit-identical to MLX's reduce
 *     (titan/kernels/moe_weighted_sum.py:51-98, round2/wsum10/test-20260912.txt)
 *   - the int8 error bar rel-RMS < 0.02 vs the bf16-activation path
 *     (tests/kernels/test_moe_gather_int8.py:28,66-101)
 *   - lowest-index tie rule of the fused router
 *     (engine/patches/decode-fusion/fused_kernels.py:295-307)
 *
 * Where MLX leaves an order or a rounding unspecified (dot-product order of
 * the router Linear, the exp used by softmax/sigmoid, simd_sum order of the
 * quantiser's group sum) this file fixes a CANONICAL order, stated at each
 * function, and the CUDA kernels implement the same order so that routing
 * indices and integer codes compare bit-exactly.
 *
 * All float arithmetic is IEEE binary32 with round-to-nearest-even, explicit
 * fmaf where an FMA is meant; build with -ffp-contract=off, no fast-math.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ bf16 */

static inline float bf2f(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float bits2f(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

int orc_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

void orc_f32_to_bf16(const float* in, uint16_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = f2bf(in[i]);
}

/* ------------------------------------------------------------ canonical exp
 * Cody & Waite range reduction (x = n*ln2 + r, ln2 split hi/lo so n*ln2_hi is
 * exact) followed by the degree-7 Taylor polynomial of e^r on
 * |r| <= ln2/2 (truncation error < 6e-9 relative), scaled by 2^n in two exact
 * power-of-two steps.  The CUDA kernels evaluate the identical sequence of
 * IEEE operations, so softmax, sigmoid and SiLU compare bit-exactly.
 */
float orc_exp(float x) {
    if (x != x) return x;
    if (x > 88.7228393554688f) return INFINITY;
    if (x < -103.972084045410f) return 0.0f;
    float n = rintf(x * 1.44269504088896341f);
    float r = fmaf(-n, 0.693145751953125f, x);
    r = fmaf(-n, 1.42860682030941723e-06f, r);
    float p = 1.98412698412698413e-4f;          /* 1/7! */
    p = fmaf(p, r, 1.38888888888888889e-3f);    /* 1/6! */
    p = fmaf(p, r, 8.33333333333333333e-3f);    /* 1/5! */
    p = fmaf(p, r, 4.16666666666666667e-2f);    /* 1/4! */
    p = fmaf(p, r, 1.66666666666666667e-1f);    /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    int n1 = ni / 2;
    int n2 = ni - n1;
    float s1 = bits2f((uint32_t)(n1 + 127) << 23);
    float s2 = bits2f((uint32_t)(n2 + 127) << 23);
    return (p * s1) * s2;
}

/* sigmoid in fp32: 1 / (1 + e^-x), IEEE divide. */
float orc_sigmoid(float x) { return 1.0f / (1.0f + orc_exp(-x)); }

/* ------------------------------------------------------- canonical bf16 dot
 * Router Linear (qwen3_5_moe/language.py:54,65): bf16 x, bf16 W, fp32
 * accumulate, bf16 result.  Canonical order: 8 partials; the 8-element chunk
 * c (elements 8c..8c+7) goes to partial c mod 8, accumulated with fmaf in
 * ascending c and element order; then the xor tree over offsets 4,2,1:
 * v_p = p_p + p_(p^4); w_p = v_p + v_(p^2); result = w_0 + w_1.
 */
static float dot_canon(const uint16_t* x, const uint16_t* w, int H) {
    float part[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = 0; c * 8 < H; ++c)
        for (int u = 0; u < 8; ++u) {
            int k = c * 8 + u;
            part[c & 7] = fmaf(bf2f(x[k]), bf2f(w[k]), part[c & 7]);
        }
    float v[4], w2[2];
    for (int p = 0; p < 4; ++p) v[p] = part[p] + part[p + 4];
    for (int p = 0; p < 2; ++p) w2[p] = v[p] + v[p + 2];
    return w2[0] + w2[1];
}

/* xor-butterfly sum of 32 lane values over offsets 16,8,4,2,1 (a warp
 * reduction with __shfl_xor): the softmax denominator and the quantiser's
 * group sum use this tree. */
static float butterfly32(float* part) {
    for (int off = 16; off >= 1; off >>= 1) {
        float t[32];
        for (int l = 0; l < 32; ++l) t[l] = part[l] + part[l ^ off];
        memcpy(part, t, sizeof(float) * 32);
    }
    return part[0];
}

/* ------------------------------------------------------------------ router
 * qwen3_5_moe/language.py:65-71:
 *   gates  = bf16(x @ Wr^T)                      (dot_canon, bf16 round)
 *   gates  = softmax(gates, precise=True)        fp32 inside, bf16 out
 *   inds   = top-k of the bf16 probabilities     (argpartition)
 *   scores = take_along_axis(gates, inds); scores / scores.sum()  (bf16)
 * Canonical choices: softmax max is exact; e_i = orc_exp(l_i - max); the sum
 * uses 32 lane partials over e = 32*c + l (c ascending, fadd) and the
 * butterfly; p_i = bf16(e_i * (1/sum)).  Selection is by bf16 value with the
 * LOWEST expert index winning ties (fused_kernels.py:295-307), emitted in
 * selection order (descending value, ascending index).  The renormalising sum
 * is a sequential fp32 sum over the selected k in that order, rounded to
 * bf16; score_j = bf16(p_j / sum_bf16).
 * Outputs: idx [T,k] int32, scores [T,k] bf16; optional logits/probs [T,E].
 */
void orc_router(const uint16_t* x, const uint16_t* wr, int T, int H, int E, int k,
                int32_t* idx, uint16_t* scores, uint16_t* logits_out, uint16_t* probs_out) {
#pragma omp parallel for schedule(dynamic, 4)
    for (int t = 0; t < T; ++t) {
        uint16_t* lg = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)E);
        uint16_t* pb = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)E);
        float* ex = (float*)malloc(sizeof(float) * (size_t)E);
        unsigned char* taken = (unsigned char*)calloc((size_t)E, 1);
        const uint16_t* xt = x + (size_t)t * H;
        for (int e = 0; e < E; ++e) lg[e] = f2bf(dot_canon(xt, wr + (size_t)e * H, H));
        float m = -INFINITY;
        for (int e = 0; e < E; ++e) m = fmaxf(m, bf2f(lg[e]));
        float part[32];
        for (int l = 0; l < 32; ++l) part[l] = 0.0f;
        for (int e = 0; e < E; ++e) {
            ex[e] = orc_exp(bf2f(lg[e]) - m);
            part[e % 32] = part[e % 32] + ex[e];
        }
        float sum = butterfly32(part);
        float inv = 1.0f / sum;
        for (int e = 0; e < E; ++e) pb[e] = f2bf(ex[e] * inv);
        float ssum = 0.0f;
        for (int j = 0; j < k; ++j) {
            int best = -1;
            for (int e = 0; e < E; ++e) {
                if (taken[e]) continue;
                if (best < 0 || pb[e] > pb[best]) best = e; /* p >= 0: bits are monotone */
            }
            taken[best] = 1;
            idx[(size_t)t * k + j] = best;
            ssum = ssum + bf2f(pb[best]);
        }
        float sb = bf2f(f2bf(ssum));
        for (int j = 0; j < k; ++j)
            scores[(size_t)t * k + j] = f2bf(bf2f(pb[idx[(size_t)t * k + j]]) / sb);
        if (logits_out) memcpy(logits_out + (size_t)t * E, lg, sizeof(uint16_t) * (size_t)E);
        if (probs_out) memcpy(probs_out + (size_t)t * E, pb, sizeof(uint16_t) * (size_t)E);
        free(lg); free(pb); free(ex); free(taken);
    }
}

/* ---------------------------------------------------------- routing sort
 * switch_layers.py:13-25 (_gather_sort/_scatter_unsort): order = stable
 * argsort of the flat expert ids, inv_order = argsort(order).  A stable
 * counting sort gives the same permutation.  offsets[e] = first sorted row of
 * expert e, offsets[E] = R (moe_gather_ws.py:133-150).
 */
void orc_sort_routes(const int32_t* idx, int R, int E, int32_t* order, int32_t* inv_order,
                     int32_t* offsets) {
    int32_t* cnt = (int32_t*)calloc((size_t)E + 1, sizeof(int32_t));
    for (int r = 0; r < R; ++r) cnt[idx[r] + 1]++;
    for (int e = 0; e < E; ++e) cnt[e + 1] += cnt[e];
    if (offsets) memcpy(offsets, cnt, sizeof(int32_t) * ((size_t)E + 1));
    for (int r = 0; r < R; ++r) {
        int p = cnt[idx[r]]++;
        order[p] = r;
        inv_order[r] = p;
    }
    free(cnt);
}

/* ----------------------------------------------------- activation quantiser
 * moe_gather_int8.py:132-165 (titan_i8_actquant), per (row m, 64-group g):
 *   sc  = max(amax, 1e-30) / 127          (IEEE divide)
 *   inv = 1 / sc
 *   xu  = clamp(rint(x * inv) + 128, 0, 255)    uint8, zero point 128
 *   xrs = sum of the UNQUANTISED x over the group (fp32)
 *   xav = 65536 - 8 * sum(xu)                    (exact)
 * Canonical xrs order: pair sums v[2l] + v[2l+1] (l = 0..31), then the xor
 * butterfly (the reference's simd_sum over 32 lanes holding 2 values each).
 * Stored codes are the SIGNED xs = xu - 128.
 */
void orc_quantize_act(const uint16_t* x, int R, int K, int8_t* xs, float* xsc, float* xrs,
                      float* xav) {
    const int G = K / 64;
#pragma omp parallel for schedule(static)
    for (int m = 0; m < R; ++m) {
        for (int g = 0; g < G; ++g) {
            const uint16_t* v = x + (size_t)m * K + (size_t)g * 64;
            float amax = 0.0f;
            float part[32];
            for (int l = 0; l < 32; ++l) {
                float a = bf2f(v[2 * l]), b = bf2f(v[2 * l + 1]);
                amax = fmaxf(amax, fmaxf(fabsf(a), fabsf(b)));
                part[l] = a + b;
            }
            float sum = butterfly32(part);
            float sc = fmaxf(amax, 1e-30f) / 127.0f;
            float inv = 1.0f / sc;
            int csum = 0;
            for (int i = 0; i < 64; ++i) {
                float q = rintf(bf2f(v[i]) * inv) + 128.0f;
                q = fminf(fmaxf(q, 0.0f), 255.0f);
                int qi = (int)q;
                csum += qi;
                xs[(size_t)m * K + (size_t)g * 64 + i] = (int8_t)(qi - 128);
            }
            xsc[(size_t)m * G + g] = sc;
            xrs[(size_t)m * G + g] = sum;
            if (xav) xav[(size_t)m * G + g] = 65536.0f - 8.0f * (float)csum;
        }
    }
}

/* ------------------------------------------------------------ weight tables
 * moe_gather_int8.py:189-248 (build_tables): qsum[e,g,n] = sum of the 64
 * nibbles of row n, group g (nibble j of word w is element 8w+j, low nibble
 * first); folded bias table bv = bf16(b + 8 s); both transposed to [E,G,N].
 */
void orc_qsum(const uint32_t* wq, int E, int N, int K, uint16_t* qsum) {
    const int G = K / 64, KW = K / 8;
    for (int e = 0; e < E; ++e)
        for (int n = 0; n < N; ++n)
            for (int g = 0; g < G; ++g) {
                unsigned acc = 0;
                for (int j = 0; j < 8; ++j) {
                    uint32_t v = wq[((size_t)e * N + n) * KW + (size_t)g * 8 + j];
                    for (int t = 0; t < 8; ++t) acc += (v >> (4 * t)) & 0xfu;
                }
                qsum[((size_t)e * G + g) * N + n] = (uint16_t)acc;
            }
}

void orc_prepare_tables(const uint16_t* scales, const uint16_t* biases, int E, int N, int G,
                        uint16_t* scales_t, uint16_t* bfold_t) {
    for (int e = 0; e < E; ++e)
        for (int n = 0; n < N; ++n)
            for (int g = 0; g < G; ++g) {
                size_t src = ((size_t)e * N + n) * G + g;
                size_t dst = ((size_t)e * G + g) * N + n;
                float s = bf2f(scales[src]);
                float b = bf2f(biases[src]);
                scales_t[dst] = scales[src];
                bfold_t[dst] = f2bf(b + 8.0f * s);
            }
}

/* --------------------------------------------------- MLX affine quantiser
 * Third-party algorithm, not under the reference tree: MLX 0.32.2
 * mx.quantize(w, group_size=64, bits=4, mode="affine") (call sites
 * switch_layers.py:42,179; tests/kernels/test_moe_gather_int8.py:31-36).
 * Restated from MLX's published source: per group of 64,
 *   mask  = |min| > |max|
 *   scale = max((max - min) / 15, 1e-7), negated unless mask
 *   edge  = mask ? min : max
 *   q0    = rint(edge / scale);  if q0 != 0: scale = edge / q0, bias = edge
 *                                else bias = 0
 *   q     = clamp(rint((w - bias) / scale), 0, 15), packed 8 per uint32,
 *           element 8w+j in bits 4j..4j+3
 * Scales and biases come out fp32 and are rounded to bf16 (the configs keep
 * bf16 scales/biases).
 */
void orc_affine_quantize(const float* w, int64_t rows, int K, uint32_t* wq, uint16_t* scales,
                         uint16_t* biases) {
    const int G = K / 64, KW = K / 8;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        for (int g = 0; g < G; ++g) {
            const float* v = w + (size_t)r * K + (size_t)g * 64;
            float mn = INFINITY, mx = -INFINITY;
            for (int i = 0; i < 64; ++i) {
                mx = fmaxf(mx, v[i]);
                mn = fminf(mn, v[i]);
            }
            int mask = fabsf(mn) > fabsf(mx);
            float scale = fmaxf((mx - mn) / 15.0f, 1e-7f);
            scale = mask ? scale : -scale;
            float edge = mask ? mn : mx;
            float q0 = rintf(edge / scale);
            float bias = 0.0f;
            if (q0 != 0.0f) {
                scale = edge / q0;
                bias = edge;
            }
            for (int j = 0; j < 8; ++j) {
                uint32_t word = 0;
                for (int t = 0; t < 8; ++t) {
                    float q = rintf((v[j * 8 + t] - bias) / scale);
                    q = fminf(fmaxf(q, 0.0f), 15.0f);
                    word |= ((uint32_t)q) << (4 * t);
                }
                wq[(size_t)r * KW + (size_t)g * 8 + j] = word;
            }
            scales[(size_t)r * G + g] = f2bf(scale);
            biases[(size_t)r * G + g] = f2bf(bias);
        }
    }
}

/* affine dequant in fp32 (decode-fusion/test_exact.py:19-28): w = q*s + b. */
void orc_dequant(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases, int64_t rows,
                 int K, float* out) {
    const int G = K / 64, KW = K / 8;
    for (int64_t r = 0; r < rows; ++r)
        for (int k = 0; k < K; ++k) {
            uint32_t q = (wq[(size_t)r * KW + k / 8] >> (4 * (k % 8))) & 0xfu;
            int g = k / 64;
            out[(size_t)r * K + k] = (float)q * bf2f(scales[(size_t)r * G + g]) +
                                     bf2f(biases[(size_t)r * G + g]);
        }
}

static inline unsigned nib(const uint32_t* row, int k) { return (row[k >> 3] >> (4 * (k & 7))) & 0xfu; }

/* ------------------------------------------------ int8 x int4 sorted gather
 * moe_gather_int8.py:256-349 (titan_moe_i8i4), per sorted row m (expert
 * rhs[m]) and output column n, over groups g:
 *   D   = sum_k xu[m,k] * q[n,k]                 exact int
 *   tt  = D + xav[m,g]
 *   qv  = s * (128 * qsum[n,g])
 *   acc = fma(xsc[m,g], fma(tt, s, -qv), acc);  acc = fma(xrs[m,g], bv, acc)
 * with s = scale, bv = bf16(b + 8 s); output bf16(acc).   (order = 0)
 *
 * order = 1 evaluates the re-centred form the CUDA kernel uses:
 *   D'' = sum_k (xu-128)(q-8) = tt - 128 qsum    exact int
 *   acc = fma(D'' * s, xsc, acc);  acc = fma(xrs, bv, acc)
 * Both are the same real number up to fp32 rounding.
 * x is bf16 [R,K] (rows already in sorted order); y bf16 [R,N].
 */
void orc_gather_qmm_int8(const uint16_t* x, const uint32_t* wq, const uint16_t* scales,
                         const uint16_t* biases, const int32_t* rhs, int R, int N, int K,
                         int order, uint16_t* y) {
    const int G = K / 64, KW = K / 8;
    int8_t* xs = (int8_t*)malloc((size_t)R * K);
    float* xsc = (float*)malloc(sizeof(float) * (size_t)R * G);
    float* xrs = (float*)malloc(sizeof(float) * (size_t)R * G);
    float* xav = (float*)malloc(sizeof(float) * (size_t)R * G);
    orc_quantize_act(x, R, K, xs, xsc, xrs, xav);
#pragma omp parallel for schedule(dynamic, 1)
    for (int m = 0; m < R; ++m) {
        const int e = rhs[m];
        const int8_t* xm = xs + (size_t)m * K;
        for (int n = 0; n < N; ++n) {
            const uint32_t* wr = wq + ((size_t)e * N + n) * KW;
            const uint16_t* sr = scales + ((size_t)e * N + n) * G;
            const uint16_t* br = biases + ((size_t)e * N + n) * G;
            float acc = 0.0f;
            for (int g = 0; g < G; ++g) {
                float s = bf2f(sr[g]);
                float bv = bf2f(f2bf(bf2f(br[g]) + 8.0f * s));
                float sc = xsc[(size_t)m * G + g], rs = xrs[(size_t)m * G + g];
                if (order == 0) {
                    int D = 0, qs = 0;
                    for (int k = g * 64; k < g * 64 + 64; ++k) {
                        int q = (int)nib(wr, k);
                        D += ((int)xm[k] + 128) * q;
                        qs += q;
                    }
                    float tt = (float)D + xav[(size_t)m * G + g];
                    float qv = s * (128.0f * (float)qs);
                    acc = fmaf(sc, fmaf(tt, s, -qv), acc);
                    acc = fmaf(rs, bv, acc);
                } else {
                    int Dpp = 0;
                    for (int k = g * 64; k < g * 64 + 64; ++k)
                        Dpp += (int)xm[k] * ((int)nib(wr, k) - 8);
                    float t1 = (float)Dpp * s;
                    acc = fmaf(t1, sc, acc);
                    acc = fmaf(rs, bv, acc);
                }
            }
            y[(size_t)m * N + n] = f2bf(acc);
        }
    }
    free(xs); free(xsc); free(xrs); free(xav);
}

/* ----------------------------------------------- bf16-activation gather
 * The stock mx.gather_qmm (switch_layers.py:86-98): bf16 x times the exactly
 * dequantised int4 weights, accumulated in double here (the exact ruler of
 * decode-fusion/test_exact.py:31-50), rounded to fp32 and then to bf16 unless
 * y_f32 is requested.  rhs may be NULL (expert 0 for every row, i.e. a dense
 * quantised Linear such as the shared expert).
 */
void orc_gather_qmm_exact(const uint16_t* x, const uint32_t* wq, const uint16_t* scales,
                          const uint16_t* biases, const int32_t* rhs, int R, int N, int K,
                          uint16_t* y_bf16, float* y_f32) {
    const int G = K / 64, KW = K / 8;
#pragma omp parallel for schedule(dynamic, 1)
    for (int m = 0; m < R; ++m) {
        const int e = rhs ? rhs[m] : 0;
        const uint16_t* xm = x + (size_t)m * K;
        for (int n = 0; n < N; ++n) {
            const uint32_t* wr = wq + ((size_t)e * N + n) * KW;
            const uint16_t* sr = scales + ((size_t)e * N + n) * G;
            const uint16_t* br = biases + ((size_t)e * N + n) * G;
            double acc = 0.0;
            for (int g = 0; g < G; ++g) {
                double s = bf2f(sr[g]), b = bf2f(br[g]);
                double dq = 0.0, dx = 0.0;
                for (int k = g * 64; k < g * 64 + 64; ++k) {
                    double xv = bf2f(xm[k]);
                    dq += xv * (double)nib(wr, k);
                    dx += xv;
                }
                acc += s * dq + b * dx;
            }
            if (y_f32) y_f32[(size_t)m * N + n] = (float)acc;
            if (y_bf16) y_bf16[(size_t)m * N + n] = f2bf((float)acc);
        }
    }
}

/* fp32-input variant (h kept in fp32 on the decode path); rows split over
 * threads when par != 0. */
static void gather_exact_f32in(const float* x, const uint32_t* wq, const uint16_t* scales,
                               const uint16_t* biases, int e, int N, int K, double* y, int par) {
    const int G = K / 64, KW = K / 8;
#pragma omp parallel for schedule(static) if (par)
    for (int n = 0; n < N; ++n) {
        const uint32_t* wr = wq + ((size_t)e * N + n) * KW;
        const uint16_t* sr = scales + ((size_t)e * N + n) * G;
        const uint16_t* br = biases + ((size_t)e * N + n) * G;
        double acc = 0.0;
        for (int g = 0; g < G; ++g) {
            double s = bf2f(sr[g]), b = bf2f(br[g]);
            double dq = 0.0, dx = 0.0;
            for (int k = g * 64; k < g * 64 + 64; ++k) {
                dq += (double)x[k] * (double)nib(wr, k);
                dx += (double)x[k];
            }
            acc += s * dq + b * dx;
        }
        y[n] = acc;
    }
}

/* ------------------------------------------------------------------ SwiGLU
 * activations.py:9-11, switch_layers.py:229-237: gate = cols [0,I), up =
 * cols [I,2I); h = silu(gate) * up with bf16 rounding after each op:
 *   sg = bf16(sigmoid(g)); a = bf16(g * sg); h = bf16(a * u).
 */
static inline uint16_t swiglu_bf16(uint16_t g, uint16_t u) {
    float gf = bf2f(g);
    float sg = bf2f(f2bf(orc_sigmoid(gf)));
    float a = bf2f(f2bf(gf * sg));
    return f2bf(a * bf2f(u));
}

void orc_swiglu(const uint16_t* gu, int R, int I, uint16_t* h) {
    for (int r = 0; r < R; ++r)
        for (int i = 0; i < I; ++i)
            h[(size_t)r * I + i] = swiglu_bf16(gu[(size_t)r * 2 * I + i], gu[(size_t)r * 2 * I + I + i]);
}

/* ------------------------------------------------------------ weighted sum
 * moe_weighted_sum.py:51-98, clone mode (default): for output (t, d),
 * prod_j = bf16(score[t,j] * ys[inv[t*k+j], d]); acc[j%8] = bf16(acc[j%8] + prod_j);
 * result = bf16 sequential combine of acc[0..7].  mode 1 ("fast"): fp32
 * products and eight fp32 partials, combined in fp32, one final rounding.
 * inv may be NULL (token-major layout).
 */
void orc_weighted_sum(const uint16_t* ys, const int32_t* inv, const uint16_t* scores, int T, int k,
                      int D, int mode, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        for (int d = 0; d < D; ++d) {
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int j = 0; j < k; ++j) {
                int p = t * k + j;
                int src = inv ? inv[p] : p;
                float s = bf2f(scores[p]);
                float prod = s * bf2f(ys[(size_t)src * D + d]);
                if (mode == 0) prod = bf2f(f2bf(prod));
                float tt = acc[j % 8] + prod;
                acc[j % 8] = (mode == 0) ? bf2f(f2bf(tt)) : tt;
            }
            float a = acc[0];
            for (int j = 1; j < 8; ++j) {
                a = a + acc[j];
                if (mode == 0) a = bf2f(f2bf(a));
            }
            out[(size_t)t * D + d] = f2bf(a);
        }
    }
}

/* ------------------------------------------------------------ whole block
 * Qwen3_5MoeSparseMoeBlock.__call__ (qwen3_5_moe/language.py:60-91) with the
 * int8 overlay installed (engine/patches/moe-int8/patch.py:105-122):
 *   route -> sort -> gate_up (int8) -> SwiGLU -> down (int8 or bf16) ->
 *   unsort + weighted sum (clone) -> + sigmoid(x wg) * shared(x)
 * Shared expert (qwen3_5/language.py:1590-1601) is the stock bf16-activation
 * quantised MLP; its gate logit uses dot_canon and is rounded to bf16, then
 * sigmoid -> bf16, product -> bf16, final add -> bf16.
 * shared weights may be NULL (no shared expert).  down_int8 = 0 keeps the
 * down projection on the bf16-activation path (OMLX_MOE_INT8_SKIP_DOWN=1).
 * Optional outputs: idx/scores for the routing check.
 */
typedef struct {
    int T, H, E, k, I, Is;
    const uint16_t* wr;                                  /* [E,H] */
    const uint32_t* gu_w; const uint16_t* gu_s; const uint16_t* gu_b;  /* [E,2I,*] */
    const uint32_t* dn_w; const uint16_t* dn_s; const uint16_t* dn_b;  /* [E,H,*]  */
    const uint32_t* sgu_w; const uint16_t* sgu_s; const uint16_t* sgu_b; /* [2Is,H/8..] */
    const uint32_t* sdn_w; const uint16_t* sdn_s; const uint16_t* sdn_b; /* [H,Is/8..] */
    const uint16_t* wg;                                  /* [H] shared gate */
} orc_moe_desc;

static void shared_prefill(const orc_moe_desc* d, const uint16_t* x, uint16_t* sh) {
    const int T = d->T, H = d->H, Is = d->Is;
    uint16_t* gu = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * 2 * Is);
    uint16_t* hs = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * Is);
    uint16_t* ys = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * H);
    orc_gather_qmm_exact(x, d->sgu_w, d->sgu_s, d->sgu_b, NULL, T, 2 * Is, H, gu, NULL);
    orc_swiglu(gu, T, Is, hs);
    orc_gather_qmm_exact(hs, d->sdn_w, d->sdn_s, d->sdn_b, NULL, T, H, Is, ys, NULL);
    for (int t = 0; t < T; ++t) {
        float gl = bf2f(f2bf(dot_canon(x + (size_t)t * H, d->wg, H)));
        float sg = bf2f(f2bf(orc_sigmoid(gl)));
        for (int c = 0; c < H; ++c)
            sh[(size_t)t * H + c] = f2bf(sg * bf2f(ys[(size_t)t * H + c]));
    }
    free(gu); free(hs); free(ys);
}

/* int8_mode: 0 = stock (bf16 activations everywhere, no overlay installed),
 * 1 = int8 gate_up only (OMLX_MOE_INT8_SKIP_DOWN=1), 3 = int8 gate_up and
 * down (the overlay's default).  Adding 4 evaluates the int8 gathers in the
 * re-centred order (order = 1 of orc_gather_qmm_int8) instead of the
 * reference's FMA order. */
/* Optional capture of the two operands of the final bf16 add (routed sum and
 * gated shared term), for tests that count ULPs where that add cancels. */
static uint16_t* g_routed_out = NULL;
static uint16_t* g_shared_out = NULL;
static uint16_t* g_termmax_out = NULL;  /* max_j |bf16(score_j * Y_j)| per output */

void orc_set_parts_out(uint16_t* routed, uint16_t* shared, uint16_t* termmax) {
    g_routed_out = routed;
    g_shared_out = shared;
    g_termmax_out = termmax;
}

void orc_moe_prefill(const orc_moe_desc* d, const uint16_t* x, int int8_mode, int32_t* idx_out,
                     uint16_t* scores_out, uint16_t* y) {
    const int gate_up_int8 = int8_mode & 1, down_int8 = (int8_mode & 2) != 0;
    const int qorder = (int8_mode & 4) ? 1 : 0;
    const int T = d->T, H = d->H, E = d->E, k = d->k, I = d->I, R = T * k;
    int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * (size_t)R);
    uint16_t* sc = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)R);
    orc_router(x, d->wr, T, H, E, k, idx, sc, NULL, NULL);
    int32_t* order = (int32_t*)malloc(sizeof(int32_t) * (size_t)R);
    int32_t* inv = (int32_t*)malloc(sizeof(int32_t) * (size_t)R);
    int32_t* srt = (int32_t*)malloc(sizeof(int32_t) * (size_t)R);
    orc_sort_routes(idx, R, E, order, inv, NULL);
    uint16_t* xsrt = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)R * H);
    for (int r = 0; r < R; ++r) {
        srt[r] = idx[order[r]];
        memcpy(xsrt + (size_t)r * H, x + (size_t)(order[r] / k) * H, sizeof(uint16_t) * (size_t)H);
    }
    uint16_t* gu = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)R * 2 * I);
    if (gate_up_int8)
        orc_gather_qmm_int8(xsrt, d->gu_w, d->gu_s, d->gu_b, srt, R, 2 * I, H, qorder, gu);
    else
        orc_gather_qmm_exact(xsrt, d->gu_w, d->gu_s, d->gu_b, srt, R, 2 * I, H, gu, NULL);
    free(xsrt);
    uint16_t* h = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)R * I);
    orc_swiglu(gu, R, I, h);
    free(gu);
    uint16_t* ys = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)R * H);
    if (down_int8)
        orc_gather_qmm_int8(h, d->dn_w, d->dn_s, d->dn_b, srt, R, H, I, qorder, ys);
    else
        orc_gather_qmm_exact(h, d->dn_w, d->dn_s, d->dn_b, srt, R, H, I, ys, NULL);
    free(h);
    orc_weighted_sum(ys, inv, sc, T, k, H, 0, y);
    if (g_termmax_out)
        for (int t = 0; t < T; ++t)
            for (int c = 0; c < H; ++c) {
                float m = 0.0f;
                for (int j = 0; j < k; ++j) {
                    int p = t * k + j;
                    float v = fabsf(bf2f(f2bf(bf2f(sc[p]) * bf2f(ys[(size_t)inv[p] * H + c]))));
                    m = fmaxf(m, v);
                }
                g_termmax_out[(size_t)t * H + c] = f2bf(m);
            }
    free(ys);
    if (g_routed_out) memcpy(g_routed_out, y, sizeof(uint16_t) * (size_t)T * H);
    if (d->Is > 0 && d->sgu_w) {
        uint16_t* sh = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * H);
        shared_prefill(d, x, sh);
        for (size_t i = 0; i < (size_t)T * H; ++i) y[i] = f2bf(bf2f(y[i]) + bf2f(sh[i]));
        if (g_shared_out) memcpy(g_shared_out, sh, sizeof(uint16_t) * (size_t)T * H);
        free(sh);
    }
    if (idx_out) memcpy(idx_out, idx, sizeof(int32_t) * (size_t)R);
    if (scores_out) memcpy(scores_out, sc, sizeof(uint16_t) * (size_t)R);
    free(idx); free(sc); free(order); free(inv); free(srt);
}

/* Decode semantics (engine/patches/decode-fusion/fused_kernels.py:31-169 and
 * its fp32 golden, test_exact.py:31-50): fp32 gate/up, h = silu(g)*u kept in
 * fp32, y = sum_j score_j * (Wd h_j) + sigmoid(x wg) * shared(x), rounded to
 * bf16 once.  The oracle evaluates the sums in double (the exact ruler).
 * Routing is the same canonical router as the prefill path.
 */
void orc_moe_decode(const orc_moe_desc* d, const uint16_t* x, int32_t* idx_out,
                    uint16_t* scores_out, uint16_t* y) {
    const int T = d->T, H = d->H, E = d->E, k = d->k, I = d->I, Is = d->Is;
    int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * (size_t)T * k);
    uint16_t* sc = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * k);
    orc_router(x, d->wr, T, H, E, k, idx, sc, NULL, NULL);
    const int outer = T >= orc_threads();
#pragma omp parallel for schedule(dynamic, 1) if (outer)
    for (int t = 0; t < T; ++t) {
        int Imax = I > Is ? I : Is;
        float* xf = (float*)malloc(sizeof(float) * (size_t)H);
        double* gu = (double*)malloc(sizeof(double) * 2 * (size_t)Imax);
        float* hf = (float*)malloc(sizeof(float) * (size_t)Imax);
        double* yd = (double*)calloc((size_t)H, sizeof(double));
        double* tmp = (double*)malloc(sizeof(double) * (size_t)H);
        for (int c = 0; c < H; ++c) xf[c] = bf2f(x[(size_t)t * H + c]);
        for (int j = 0; j < k; ++j) {
            int e = idx[(size_t)t * k + j];
            double s = bf2f(sc[(size_t)t * k + j]);
            gather_exact_f32in(xf, d->gu_w, d->gu_s, d->gu_b, e, 2 * I, H, gu, !outer);
            for (int i = 0; i < I; ++i) {
                double g = (float)gu[i], u = (float)gu[I + i];
                hf[i] = (float)(g / (1.0 + exp(-g)) * u);
            }
            gather_exact_f32in(hf, d->dn_w, d->dn_s, d->dn_b, e, H, I, tmp, !outer);
            for (int c = 0; c < H; ++c) yd[c] += s * tmp[c];
        }
        if (Is > 0 && d->sgu_w) {
            gather_exact_f32in(xf, d->sgu_w, d->sgu_s, d->sgu_b, 0, 2 * Is, H, gu, !outer);
            for (int i = 0; i < Is; ++i) {
                double g = (float)gu[i], u = (float)gu[Is + i];
                hf[i] = (float)(g / (1.0 + exp(-g)) * u);
            }
            gather_exact_f32in(hf, d->sdn_w, d->sdn_s, d->sdn_b, 0, H, Is, tmp, !outer);
            double gl = 0.0;
            for (int c = 0; c < H; ++c) gl += (double)xf[c] * (double)bf2f(d->wg[c]);
            double sg = 1.0 / (1.0 + exp(-gl));
            for (int c = 0; c < H; ++c) yd[c] += sg * tmp[c];
        }
        for (int c = 0; c < H; ++c) y[(size_t)t * H + c] = f2bf((float)yd[c]);
        free(xf); free(gu); free(hf); free(yd); free(tmp);
    }
    if (idx_out) memcpy(idx_out, idx, sizeof(int32_t) * (size_t)T * k);
    if (scores_out) memcpy(scores_out, sc, sizeof(uint16_t) * (size_t)T * k);
    free(idx); free(sc);
}

/* ------------------------------------------- the steps either side of the block
 * RMSNorm (qwen3_5_moe/language.py:103-107, 137): lane partials over
 * e = 32c + l (fma, c ascending), the xor butterfly; ms = sum / H;
 * r = 1 / sqrt(ms + eps); out = bf16((x * r) * w).  Residual write-back:
 * n = 0: out = bf16(branch + residual); n > 0 (hyper-connection inject,
 * qwen4_exp/language.py:3198-3218): out[t, j] = bf16(residual[t, j] +
 * bf16(branch[t] * w[t, j])). */
void orc_rmsnorm(const uint16_t* x, const uint16_t* w, int T, int H, float eps, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const uint16_t* xr = x + (size_t)t * H;
        float part[32];
        for (int l = 0; l < 32; ++l) {
            float s = 0.0f;
            for (int e = l; e < H; e += 32) {
                float v = bf2f(xr[e]);
                s = fmaf(v, v, s);
            }
            part[l] = s;
        }
        float s = butterfly32(part);
        float ms = s / (float)H;
        float r = 1.0f / sqrtf(ms + eps);
        for (int e = 0; e < H; ++e) out[(size_t)t * H + e] = f2bf((bf2f(xr[e]) * r) * bf2f(w[e]));
    }
}

void orc_inject(const uint16_t* branch, const uint16_t* res, const uint16_t* wts, int T, int H,
                int n, uint16_t* out) {
    int ns = n > 0 ? n : 1;
    for (int t = 0; t < T; ++t)
        for (int j = 0; j < ns; ++j)
            for (int c = 0; c < H; ++c) {
                size_t i = ((size_t)t * ns + j) * H + c;
                float b = bf2f(branch[(size_t)t * H + c]);
                float p = n > 0 ? bf2f(f2bf(b * bf2f(wts[(size_t)t * n + j]))) : b;
                out[i] = f2bf(p + bf2f(res[i]));
            }
}
