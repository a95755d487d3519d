// Register-fragment helpers shared by the decode kernels (sm_100a):
// m16n8k16 fp16 MMAs on exact integer weights, the nibble unpacking that
// feeds them, the permuted activation layout that matches it, the router's
// canonical 8-partial bf16 dot product and the one-warp softmax + top-k of a
// token.
#pragma once

#include "common.cuh"

namespace tmoe {

TMOE_DEV void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// All four pairs of a packed word: out[i] = (q_i - 8, q_{i+4} - 8) as half2,
// exact.  Pairs 1 and 3 are read 4 bits up, so they come out as 1024 + 16q and
// one HFMA2 (x/16 - 72) re-centres them.
TMOE_DEV void qpairs4(uint32_t w, uint32_t* out) {
  const __half2 off = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
  const __half2 sixteenth = __halves2half2(__ushort_as_half(0x2c00), __ushort_as_half(0x2c00));
  const __half2 m72 = __halves2half2(__ushort_as_half(0xd480), __ushort_as_half(0xd480));
  const uint32_t w8 = w >> 8;
  uint32_t v[4] = {(w & 0x000f000fu) | 0x64006400u, (w & 0x00f000f0u) | 0x64006400u,
                   (w8 & 0x000f000fu) | 0x64006400u, (w8 & 0x00f000f0u) | 0x64006400u};
  __half2 h0 = __hsub2(*reinterpret_cast<__half2*>(&v[0]), off);
  __half2 h1 = __hfma2(*reinterpret_cast<__half2*>(&v[1]), sixteenth, m72);
  __half2 h2 = __hsub2(*reinterpret_cast<__half2*>(&v[2]), off);
  __half2 h3 = __hfma2(*reinterpret_cast<__half2*>(&v[3]), sixteenth, m72);
  out[0] = *reinterpret_cast<uint32_t*>(&h0);
  out[1] = *reinterpret_cast<uint32_t*>(&h1);
  out[2] = *reinterpret_cast<uint32_t*>(&h2);
  out[3] = *reinterpret_cast<uint32_t*>(&h3);
}

// Position of element k (0..15) of a 16-element block in the fp16 operand
// layout: the order in which a packed word unpacks (pairs (i, i+4)).
TMOE_DEV int f16p_pos(int k) {
  const int hi = k & 8, r = k & 7;
  return hi + ((r & 3) << 1) + (r >> 2);
}

TMOE_DEV float tree8(float v) {
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return v;
}

// One canonical partial (chunks p, p+8, ...) of one row for NT tokens.
template <int NT>
TMOE_DEV void router_dots(const uint4* wrow_s, const uint4* xsm, int nch, int p, float* acc) {
#pragma unroll 4
  for (int c = p; c < nch; c += 8) {
    float wf[8];
    unpack8_bf16(wrow_s[c], wf);
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) {
      float xf[8];
      unpack8_bf16(xsm[tt * nch + c], xf);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[tt] = __fmaf_rn(xf[q], wf[q], acc[tt]);
    }
  }
}

struct RouteOut {
  int e;            // lane j < k: the j-th selected expert
  uint16_t score;   // its normalised bf16 score
};

// Softmax + top-k of one token by one warp, keys in registers (lane l holds
// e = 32c + l): the max, exponentials cexp(l - max), the canonical
// denominator (lane partials over c ascending, then the butterfly), bf16
// probabilities, keys (prob << 16 | 0xffff - e) so ties go to the lowest
// index; each lane sorts its keys (bitonic network, descending) and each of
// the k rounds takes the warp max of the lane heads, the winning lane dropping
// its head.  The selected probabilities are summed in selection order and
// rounded to bf16; score_j = bf16(p_j / sum).
template <int PER>
TMOE_DEV RouteOut route_token(const uint16_t* lg, int E, int k, int lane) {
  float v[PER];
  float m = -__int_as_float(0x7f800000);
#pragma unroll
  for (int c = 0; c < PER; ++c) {
    const int e = 32 * c + lane;
    v[c] = e < E ? bf2f(lg[e]) : -__int_as_float(0x7f800000);
    m = fmaxf(m, v[c]);
  }
  m = warp_max(m);
  float part = 0.0f;
#pragma unroll
  for (int c = 0; c < PER; ++c)
    if (32 * c + lane < E) {
      v[c] = cexp(__fsub_rn(v[c], m));
      part = __fadd_rn(part, v[c]);
    }
  const float inv = __fdiv_rn(1.0f, warp_butterfly_sum(part));
  uint32_t key[PER];
#pragma unroll
  for (int c = 0; c < PER; ++c) {
    const int e = 32 * c + lane;
    key[c] = e < E ? (((uint32_t)f2bf(__fmul_rn(v[c], inv)) << 16) | (uint32_t)(0xffff - e)) : 0u;
  }
#pragma unroll
  for (int kk = 2; kk <= PER; kk <<= 1)
#pragma unroll
    for (int jj = kk >> 1; jj > 0; jj >>= 1)
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int l = i ^ jj;
        if (l > i) {
          const uint32_t a = key[i], b = key[l];
          const bool desc = (i & kk) == 0;
          key[i] = desc ? max(a, b) : min(a, b);
          key[l] = desc ? min(a, b) : max(a, b);
        }
      }
  float ssum = 0.0f;
  uint32_t my_key = 0;
  for (int j = 0; j < k; ++j) {
    const uint32_t win = __reduce_max_sync(0xffffffffu, key[0]);
    const bool mine = key[0] == win;          // keys are distinct: one lane
#pragma unroll
    for (int c = 0; c < PER - 1; ++c) key[c] = mine ? key[c + 1] : key[c];
    key[PER - 1] = mine ? 0u : key[PER - 1];
    ssum = __fadd_rn(ssum, bf2f((uint16_t)(win >> 16)));
    if (lane == j) my_key = win;
  }
  const float sb = bfround(ssum);
  RouteOut r;
  r.e = 0xffff - (int)(my_key & 0xffffu);
  r.score = f2bf(__fdiv_rn(bf2f((uint16_t)(my_key >> 16)), sb));
  return r;
}

}  // namespace tmoe
