// Register-fragment helpers shared by the decode kernels (sm_100a):
// m16n8k16 fp16 MMAs on exact integer weights, the nibble unpacking that
// feeds them, the permuted activation layout that matches it, and the
// router's canonical 8-partial bf16 dot product.
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

}  // namespace tmoe
