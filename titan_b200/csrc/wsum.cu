// Unsort + routed weighted top-k sum, plus the sigmoid-gated shared expert.
//
// Follows titan/kernels/moe_weighted_sum.py:51-98 and
// qwen3_5_moe/language.py:78-91.  Modes:
//   clone (0): bf16 products, eight bf16 partial accumulators (slot j % 8),
//              sequential bf16 combine — bit-identical to MLX's bf16 reduce;
//   fast  (1): fp32 products and partials, one rounding at the end.
// Optional shared term: y = bf16(y_routed) + bf16(bf16(sigmoid(bf16(gl))) * sh).
// One thread owns 8 consecutive columns (one 16-byte load per expert row).
#include "common.cuh"
#include "tmoe_internal.h"

namespace tmoe {

__global__ void __launch_bounds__(256) wsum_kernel(const uint16_t* __restrict__ ys,
                                                   const int32_t* __restrict__ inv,
                                                   const uint16_t* __restrict__ scores, int T,
                                                   int k, int D, int mode,
                                                   const uint16_t* __restrict__ sh,
                                                   const float* __restrict__ gate_logit,
                                                   uint16_t* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int dv = D / 8;
  if (i >= (long long)T * dv) return;
  const int t = (int)(i / dv), d0 = (int)(i % dv) * 8;
  float acc[8][8];
#pragma unroll
  for (int v = 0; v < 8; ++v)
#pragma unroll
    for (int a = 0; a < 8; ++a) acc[v][a] = 0.0f;
  for (int j = 0; j < k; ++j) {
    const int p = t * k + j;
    const int src = inv ? inv[p] : p;
    const float s = bf2f(scores[p]);
    float yv[8];
    unpack8_bf16(__ldg(reinterpret_cast<const uint4*>(ys + (size_t)src * D + d0)), yv);
    const int slot = j & 7;
#pragma unroll
    for (int v = 0; v < 8; ++v) {
#pragma unroll
      for (int a = 0; a < 8; ++a) {
        if (a != slot) continue;
        float prod = __fmul_rn(s, yv[v]);
        if (mode == 0) prod = bfround(prod);
        const float tt = __fadd_rn(acc[v][a], prod);
        acc[v][a] = (mode == 0) ? bfround(tt) : tt;
      }
    }
  }
  float sg = 0.0f;
  if (sh) sg = bfround(csigmoid(bfround(gate_logit[t])));
  uint16_t o[8];
#pragma unroll
  for (int v = 0; v < 8; ++v) {
    float a = acc[v][0];
#pragma unroll
    for (int j = 1; j < 8; ++j) {
      a = __fadd_rn(a, acc[v][j]);
      if (mode == 0) a = bfround(a);
    }
    a = bfround(a);
    if (sh) {
      const float shv = bfround(__fmul_rn(sg, bf2f(sh[(size_t)t * D + d0 + v])));
      a = __fadd_rn(a, shv);
    }
    o[v] = f2bf(a);
  }
  uint4 pk;
  pk.x = o[0] | ((uint32_t)o[1] << 16);
  pk.y = o[2] | ((uint32_t)o[3] << 16);
  pk.z = o[4] | ((uint32_t)o[5] << 16);
  pk.w = o[6] | ((uint32_t)o[7] << 16);
  *reinterpret_cast<uint4*>(out + (size_t)t * D + d0) = pk;
}

// The same arithmetic with every expert row of the thread in flight at once:
// the k source indices, scores and 16-byte row loads are issued before any
// product, so a thread waits for one memory latency instead of k.  Slot s
// accumulates the products j = s, s + 8, ... in order (clone mode rounds each
// step to bf16), then the eight slots combine in order — the bits of
// wsum_kernel.
template <int KMAX>
__global__ void __launch_bounds__(128) wsum_prefetch_kernel(const uint16_t* __restrict__ ys,
                                                            const int32_t* __restrict__ inv,
                                                            const uint16_t* __restrict__ scores,
                                                            int T, int k, int D, int mode,
                                                            const uint16_t* __restrict__ sh,
                                                            const float* __restrict__ gate_logit,
                                                            uint16_t* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int dv = D / 8;
  if (i >= (long long)T * dv) return;
  const int t = (int)(i / dv), d0 = (int)(i % dv) * 8;
  int src[KMAX];
  float sc[KMAX];
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    if (j < k) {
      const int p = t * k + j;
      src[j] = inv ? __ldg(inv + p) : p;
      sc[j] = bf2f(__ldg(scores + p));
    }
  }
  uint4 raw[KMAX];
#pragma unroll
  for (int j = 0; j < KMAX; ++j)
    if (j < k) raw[j] = __ldg(reinterpret_cast<const uint4*>(ys + (size_t)src[j] * D + d0));
  float sg = 0.0f;
  float shv8[8];
  if (sh) {
    sg = bfround(csigmoid(bfround(gate_logit[t])));
    unpack8_bf16(__ldg(reinterpret_cast<const uint4*>(sh + (size_t)t * D + d0)), shv8);
  }
  // two columns at a time (the two bf16 of one 32-bit word): packed f32x2
  // multiplies and adds and bf16x2 roundings, the same operations per column
  uint32_t o2[4];
#pragma unroll
  for (int vp = 0; vp < 4; ++vp) {
    float2 part[8];
#pragma unroll
    for (int a = 0; a < 8; ++a) part[a] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      if (j < k) {
        const uint32_t wd = vp == 0 ? raw[j].x : vp == 1 ? raw[j].y : vp == 2 ? raw[j].z : raw[j].w;
        const float2 y2 = make_float2(__uint_as_float(wd << 16), __uint_as_float(wd & 0xffff0000u));
        // scalar products (never fused into the following add)
        float2 prod = make_float2(__fmul_rn(sc[j], y2.x), __fmul_rn(sc[j], y2.y));
        if (mode == 0) prod = bfround2(prod);
        const float2 tt = __fadd2_rn(part[j & 7], prod);
        part[j & 7] = (mode == 0) ? bfround2(tt) : tt;
      }
    }
    float2 a = part[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) {
      a = __fadd2_rn(a, part[j]);
      if (mode == 0) a = bfround2(a);
    }
    a = bfround2(a);
    if (sh)
      a = __fadd2_rn(a, bfround2(__fmul2_rn(make_float2(sg, sg),
                                            make_float2(shv8[2 * vp], shv8[2 * vp + 1]))));
    o2[vp] = (uint32_t)f2bf(a.x) | ((uint32_t)f2bf(a.y) << 16);
  }
  *reinterpret_cast<uint4*>(out + (size_t)t * D + d0) = make_uint4(o2[0], o2[1], o2[2], o2[3]);
}

cudaError_t launch_wsum(const uint16_t* ys, const int32_t* inv, const uint16_t* scores, int T, int k,
                        int D, int mode, const uint16_t* sh, const float* gate_logit, uint16_t* out,
                        cudaStream_t s) {
  const long long n = (long long)T * (D / 8);
  if (n <= 0) return cudaGetLastError();
  const unsigned grid = (unsigned)((n + 127) / 128), grid256 = (unsigned)((n + 255) / 256);
  if (k <= 8)
    wsum_prefetch_kernel<8><<<grid, 128, 0, s>>>(ys, inv, scores, T, k, D, mode, sh, gate_logit, out);
  else if (k <= 12)
    wsum_prefetch_kernel<12><<<grid, 128, 0, s>>>(ys, inv, scores, T, k, D, mode, sh, gate_logit,
                                                 out);
  else if (k <= 16)
    wsum_prefetch_kernel<16><<<grid, 128, 0, s>>>(ys, inv, scores, T, k, D, mode, sh, gate_logit,
                                                 out);
  else
    wsum_kernel<<<grid256, 256, 0, s>>>(ys, inv, scores, T, k, D, mode, sh, gate_logit, out);
  return cudaGetLastError();
}

// SwiGLU over a [R, 2I] gate|up tensor, bf16 rounding after each op.
__global__ void __launch_bounds__(256) swiglu_kernel(const uint16_t* __restrict__ gu, long long R,
                                                     int I, uint16_t* __restrict__ h) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R * I) return;
  const long long r = i / I;
  const int c = (int)(i % I);
  h[i] = f2bf(swiglu_bf16(bf2f(gu[r * 2 * I + c]), bf2f(gu[r * 2 * I + I + c])));
}

cudaError_t launch_swiglu(const uint16_t* gu, int R, int I, uint16_t* h, cudaStream_t s) {
  const long long n = (long long)R * I;
  if (n > 0) swiglu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(gu, R, I, h);
  return cudaGetLastError();
}

}  // namespace tmoe
