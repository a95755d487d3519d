// Decode-shaped MoE (a handful of tokens): grouped GEMVs over the distinct
// experts the batch selected, on the tensor cores.
//
// Follows engine/patches/decode-fusion/fused_kernels.py:31-229 (gate_up_silu
// and down_wsum): fp32 accumulation, h = silu(g)*u kept in fp32, the routed
// weighted sum and the sigmoid-gated shared expert folded in fp32 and rounded
// to bf16 once.
//
// B200 mapping: each warp owns 16 weight rows and runs m16n8k16 MMAs with the
// weights as the A operand and up to 8 tokens (or (token, slot) pairs) as the
// N columns.  A = (q - 8) in fp16 straight from the packed nibbles (one LOP3
// and one HSUB2 per two weights: 0x6400|q is 1024+q); B = the activation in
// fp16 (bf16 x converts exactly; fp32 h is split into hi + lo fp16 halves and
// both are multiplied).  Per 64-group the fp32 MMA result is scaled on the
// CUDA cores: acc += s * D + (b + 8s) * sum(x over the group).  Every expert's
// weights are streamed once per call regardless of how many tokens chose it.
#include "common.cuh"
#include "tmoe_internal.h"

namespace tmoe {

namespace {

TMOE_DEV void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// pair i of word w as half2 (q_i - 8, q_{i+4} - 8), exact.
TMOE_DEV uint32_t qpair(uint32_t w, int i) {
  uint32_t v = ((w >> (4 * i)) & 0x000f000fu) | 0x64006400u;
  const __half2 off = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
  __half2 h = __hsub2(*reinterpret_cast<__half2*>(&v), off);
  return *reinterpret_cast<uint32_t*>(&h);
}

TMOE_DEV uint2 ldg64(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

TMOE_DEV int f16p_pos(int k) {
  const int hi = k & 8, r = k & 7;
  return hi + ((r & 3) << 1) + (r >> 2);
}

}  // namespace

// Activation prep: bf16 rows -> fp16 operand layout + exact group sums
// (canonical pair-sum + butterfly order), written at xsum[m*sm + g*sg].
// One warp per (row, group); lane l holds elements 2l, 2l+1.
__global__ void __launch_bounds__(256) prep_x_kernel(const uint16_t* __restrict__ x, int R, int K,
                                                      uint16_t* __restrict__ x16p,
                                                      float* __restrict__ xsum, long long sm,
                                                      long long sg) {
  const int lane = threadIdx.x & 31;
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int G = K / kGroup;
  if (w >= (long long)R * G) return;
  const int m = (int)(w / G), g = (int)(w % G);
  const uint16_t* src = x + (size_t)m * K + g * kGroup;
  const float a = bf2f(src[2 * lane]), b = bf2f(src[2 * lane + 1]);
  const float s = warp_butterfly_sum(__fadd_rn(a, b));
  uint16_t* dst = x16p + (size_t)m * K + g * kGroup;
  const int k0 = 2 * lane;
  dst[(k0 & ~15) + f16p_pos(k0 & 15)] = __half_as_ushort(__float2half_rn(a));
  dst[((k0 + 1) & ~15) + f16p_pos((k0 + 1) & 15)] = __half_as_ushort(__float2half_rn(b));
  if (lane == 0) xsum[m * sm + g * sg] = s;
}

// fp32 h rows -> hi/lo fp16 operand layout + group sums of (hi + lo).
__global__ void __launch_bounds__(256) prep_h_kernel(const float* __restrict__ h, int R, int K,
                                                      uint16_t* __restrict__ hhi,
                                                      uint16_t* __restrict__ hlo,
                                                      float* __restrict__ hsum) {
  const int lane = threadIdx.x & 31;
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int G = K / kGroup;
  if (w >= (long long)R * G) return;
  const int m = (int)(w / G), g = (int)(w % G);
  const float* src = h + (size_t)m * K + g * kGroup;
  float part = 0.0f;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int k0 = 2 * lane + u;
    const float v = src[k0];
    const __half hi = __float2half_rn(v);
    const float r = __fsub_rn(v, __half2float(hi));
    const __half lo = __float2half_rn(r);
    const size_t o = (size_t)m * K + g * kGroup + (k0 & ~15) + f16p_pos(k0 & 15);
    hhi[o] = __half_as_ushort(hi);
    hlo[o] = __half_as_ushort(lo);
    part = __fadd_rn(part, __fadd_rn(__half2float(hi), __half2float(lo)));
  }
  const float s = warp_butterfly_sum(part);
  if (lane == 0) hsum[(size_t)m * G + g] = s;
}

constexpr int kNC = 4;  // 8-column chunks held per sweep (32 columns)

__global__ void __launch_bounds__(128) gemv_tc_kernel(GemvParams P) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int u = blockIdx.x;
  const bool shared = P.Wsh != nullptr && u == P.umax;
  if (!shared && u >= P.nuniq[0]) return;
  const int e = shared ? 0 : P.uexp[u];
  const int p0 = shared ? 0 : P.ustart[u];
  const int ncol = shared ? P.nsh : (P.ustart[u + 1] - p0);
  const int N = shared ? P.Nsh : P.N;
  const int K = shared ? P.K_sh : P.K, G = K / kGroup, KW = K / 8;
  const uint16_t* act_hi = shared ? P.bh_sh : P.bh;
  const uint16_t* act_lo = shared ? P.bl_sh : P.bl;
  const float* act_sum = shared ? P.bsum_sh : P.bsum;
  const uint32_t* We = shared ? P.Wsh : P.W + (size_t)e * N * KW;
  const uint16_t* Se = shared ? P.Ssh : P.S + (size_t)e * N * G;
  const uint16_t* Be = shared ? P.Bsh : P.B + (size_t)e * N * G;
  int r_lo, r_hi;
  if (P.swiglu) {
    const int i = blockIdx.y * 32 + warp * 8 + g;
    if (blockIdx.y * 32 >= N / 2) return;
    r_lo = i;
    r_hi = N / 2 + i;
  } else {
    const int r0 = blockIdx.y * 64 + warp * 16;
    if (blockIdx.y * 64 >= N) return;
    r_lo = r0 + g;
    r_hi = r0 + g + 8;
  }
  const uint32_t* wlo = We + (size_t)r_lo * KW;
  const uint32_t* whi = We + (size_t)r_hi * KW;

  for (int cb = 0; cb < ncol; cb += 8 * kNC) {
    // activation rows of the columns this thread loads (col g of each chunk)
    // and of the columns it owns in C (2t, 2t+1 of each chunk).
    int brow[kNC], crow[kNC][2];
#pragma unroll
    for (int c = 0; c < kNC; ++c) {
      const int colb = cb + 8 * c + g;
      brow[c] = colb < ncol ? (shared ? colb : P.order[p0 + colb] / P.col_div) : -1;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int colc = cb + 8 * c + 2 * t + h;
        crow[c][h] = colc < ncol ? (shared ? colc : P.order[p0 + colc] / P.col_div) : -1;
      }
    }
    float acc[kNC][4];
#pragma unroll
    for (int c = 0; c < kNC; ++c)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[c][q] = 0.0f;

#pragma unroll 2
    for (int grp = 0; grp < G; ++grp) {
      const uint2 wl = ldg64(wlo + grp * 8 + 2 * t);
      const uint2 wh = ldg64(whi + grp * 8 + 2 * t);
      const float s_lo = bf2f(Se[(size_t)r_lo * G + grp]), s_hi = bf2f(Se[(size_t)r_hi * G + grp]);
      const float bv_lo = __fadd_rn(bf2f(Be[(size_t)r_lo * G + grp]), __fmul_rn(8.0f, s_lo));
      const float bv_hi = __fadd_rn(bf2f(Be[(size_t)r_hi * G + grp]), __fmul_rn(8.0f, s_hi));
      uint32_t a[4][4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const uint32_t wL = (m < 2) ? wl.x : wl.y;
        const uint32_t wH = (m < 2) ? wh.x : wh.y;
        const int pi = (m & 1) * 2;
        a[m][0] = qpair(wL, pi);
        a[m][1] = qpair(wH, pi);
        a[m][2] = qpair(wL, pi + 1);
        a[m][3] = qpair(wH, pi + 1);
      }
#pragma unroll
      for (int c = 0; c < kNC; ++c) {
        if (cb + 8 * c >= ncol) break;
        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const uint16_t* bsrc = part ? act_lo : act_hi;
          if (!bsrc) continue;
          uint4 v0 = make_uint4(0, 0, 0, 0), v1 = make_uint4(0, 0, 0, 0);
          if (brow[c] >= 0) {
            const uint4* bp = reinterpret_cast<const uint4*>(bsrc + (size_t)brow[c] * K + grp * kGroup + t * 16);
            v0 = __ldg(bp);
            v1 = __ldg(bp + 1);
          }
          mma16816(d, a[0][0], a[0][1], a[0][2], a[0][3], v0.x, v0.y);
          mma16816(d, a[1][0], a[1][1], a[1][2], a[1][3], v0.z, v0.w);
          mma16816(d, a[2][0], a[2][1], a[2][2], a[2][3], v1.x, v1.y);
          mma16816(d, a[3][0], a[3][1], a[3][2], a[3][3], v1.z, v1.w);
        }
        const float xs0 = crow[c][0] >= 0 ? act_sum[(size_t)crow[c][0] * G + grp] : 0.0f;
        const float xs1 = crow[c][1] >= 0 ? act_sum[(size_t)crow[c][1] * G + grp] : 0.0f;
        acc[c][0] = __fmaf_rn(s_lo, d[0], __fmaf_rn(bv_lo, xs0, acc[c][0]));
        acc[c][1] = __fmaf_rn(s_lo, d[1], __fmaf_rn(bv_lo, xs1, acc[c][1]));
        acc[c][2] = __fmaf_rn(s_hi, d[2], __fmaf_rn(bv_hi, xs0, acc[c][2]));
        acc[c][3] = __fmaf_rn(s_hi, d[3], __fmaf_rn(bv_hi, xs1, acc[c][3]));
      }
    }
    // epilogue
#pragma unroll
    for (int c = 0; c < kNC; ++c) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int colc = cb + 8 * c + 2 * t + h;
        if (colc >= ncol) continue;
        const int orow = shared ? colc : P.order[p0 + colc];
        float* out = shared ? P.out_sh : P.out;
        if (P.swiglu) {
          const int Ih = N / 2;
          out[(size_t)orow * Ih + r_lo] = silu_mul_f32(acc[c][h], acc[c][2 + h]);
        } else if (P.outb && !shared) {
          P.outb[(size_t)orow * N + r_lo] = f2bf(acc[c][h]);
          P.outb[(size_t)orow * N + r_hi] = f2bf(acc[c][2 + h]);
        } else {
          out[(size_t)orow * N + r_lo] = acc[c][h];
          out[(size_t)orow * N + r_hi] = acc[c][2 + h];
        }
      }
    }
  }
}

// y[t,d] = bf16( sum_j score[t,j] * part[t*k+j, d] + sigmoid(gl[t]) * shared[t,d] )
// Scores are bf16 (router output) or fp32 (scores_f32, the decode-fusion API).
__global__ void __launch_bounds__(256) decode_combine_kernel(
    const float* __restrict__ part, const uint16_t* __restrict__ scores,
    const float* __restrict__ scores_f32, int T, int k, int D, const float* __restrict__ shared,
    const float* __restrict__ gate_logit, uint16_t* __restrict__ y) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)T * D) return;
  const int t = (int)(i / D), d = (int)(i % D);
  float acc = 0.0f;
  for (int j = 0; j < k; ++j) {
    const float sc = scores_f32 ? scores_f32[(size_t)t * k + j] : bf2f(scores[(size_t)t * k + j]);
    acc = __fmaf_rn(sc, part[((size_t)t * k + j) * D + d], acc);
  }
  if (shared) acc = __fmaf_rn(csigmoid(gate_logit[t]), shared[(size_t)t * D + d], acc);
  y[i] = f2bf(acc);
}

cudaError_t launch_prep_x(const uint16_t* x, int R, int K, uint16_t* x16p, float* xsum,
                          long long sum_sm, long long sum_sg, cudaStream_t s) {
  const long long warps = (long long)R * (K / kGroup);
  if (warps > 0)
    prep_x_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(x, R, K, x16p, xsum, sum_sm,
                                                                       sum_sg);
  return cudaGetLastError();
}

cudaError_t launch_prep_h(const float* h, int R, int K, uint16_t* hhi, uint16_t* hlo, float* hsum,
                          cudaStream_t s) {
  const long long warps = (long long)R * (K / kGroup);
  if (warps > 0)
    prep_h_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(h, R, K, hhi, hlo, hsum);
  return cudaGetLastError();
}

cudaError_t launch_gemv_tc(const GemvParams& P, cudaStream_t s) {
  const int nb_x = P.umax + (P.Wsh ? 1 : 0);
  const int nmax = P.Wsh && P.Nsh > P.N ? P.Nsh : P.N;
  const int nb_y = P.swiglu ? (nmax / 2 + 31) / 32 : (nmax + 63) / 64;
  if (nb_x <= 0 || nb_y <= 0) return cudaSuccess;
  gemv_tc_kernel<<<dim3(nb_x, nb_y), 128, 0, s>>>(P);
  return cudaGetLastError();
}

cudaError_t launch_decode_combine(const float* part, const uint16_t* scores,
                                  const float* scores_f32, int T, int k, int D,
                                  const float* shared, const float* gate_logit, uint16_t* y,
                                  cudaStream_t s) {
  const long long n = (long long)T * D;
  if (n > 0)
    decode_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, scores, scores_f32, T, k,
                                                                      D, shared, gate_logit, y);
  return cudaGetLastError();
}

}  // namespace tmoe
