// Decode-shaped MoE (a handful of tokens): grouped GEMVs over the distinct
// experts the batch selected, on the tensor cores.
//
// Follows engine/patches/decode-fusion/fused_kernels.py:31-229 (gate_up_silu
// and down_wsum): fp32 accumulation, h = silu(g)*u kept in fp32, the routed
// weighted sum and the sigmoid-gated shared expert folded in fp32 and rounded
// to bf16 once.
//
// B200 mapping.  A CTA owns one (expert, 64-row weight slab).  It first
// issues cp.async copies of the whole slab — packed int4 rows, scales and
// biases — and of the activation columns into shared memory, so every CTA's
// bytes are in flight at once (the kernel is HBM-bound; latency hiding is the
// whole game), then runs m16n8k16 MMAs from shared memory: the weights are the
// A operand as exact fp16 (q - 8) (one LOP3 + one HSUB2 per two weights:
// 0x6400|q is 1024+q), the activations the B operand (bf16 x converts to
// fp16 exactly; fp32 h is split into hi + lo fp16 halves, both multiplied).
// Per 64-group the fp32 MMA result is scaled on the CUDA cores:
// acc += s * D + (b + 8s) * sum(column over the group).
//
// Modes: 0 = gate_up rows (i, I+i) -> h = silu(g)*u fp32; 1 = down -> fp32
// partial per (token, slot) and, in the last CTA to finish an output slab
// (a device-wide counter, no waiting), the ordered weighted sum plus the gated
// shared expert -> bf16 y; 2 = plain bf16 output rows (the stock gather).
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

TMOE_DEV int f16p_pos(int k) {
  const int hi = k & 8, r = k & 7;
  return hi + ((r & 3) << 1) + (r >> 2);
}

constexpr int kRows = 64;      // weight rows per CTA (4 warps x 16)
constexpr int kCols = 8;       // activation columns per MMA pass
constexpr int kThreads = 128;

// Shared-memory plan for a slab with reduction length K.  Weight rows are
// padded to 8 words mod 32 and activation columns to 4 words mod 32 so the
// fragment loads are bank-conflict free.
struct Smem {
  int w_ld, c_ld, G;
  int w_off, s_off, b_off, hi_off, lo_off, sum_off, total;
  TMOE_DEV Smem(int K, bool lo) {
    G = K / kGroup;
    w_ld = K / 2 + 32;
    c_ld = K * 2 + 16;
    w_off = 0;
    s_off = w_off + kRows * w_ld;
    b_off = s_off + ((kRows * G * 2 + 15) & ~15);
    hi_off = b_off + ((kRows * G * 2 + 15) & ~15);
    lo_off = hi_off + kCols * c_ld;
    sum_off = lo_off + (lo ? kCols * c_ld : 0);
    total = sum_off + kCols * G * 4;
  }
};

}  // namespace

size_t gemv_stream_smem(int K, bool lo) {
  const int G = K / kGroup;
  const size_t w = (size_t)kRows * (K / 2 + 32);
  const size_t sb = 2 * (((size_t)kRows * G * 2 + 15) & ~size_t(15));
  const size_t c = (size_t)kCols * (K * 2 + 16) * (lo ? 2 : 1);
  return w + sb + c + (size_t)kCols * G * 4;
}

template <int MODE>
__global__ void __launch_bounds__(kThreads) gemv_stream_kernel(StreamParams P) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int u = blockIdx.x;
  const bool shared = P.Wsh != nullptr && u == P.umax;
  const int nuniq = P.nuniq[0];
  if (!shared && u >= nuniq) return;
  const int e = shared ? 0 : P.uexp[u];
  const int p0 = shared ? 0 : P.ustart[u];
  const int ncol = shared ? P.nsh : (P.ustart[u + 1] - p0);
  const int N = shared ? P.Nsh : P.N;
  const int K = shared ? P.K_sh : P.K;
  const int G = K / kGroup, KW = K / 8;
  const int slab = blockIdx.y;
  const int rows_here = (MODE == 0) ? N / 2 : N;
  if (slab * (MODE == 0 ? kRows / 2 : kRows) >= rows_here) return;
  const Smem L(K, MODE == 1);
  const uint32_t* We = shared ? P.Wsh : P.W + (size_t)e * N * KW;
  const uint16_t* Se = shared ? P.Ssh : P.S + (size_t)e * N * G;
  const uint16_t* Be = shared ? P.Bsh : P.B + (size_t)e * N * G;

  // smem row r <-> weight row (mode 0: 32 gate rows then the 32 matching up rows)
  auto wrow_of = [&](int r) -> int {
    if (MODE == 0) return (r < 32) ? slab * 32 + r : N / 2 + slab * 32 + (r - 32);
    return slab * kRows + r;
  };

  // ---- stage the weight slab (one shot; it stays for every column pass)
  {
    const int wchunks = KW / 4;                      // 16-byte chunks per row
    for (int i = tid; i < kRows * wchunks; i += kThreads) {
      const int r = i / wchunks, c = i % wchunks;
      cp_async16(sm + L.w_off + r * L.w_ld + c * 16, We + (size_t)wrow_of(r) * KW + c * 4);
    }
    const int sw = G / 2;                            // scales / biases: 4-byte copies
    for (int i = tid; i < kRows * sw; i += kThreads) {
      const int r = i / sw, c = i % sw;
      const size_t src = (size_t)wrow_of(r) * G + 2 * c;
      cp_async4(sm + L.s_off + (r * G + 2 * c) * 2, Se + src);
      cp_async4(sm + L.b_off + (r * G + 2 * c) * 2, Be + src);
    }
    cp_async_commit();
  }

  const int rl = (MODE == 0) ? warp * 8 + g : warp * 16 + g;       // smem rows of this thread
  const int rh = (MODE == 0) ? 32 + warp * 8 + g : warp * 16 + g + 8;
  const uint8_t* wl = sm + L.w_off + rl * L.w_ld;
  const uint8_t* wh = sm + L.w_off + rh * L.w_ld;
  const uint16_t* ss = reinterpret_cast<const uint16_t*>(sm + L.s_off);
  const uint16_t* bs = reinterpret_cast<const uint16_t*>(sm + L.b_off);
  const uint8_t* chi = sm + L.hi_off;
  const uint8_t* clo = sm + L.lo_off;
  const float* csum = reinterpret_cast<const float*>(sm + L.sum_off);

  for (int cb = 0; cb < ncol; cb += kCols) {
    const int nc = min(kCols, ncol - cb);
    __syncthreads();                                  // previous pass done with the columns
    if (MODE == 1) {
      // fp32 h -> hi/lo fp16 operand layout + group sums, one warp per (col, group)
      for (int task = warp; task < kCols * G; task += kThreads / 32) {
        const int c = task / G, grp = task % G;
        float a = 0.0f, b = 0.0f;
        if (c < nc) {
          const int col = cb + c;
          const float* src = shared ? P.h_sh + (size_t)col * K
                                    : P.h + (size_t)P.order[p0 + col] * K;
          const float2 v = *reinterpret_cast<const float2*>(src + grp * kGroup + 2 * lane);
          a = v.x;
          b = v.y;
        }
        const __half ah = __float2half_rn(a), bh = __float2half_rn(b);
        const __half al = __float2half_rn(__fsub_rn(a, __half2float(ah)));
        const __half bl = __float2half_rn(__fsub_rn(b, __half2float(bh)));
        const int k0 = grp * kGroup + 2 * lane;
        uint16_t* hp = reinterpret_cast<uint16_t*>(sm + L.hi_off + c * L.c_ld);
        uint16_t* lp = reinterpret_cast<uint16_t*>(sm + L.lo_off + c * L.c_ld);
        hp[(k0 & ~15) + f16p_pos(k0 & 15)] = __half_as_ushort(ah);
        hp[((k0 + 1) & ~15) + f16p_pos((k0 + 1) & 15)] = __half_as_ushort(bh);
        lp[(k0 & ~15) + f16p_pos(k0 & 15)] = __half_as_ushort(al);
        lp[((k0 + 1) & ~15) + f16p_pos((k0 + 1) & 15)] = __half_as_ushort(bl);
        const float part = __fadd_rn(__fadd_rn(__half2float(ah), __half2float(al)),
                                     __fadd_rn(__half2float(bh), __half2float(bl)));
        const float s = warp_butterfly_sum(part);
        if (lane == 0) reinterpret_cast<float*>(sm + L.sum_off)[c * G + grp] = s;
      }
    } else {
      const int cchunks = K / 8;                      // 16-byte chunks per column
      for (int i = tid; i < kCols * cchunks; i += kThreads) {
        const int c = i / cchunks, q = i % cchunks;
        const int col = cb + (c < nc ? c : 0);
        const int arow = shared ? col : P.order[p0 + col] / P.col_div;
        cp_async16(sm + L.hi_off + c * L.c_ld + q * 16, P.x16p + (size_t)arow * K + q * 8);
      }
      for (int i = tid; i < kCols * G; i += kThreads) {
        const int c = i / G, grp = i % G;
        const int col = cb + (c < nc ? c : 0);
        const int arow = shared ? col : P.order[p0 + col] / P.col_div;
        cp_async4(sm + L.sum_off + (c * G + grp) * 4, P.xsum + (size_t)arow * G + grp);
      }
      cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();

    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int bcol = g;                                // B column this thread loads
#pragma unroll 2
    for (int grp = 0; grp < G; ++grp) {
      const uint2 wL = *reinterpret_cast<const uint2*>(wl + grp * 32 + t * 8);
      const uint2 wH = *reinterpret_cast<const uint2*>(wh + grp * 32 + t * 8);
      uint32_t a[4][4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const uint32_t xL = (m < 2) ? wL.x : wL.y;
        const uint32_t xH = (m < 2) ? wH.x : wH.y;
        const int pi = (m & 1) * 2;
        a[m][0] = qpair(xL, pi);
        a[m][1] = qpair(xH, pi);
        a[m][2] = qpair(xL, pi + 1);
        a[m][3] = qpair(xH, pi + 1);
      }
      float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      {
        const uint4* bp = reinterpret_cast<const uint4*>(chi + bcol * L.c_ld + grp * 128 + t * 32);
        const uint4 v0 = bp[0], v1 = bp[1];
        mma16816(d, a[0][0], a[0][1], a[0][2], a[0][3], v0.x, v0.y);
        mma16816(d, a[1][0], a[1][1], a[1][2], a[1][3], v0.z, v0.w);
        mma16816(d, a[2][0], a[2][1], a[2][2], a[2][3], v1.x, v1.y);
        mma16816(d, a[3][0], a[3][1], a[3][2], a[3][3], v1.z, v1.w);
      }
      if (MODE == 1) {
        const uint4* bp = reinterpret_cast<const uint4*>(clo + bcol * L.c_ld + grp * 128 + t * 32);
        const uint4 v0 = bp[0], v1 = bp[1];
        mma16816(d, a[0][0], a[0][1], a[0][2], a[0][3], v0.x, v0.y);
        mma16816(d, a[1][0], a[1][1], a[1][2], a[1][3], v0.z, v0.w);
        mma16816(d, a[2][0], a[2][1], a[2][2], a[2][3], v1.x, v1.y);
        mma16816(d, a[3][0], a[3][1], a[3][2], a[3][3], v1.z, v1.w);
      }
      const float s_lo = bf2f(ss[rl * G + grp]), s_hi = bf2f(ss[rh * G + grp]);
      const float bv_lo = __fadd_rn(bf2f(bs[rl * G + grp]), __fmul_rn(8.0f, s_lo));
      const float bv_hi = __fadd_rn(bf2f(bs[rh * G + grp]), __fmul_rn(8.0f, s_hi));
      const float xs0 = csum[(2 * t) * G + grp], xs1 = csum[(2 * t + 1) * G + grp];
      acc[0] = __fmaf_rn(s_lo, d[0], __fmaf_rn(bv_lo, xs0, acc[0]));
      acc[1] = __fmaf_rn(s_lo, d[1], __fmaf_rn(bv_lo, xs1, acc[1]));
      acc[2] = __fmaf_rn(s_hi, d[2], __fmaf_rn(bv_hi, xs0, acc[2]));
      acc[3] = __fmaf_rn(s_hi, d[3], __fmaf_rn(bv_hi, xs1, acc[3]));
    }
    // epilogue for columns 2t, 2t+1 of this pass
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = 2 * t + h;
      if (c >= nc) continue;
      const int col = cb + c;
      const int orow = shared ? col : P.order[p0 + col];
      if (MODE == 0) {
        const int i = slab * 32 + warp * 8 + g;
        float* out = shared ? P.out_sh : P.out;
        out[(size_t)orow * (N / 2) + i] = silu_mul_f32(acc[h], acc[2 + h]);
      } else if (MODE == 1) {
        float* out = shared ? P.out_sh : P.out;
        const int d0 = slab * kRows + warp * 16 + g;
        out[(size_t)orow * N + d0] = acc[h];
        out[(size_t)orow * N + d0 + 8] = acc[2 + h];
      } else {
        const int d0 = slab * kRows + warp * 16 + g;
        P.outb[(size_t)orow * N + d0] = f2bf(acc[h]);
        P.outb[(size_t)orow * N + d0 + 8] = f2bf(acc[2 + h]);
      }
    }
  }

  if (MODE == 1) {
    // The last CTA to finish this output slab folds the partials: ordered
    // weighted sum over the k slots plus the gated shared expert.  Nobody
    // waits: every CTA counts itself in and only the last one does the sum.
    __shared__ int last;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int contributors = nuniq + (P.Wsh ? 1 : 0);
      last = (atomicAdd(&P.counters[slab], 1) == contributors - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int D = P.N;
    for (int i = tid; i < P.T * kRows; i += kThreads) {
      const int tt = i / kRows, d = slab * kRows + (i % kRows);
      float a = 0.0f;
      for (int j = 0; j < P.k; ++j) {
        const size_t p = (size_t)tt * P.k + j;
        const float sc = P.scores_f32 ? P.scores_f32[p] : bf2f(P.scores[p]);
        a = __fmaf_rn(sc, __ldcg(P.out + p * D + d), a);
      }
      if (P.Wsh) a = __fmaf_rn(csigmoid(P.gate_logit[tt]), __ldcg(P.out_sh + (size_t)tt * D + d), a);
      P.y[(size_t)tt * D + d] = f2bf(a);
    }
    if (tid == 0) P.counters[slab] = 0;
  }
}

cudaError_t launch_gemv_stream(int mode, const StreamParams& P, cudaStream_t s) {
  const int nb_x = P.umax + (P.Wsh ? 1 : 0);
  const int nmax = (P.Wsh && P.Nsh > P.N) ? P.Nsh : P.N;
  const int kmax = (P.Wsh && P.K_sh > P.K) ? P.K_sh : P.K;
  const int nb_y = (mode == 0) ? (nmax / 2 + 31) / 32 : (nmax + kRows - 1) / kRows;
  if (nb_x <= 0 || nb_y <= 0) return cudaSuccess;
  const size_t smem = gemv_stream_smem(kmax, mode == 1);
  dim3 grid(nb_x, nb_y);
  cudaError_t err = cudaSuccess;
  if (mode == 0) {
    err = cudaFuncSetAttribute(gemv_stream_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
    if (err == cudaSuccess) gemv_stream_kernel<0><<<grid, kThreads, smem, s>>>(P);
  } else if (mode == 1) {
    err = cudaFuncSetAttribute(gemv_stream_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
    if (err == cudaSuccess) gemv_stream_kernel<1><<<grid, kThreads, smem, s>>>(P);
  } else {
    err = cudaFuncSetAttribute(gemv_stream_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
    if (err == cudaSuccess) gemv_stream_kernel<2><<<grid, kThreads, smem, s>>>(P);
  }
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

// Activation prep (prefill / stock gathers): bf16 rows -> fp16 operand layout
// + exact group sums (canonical pair-sum + butterfly order), written at
// xsum[m*sm + g*sg].  One warp per (row, group); lane l holds 2l, 2l+1.
__global__ void __launch_bounds__(256) prep_x_kernel(const uint16_t* __restrict__ x, int R, int K,
                                                      uint16_t* __restrict__ x16p,
                                                      float* __restrict__ xsum, long long sm_,
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
  if (lane == 0) xsum[m * sm_ + g * sg] = s;
}

cudaError_t launch_prep_x(const uint16_t* x, int R, int K, uint16_t* x16p, float* xsum,
                          long long sum_sm, long long sum_sg, cudaStream_t s) {
  const long long warps = (long long)R * (K / kGroup);
  if (warps > 0)
    prep_x_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(x, R, K, x16p, xsum, sum_sm,
                                                                       sum_sg);
  return cudaGetLastError();
}

__global__ void zero_i32_kernel(int32_t* p, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = 0;
}

cudaError_t launch_zero_i32(int32_t* p, int n, cudaStream_t s) {
  if (n > 0) zero_i32_kernel<<<(n + 255) / 256, 256, 0, s>>>(p, n);
  return cudaGetLastError();
}

}  // namespace tmoe
