// Grouped (expert-sorted) GEMMs over a ragged tile table, mma.sync version.
//
// Two arithmetic variants share one cp.async-pipelined 128x128 CTA tile:
//
//  * I8  — the reference's int8 x int4 algebra (moe_gather_int8.py:20-32,
//    256-349): activations are signed codes xs = xu - 128 with a per
//    (row, 64-group) scale; the packed nibbles are widened in registers to
//    16*(q-8) (a signed byte), so one s8 x s8 -> s32 MMA over a group gives
//    16 * sum (xu-128)(q-8) exactly — the reference's D - 128*qsum + av
//    without any qsum table.  Per group the integer result is rescaled in
//    fp32: acc = fma(D''*s, xsc, acc); acc = fma(xrs, bf16(b + 8s), acc).
//
//  * F16 — the stock bf16-activation gather (mx.gather_qmm): A = x in fp16
//    (exact for |x| in fp16 range), B = (q-8)*s in fp16 (exact: an 8-bit
//    bf16 significand times a 4-bit integer fits fp16's 11 bits), fp32
//    accumulation on the tensor cores; the affine bias term (b + 8s) * sum(x)
//    over each group is added in fp32 from the exact group sums.
//
// K permutation: the dot product over one 64-wide group is order-free, so
// each thread's MMA fragments are assigned k values that sit contiguously in
// shared memory (A: one 16-byte load per row; B: one 8-byte load = two packed
// words per column).  A and B use the same permutation.
//
// Epilogues: plain bf16 store; fused SwiGLU (gate rows [0,I), up rows [I,2I)
// in the same CTA) followed by the per-(row, 64-group) int8 requantisation of
// h for the down projection, or by an fp16 copy of h for the F16 down GEMM.
#include "common.cuh"
#include "tmoe_internal.h"

namespace tmoe {

namespace {

constexpr int BM = 128, BN = 128;

template <bool I8>
struct Cfg {
  static constexpr int A_ROW = I8 ? 64 : 128;     // bytes of one row per group
  static constexpr int A_BYTES = BM * A_ROW;
  static constexpr int B_BYTES = BN * 32;
  static constexpr int T_BYTES = BN * 2 * 2;      // scales + biases (bf16)
  static constexpr int R_BYTES = BM * 4 * 2;      // row scale + row sum (fp32)
  static constexpr int STAGE = A_BYTES + B_BYTES + T_BYTES + R_BYTES;
  static constexpr int NST = I8 ? 4 : 3;
  static constexpr int SMEM = STAGE * NST;
};

TMOE_DEV void mma_s8(int* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                     uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

TMOE_DEV void mma_f16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                      uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

TMOE_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// 8 nibbles (element j in bits 4j..4j+3) -> two words of signed bytes
// 16*(q-8): lo = elements 0..3, hi = elements 4..7.
TMOE_DEV void widen_s8x16(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x88888888u;
  const uint32_t ev = (x << 4) & 0xf0f0f0f0u;  // byte b = element 2b in the high nibble
  const uint32_t od = x & 0xf0f0f0f0u;         // byte b = element 2b+1
  lo = prmt(ev, od, 0x5140u);
  hi = prmt(ev, od, 0x7362u);
}

// 8 nibbles -> four half2 of (q-8)*s: pair i = (element i, element i+4).
TMOE_DEV void dequant_f16(uint32_t w, __half2 s2, uint32_t* out) {
  const __half2 off = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t v = ((w >> (4 * i)) & 0x000f000fu) | 0x64006400u;
    __half2 h = *reinterpret_cast<__half2*>(&v);
    h = __hmul2(__hsub2(h, off), s2);
    out[i] = *reinterpret_cast<uint32_t*>(&h);
  }
}

// Position of element k (0..15) of a 16-element chunk in the fp16 operand
// layout that the F16 kernel's A fragments read with 16-byte loads.
TMOE_DEV int f16p_pos(int k) {
  const int hi = k & 8, r = k & 7;
  return hi + ((r & 3) << 1) + (r >> 2);
}

}  // namespace

template <bool I8, int EPI>
__global__ void __launch_bounds__(256) gemm_grouped_kernel(GemmParams P) {
  using C = Cfg<I8>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tile = blockIdx.y;
  if (tile >= P.ntiles[0]) return;
  const int e = P.tile_exp[tile], row0 = P.tile_row[tile], rowend = P.offsets[e + 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp & 1, wn = warp >> 1;
  const int gq = lane >> 2, tq = lane & 3;
  const int G = P.K / kGroup;
  constexpr bool SW = EPI != kEpiStore;
  const int Ih = P.N / 2;
  const int n0 = blockIdx.x * (SW ? 64 : 128);

  auto wrow = [&](int c) -> int {
    if (!SW) return n0 + c;
    const int wnc = c >> 5, cw = c & 31;
    return (cw < 16) ? (n0 + wnc * 16 + cw) : (Ih + n0 + wnc * 16 + cw - 16);
  };
  const size_t KW = (size_t)(P.K / 8);
  const uint32_t* We = P.W + (size_t)e * P.N * KW;
  const uint16_t* ste = P.st + (size_t)e * G * P.N;
  const uint16_t* bte = P.bt + (size_t)e * G * P.N;
  const uint8_t* Abase = static_cast<const uint8_t*>(P.A);
  const size_t a_ld = (size_t)P.K * (I8 ? 1 : 2);

  // Source rows of this thread's copy assignments, fixed for the tile.
  // Rows past the expert's end read row0 (valid memory; their results are
  // never stored).
  constexpr int ach = C::A_ROW / 16;           // 16-byte chunks per row
  constexpr int AROWS = BM * ach / 256;        // A rows copied per thread
  auto src_row = [&](int r) -> int {
    int rr = row0 + r;
    if (rr >= rowend) rr = row0;
    if (!P.a_rows) return rr;
    return P.a_map ? P.a_map[P.a_rows[rr]] : P.a_rows[rr] / P.a_div;
  };
  int arow_src[AROWS];
#pragma unroll
  for (int q = 0; q < AROWS; ++q) arow_src[q] = src_row((tid + q * 256) / ach);
  const int srow_src = src_row(tid & 127);

  auto load = [&](int s, int g) {
    uint8_t* base = smem + s * C::STAGE;
#pragma unroll
    for (int q = 0; q < AROWS; ++q) {
      const int i = tid + q * 256;
      const int r = i / ach, c = i % ach;
      cp_async16(base + r * C::A_ROW + c * 16,
                 Abase + (size_t)arow_src[q] * a_ld + (size_t)g * C::A_ROW + c * 16);
    }
    {
      const int c = tid >> 1, h = tid & 1;
      cp_async16(base + C::A_BYTES + c * 32 + h * 16,
                 reinterpret_cast<const uint8_t*>(We + (size_t)wrow(c) * KW + g * 8) + h * 16);
    }
    if (tid < 32) {
      const int tb = tid >> 4, run = (tid >> 1) & 7, h = tid & 1;
      const uint16_t* tab = tb ? bte : ste;
      cp_async16(base + C::A_BYTES + C::B_BYTES + tb * (BN * 2) + run * 32 + h * 16,
                 tab + (size_t)g * P.N + wrow(run * 16) + h * 8);
    }
    {
      const int r = tid & 127;
      if (I8 || tid >= 128) {
        const float* arr = (tid < 128) ? P.asc : P.ars;
        cp_async4(base + C::A_BYTES + C::B_BYTES + C::T_BYTES + (tid >> 7) * (BM * 4) + r * 4,
                  arr + (size_t)srow_src * P.s_r + (size_t)g * P.s_g);
      }
    }
    cp_async_commit();
  };

  float acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[i][j][q] = 0.0f;

#pragma unroll
  for (int s = 0; s < C::NST - 1; ++s) {
    if (s < G) load(s, s);
    else cp_async_commit();
  }

  for (int g = 0; g < G; ++g) {
    cp_async_wait<C::NST - 2>();
    __syncthreads();
    {
      const int gl = g + C::NST - 1;
      if (gl < G) load(gl % C::NST, gl);
      else cp_async_commit();
    }
    const uint8_t* base = smem + (g % C::NST) * C::STAGE;
    const uint8_t* Bs = base + C::A_BYTES;
    const uint16_t* Ts = reinterpret_cast<const uint16_t*>(base + C::A_BYTES + C::B_BYTES);
    const float* Rs = reinterpret_cast<const float*>(base + C::A_BYTES + C::B_BYTES + C::T_BYTES);

    // per-column tables for this thread's 8 columns
    float cs[4][2], cb[4][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = wn * 32 + j * 8 + 2 * tq;
      const uint32_t s2 = *reinterpret_cast<const uint32_t*>(Ts + c);
      const uint32_t b2 = *reinterpret_cast<const uint32_t*>(Ts + BN + c);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float s = bf2f((uint16_t)(h ? (s2 >> 16) : (s2 & 0xffffu)));
        const float b = bf2f((uint16_t)(h ? (b2 >> 16) : (b2 & 0xffffu)));
        if (I8) {
          cs[j][h] = __fmul_rn(s, 0.0625f);
          cb[j][h] = bfround(__fadd_rn(b, __fmul_rn(8.0f, s)));
        } else {
          cs[j][h] = s;
          cb[j][h] = __fadd_rn(b, __fmul_rn(8.0f, s));
        }
      }
    }

    if constexpr (I8) {
      uint32_t bfr[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = wn * 32 + j * 8 + gq;
        const uint2 w2 = *reinterpret_cast<const uint2*>(Bs + col * 32 + tq * 8);
        widen_s8x16(w2.x, bfr[j][0], bfr[j][1]);
        widen_s8x16(w2.y, bfr[j][2], bfr[j][3]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = wm * 64 + i * 16 + gq;
        const uint4 alo = *reinterpret_cast<const uint4*>(base + r * C::A_ROW + tq * 16);
        const uint4 ahi = *reinterpret_cast<const uint4*>(base + (r + 8) * C::A_ROW + tq * 16);
        const float xs0 = Rs[r], xs1 = Rs[r + 8];
        const float xr0 = Rs[BM + r], xr1 = Rs[BM + r + 8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          int d[4] = {0, 0, 0, 0};
          mma_s8(d, alo.x, ahi.x, alo.y, ahi.y, bfr[j][0], bfr[j][1]);
          mma_s8(d, alo.z, ahi.z, alo.w, ahi.w, bfr[j][2], bfr[j][3]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float xsc = (q < 2) ? xs0 : xs1;
            const float xrs = (q < 2) ? xr0 : xr1;
            const float t1 = __fmul_rn((float)d[q], cs[j][q & 1]);
            acc[i][j][q] = __fmaf_rn(t1, xsc, acc[i][j][q]);
            acc[i][j][q] = __fmaf_rn(xrs, cb[j][q & 1], acc[i][j][q]);
          }
        }
      }
    } else {
      uint32_t bfr[4][8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = wn * 32 + j * 8 + gq;
        const uint2 w2 = *reinterpret_cast<const uint2*>(Bs + col * 32 + tq * 8);
        const uint16_t sraw = Ts[col];
        const __half sh = __float2half_rn(bf2f(sraw));
        const __half2 s2 = __halves2half2(sh, sh);
        dequant_f16(w2.x, s2, &bfr[j][0]);
        dequant_f16(w2.y, s2, &bfr[j][4]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = wm * 64 + i * 16 + gq;
        const uint4 a0 = *reinterpret_cast<const uint4*>(base + r * C::A_ROW + tq * 32);
        const uint4 a1 = *reinterpret_cast<const uint4*>(base + r * C::A_ROW + tq * 32 + 16);
        const uint4 b0 = *reinterpret_cast<const uint4*>(base + (r + 8) * C::A_ROW + tq * 32);
        const uint4 b1 = *reinterpret_cast<const uint4*>(base + (r + 8) * C::A_ROW + tq * 32 + 16);
        const float xr0 = Rs[BM + r], xr1 = Rs[BM + r + 8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          mma_f16(acc[i][j], a0.x, b0.x, a0.y, b0.y, bfr[j][0], bfr[j][1]);
          mma_f16(acc[i][j], a0.z, b0.z, a0.w, b0.w, bfr[j][2], bfr[j][3]);
          mma_f16(acc[i][j], a1.x, b1.x, a1.y, b1.y, bfr[j][4], bfr[j][5]);
          mma_f16(acc[i][j], a1.z, b1.z, a1.w, b1.w, bfr[j][6], bfr[j][7]);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            acc[i][j][q] = __fmaf_rn((q < 2) ? xr0 : xr1, cb[j][q & 1], acc[i][j][q]);
        }
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  if constexpr (EPI == kEpiStore) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int row = row0 + wm * 64 + i * 16 + gq + hr * 8;
        if (row >= rowend) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int col = n0 + wn * 32 + j * 8 + 2 * tq;
          const uint32_t v = (uint32_t)f2bf(acc[i][j][2 * hr]) |
                             ((uint32_t)f2bf(acc[i][j][2 * hr + 1]) << 16);
          const int orow = P.y_rows ? P.y_rows[row] : row;
          uint16_t* yrow = P.y_ptr ? P.y_ptr[orow] : P.Y + (size_t)orow * P.N;
          *reinterpret_cast<uint32_t*>(yrow + col) = v;
        }
      }
    if (P.y_ptr) __threadfence_system();   // peer stores before the kernel ends
  } else {
    // Fused SwiGLU + per-(row, 64-group) statistics of h.
    float* psum = reinterpret_cast<float*>(smem);          // [128][33]
    float* amx = psum + BM * 33;                            // [128][4]
    float* rinv = amx + BM * 4;                             // [128]
    float hv[4][2][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          hv[i][j][q] = swiglu_bf16(bfround(acc[i][j][q]), bfround(acc[i][j + 2][q]));
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int lr = wm * 64 + i * 16 + gq + hr * 8;
        float am = 0.0f;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float a = hv[i][j][2 * hr], b = hv[i][j][2 * hr + 1];
          psum[lr * 33 + wn * 8 + j * 4 + tq] = __fadd_rn(a, b);
          am = fmaxf(am, fmaxf(fabsf(a), fabsf(b)));
        }
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        if (tq == 0) amx[lr * 4 + wn] = am;
      }
    __syncthreads();
    if (tid < BM) {
      const int lr = tid;
      const float am = fmaxf(fmaxf(amx[lr * 4 + 0], amx[lr * 4 + 1]),
                             fmaxf(amx[lr * 4 + 2], amx[lr * 4 + 3]));
      const float sum = serial_butterfly32(psum + lr * 33, 1);
      const float sc = __fdiv_rn(fmaxf(am, 1e-30f), 127.0f);
      rinv[lr] = __fdiv_rn(1.0f, sc);
      const int row = row0 + lr;
      if (row < rowend) {
        const size_t o = (size_t)blockIdx.x * P.Rpad_h + row;
        if (EPI == kEpiSwigluQ8) P.hsc[o] = sc;
        P.hrs[o] = sum;
      }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int lr = wm * 64 + i * 16 + gq + hr * 8;
        const int row = row0 + lr;
        if (row >= rowend) continue;
        const float inv = rinv[lr];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int hc = n0 + wn * 16 + j * 8 + 2 * tq;
          const float a = hv[i][j][2 * hr], b = hv[i][j][2 * hr + 1];
          if (EPI == kEpiSwigluQ8) {
            const float qa = fminf(fmaxf(__fadd_rn(rintf(__fmul_rn(a, inv)), 128.0f), 0.0f), 255.0f);
            const float qb = fminf(fmaxf(__fadd_rn(rintf(__fmul_rn(b, inv)), 128.0f), 0.0f), 255.0f);
            const uint16_t pk = (uint16_t)((uint8_t)((int)qa - 128) |
                                           ((uint16_t)(uint8_t)((int)qb - 128) << 8));
            *reinterpret_cast<uint16_t*>(P.hq + (size_t)row * Ih + hc) = pk;
          } else {
            uint16_t* hp = P.h16p + (size_t)row * Ih + (hc & ~15);
            hp[f16p_pos(hc & 15)] = __half_as_ushort(__float2half_rn(a));
            hp[f16p_pos((hc + 1) & 15)] = __half_as_ushort(__float2half_rn(b));
          }
          if (P.hbf) {
            const uint32_t v = (uint32_t)f2bf(a) | ((uint32_t)f2bf(b) << 16);
            *reinterpret_cast<uint32_t*>(P.hbf + (size_t)row * Ih + hc) = v;
          }
        }
      }
  }
}

template <bool I8, int EPI>
static cudaError_t launch_one(const GemmParams& P, int maxt, cudaStream_t s) {
  using C = Cfg<I8>;
  cudaError_t err = ensure_smem_attr((const void*)gemm_grouped_kernel<I8, EPI>, C::SMEM);
  if (err != cudaSuccess) return err;
  const int gx = (EPI == kEpiStore) ? P.N / 128 : (P.N / 2) / 64;
  dim3 grid(gx, maxt);
  gemm_grouped_kernel<I8, EPI><<<grid, 256, C::SMEM, s>>>(P);
  return cudaGetLastError();
}

cudaError_t launch_gemm_grouped(bool int8, int epi, const GemmParams& P, int maxt,
                                cudaStream_t s) {
  if (maxt <= 0) return cudaSuccess;
  if (int8) {
    if (epi == kEpiStore) return launch_one<true, kEpiStore>(P, maxt, s);
    if (epi == kEpiSwigluQ8) return launch_one<true, kEpiSwigluQ8>(P, maxt, s);
    return launch_one<true, kEpiSwigluH16>(P, maxt, s);
  }
  if (epi == kEpiStore) return launch_one<false, kEpiStore>(P, maxt, s);
  if (epi == kEpiSwigluQ8) return launch_one<false, kEpiSwigluQ8>(P, maxt, s);
  return launch_one<false, kEpiSwigluH16>(P, maxt, s);
}

// fp16 operand layout for the F16 kernel: x bf16 [R,K] -> fp16 with each
// 16-element chunk permuted (f16p_pos).  Rows are independent.
__global__ void to_f16p_kernel(const uint16_t* __restrict__ x, long long n, uint16_t* __restrict__ y) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const long long base = i & ~15LL;
  const int k = (int)(i & 15);
  y[base + f16p_pos(k)] = __half_as_ushort(__float2half_rn(bf2f(x[i])));
}

cudaError_t launch_to_f16p(const uint16_t* x, long long n, uint16_t* y, cudaStream_t s) {
  if (n > 0) to_f16p_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, n, y);
  return cudaGetLastError();
}

}  // namespace tmoe
