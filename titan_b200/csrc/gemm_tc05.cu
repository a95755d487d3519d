// Expert-sorted grouped GEMM on the 5th-generation tensor cores (tcgen05,
// TMEM accumulators), sm_100a.
//
// One CTA computes a 128-row x 128-column tile of one expert over the K
// dimension, one 64-wide quantisation group per pipeline stage.  Roles
// (384 threads):
//   warp 0      allocates TMEM, issues tcgen05.mma (one elected lane) and
//               commits stage / accumulator barriers;
//   warps 1-3   producers: copy the A rows (gathered through a_rows) with
//               cp.async and widen the packed int4 B rows into fp16 in
//               registers, both into the 128B-swizzled K-major layout that the
//               MMA descriptors address; plus the per-group scalars;
//   warps 4-11  epilogue: two warps per TMEM lane quadrant, 64 columns each.
//
// Two arithmetic modes, both on kind::f16 with fp32 accumulation:
//   INT8  — the reference's int8 x int4 algebra: A holds the activation codes
//           xu - 128 and B the re-centred nibbles q - 8, both exact in fp16,
//           so each group's MMA sum is the exact integer
//           sum (xu-128)(q-8) (|sum| < 2^24).  The accumulator is
//           double-buffered in TMEM per group and rescaled by the epilogue:
//           acc = fma(D*s, xsc, acc); acc = fma(xrs, bf16(b + 8s), acc) — the
//           arithmetic of the mma.sync kernel and the oracle's re-centred
//           order, bit for bit.  (kind::i8 would halve the MMA time but its
//           s32 accumulator needs an int->float conversion per element per
//           group; the per-group rescale then costs more issue slots than the
//           MMA saves.)
//   STOCK — the bf16-activation gather: A = x in fp16, B = (q-8)*s in fp16
//           (exact), accumulated over all groups in TMEM; the bias term
//           (b + 8s) * sum_g(x) is accumulated by the epilogue in registers.
//
// Every mbarrier wait is bounded: on timeout the thread records an error in
// g_tc05_error, raises a CTA-wide abort flag and every role leaves its loop;
// TMEM is released before the kernel returns.
#include "common.cuh"
#include "tmoe_internal.h"

namespace tmoe {

__device__ int g_tc05_error = 0;

namespace tc {

constexpr int BM = 128, BN = 128;
constexpr int NST = 4;
constexpr int A_BYTES = BM * 128;                 // 64 fp16 per row per group
constexpr int B_BYTES = BN * 128;
constexpr int SC_BYTES = (2 * BM + 2 * BN) * 4;   // xsc, xrs, s, bv (fp32)
constexpr int STAGE = 35840;                      // A + B + SC rounded to 1 KB
static_assert(A_BYTES + B_BYTES + SC_BYTES <= STAGE && STAGE % 1024 == 0, "stage layout");
constexpr int BAR_OFF = NST * STAGE;
constexpr int XCH_OFF = BAR_OFF + 256;
constexpr int SMEM = XCH_OFF + BM * 36 * 4 + 1024;
constexpr int NTHREADS = 384;
constexpr int NPROD = 96;
constexpr uint32_t kSpinLimit = 1u << 22;

TMOE_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

TMOE_DEV void mbar_init(uint32_t a, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count));
}
TMOE_DEV void mbar_arrive(uint32_t a) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(a) : "memory");
}
TMOE_DEV bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; false (with the abort flag raised) on timeout or abort.
TMOE_DEV bool mbar_wait(uint32_t a, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try(a, parity)) return true;
    if (*abort_flag) return false;
    if (i > 32) __nanosleep(128);
  }
  *abort_flag = 1;
  atomicExch(&g_tc05_error, 1);
  return false;
}

TMOE_DEV uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)64 << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16, f16 x f16 -> f32, K-major A and B, M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

TMOE_DEV void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}
TMOE_DEV void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
TMOE_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
TMOE_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

TMOE_DEV void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
TMOE_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 8 nibbles (elements 0..7 of a chunk) -> 4 half2 in the pair order
// (0,4),(1,5),(2,6),(3,7): the fp16 operand layout of every A and B chunk.
TMOE_DEV uint4 widen8(uint32_t w, bool scale, __half2 s2) {
  const __half2 off = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t v = ((w >> (4 * i)) & 0x000f000fu) | 0x64006400u;
    __half2 h = __hsub2(*reinterpret_cast<__half2*>(&v), off);
    if (scale) h = __hmul2(h, s2);
    o[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// position of element k within its 8-element chunk in the operand layout
TMOE_DEV int p8(int k) { return (k & ~7) | (((k & 3) << 1) | ((k >> 2) & 1)); }

}  // namespace tc

using namespace tc;

template <bool I8, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1) gemm_tc05_kernel(GemmParams P) {
  extern __shared__ uint8_t smem_raw[];
  const int tile = blockIdx.y;
  if (tile >= P.ntiles[0]) return;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int e = P.tile_exp[tile], row0 = P.tile_row[tile], rowend = P.offsets[e + 1];
  const int G = P.K / kGroup;
  constexpr bool SW = EPI != kEpiStore;
  const int Ih = P.N / 2;
  const int n0 = blockIdx.x * (SW ? 64 : BN);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + NST), sempty0 = smem_u32(bars + 2 * NST);
  const uint32_t tfull0 = smem_u32(bars + 3 * NST), tempty0 = smem_u32(bars + 3 * NST + 2);
  const uint32_t drain = smem_u32(bars + 3 * NST + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * NST + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * NST + 6);
  float* xch = reinterpret_cast<float*>(smem + XCH_OFF);           // [128][36]

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(full0 + 8 * s, NPROD);
      mbar_init(empty0 + 8 * s, 1);
      mbar_init(sempty0 + 8 * s, 8);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    const uint32_t ncols = I8 ? 2 * BN : BN;
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)), "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto wrow = [&](int c) -> int {
    if (!SW) return n0 + c;
    const int q = c >> 5;                 // 0: gate lo, 1: up lo, 2: gate hi, 3: up hi
    const int j = c & 31;
    return ((q & 1) ? Ih : 0) + n0 + ((q >> 1) << 5) + j;
  };

  if (warp == 0) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      for (int g = 0; g < G; ++g) {
        const int s = g % NST;
        const uint32_t ph = (g / NST) & 1;
        if (!mbar_wait(full0 + 8 * s, ph, abort_flag)) break;
        const int b = I8 ? (g & 1) : 0;
        if (I8 && !mbar_wait(tempty0 + 8 * b, ((g >> 1) & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + s * STAGE);
        const uint32_t b_base = a_base + A_BYTES;
        const uint32_t d = tmem + (uint32_t)(b * BN);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16(d, sw128_desc(a_base + kk * 32), sw128_desc(b_base + kk * 32),
                  (kk > 0 || (!I8 && g > 0)) ? 1u : 0u);
        mma_commit(empty0 + 8 * s);
        if (I8) mma_commit(tfull0 + 8 * b);
      }
      if (!I8) mma_commit(tfull0);
    }
    __syncwarp();
  } else if (warp < 4) {
    // --------------------------------------------------------------- producers
    const int pt = tid - 32;
    const size_t KW = (size_t)(P.K / 8);
    const uint32_t* We = P.W + (size_t)e * P.N * KW;
    const uint16_t* ste = P.st + (size_t)e * G * P.N;
    const uint16_t* bte = P.bt + (size_t)e * G * P.N;
    const uint16_t* A = static_cast<const uint16_t*>(P.A);
    for (int g = 0; g < G; ++g) {
      const int s = g % NST;
      const uint32_t ph = ((g / NST) & 1) ^ 1;
      if (!mbar_wait(empty0 + 8 * s, ph, abort_flag)) break;
      if (!mbar_wait(sempty0 + 8 * s, ph, abort_flag)) break;
      uint8_t* sA = smem + s * STAGE;
      uint8_t* sB = sA + A_BYTES;
      float* sc = reinterpret_cast<float*>(sB + B_BYTES);   // xsc[128] xrs[128] s[128] bv[128]
      // A: 128 rows x 8 chunks of 16 B, swizzled
      for (int i = pt; i < BM * 8; i += NPROD) {
        const int r = i >> 3, c = i & 7;
        int rr = row0 + r;
        if (rr >= rowend) rr = row0;
        const int arow = P.a_rows ? P.a_rows[rr] / P.a_div : rr;
        cp_async16(sA + r * 128 + ((c ^ (r & 7)) << 4), A + (size_t)arow * P.K + g * 64 + c * 8);
      }
      cp_async_commit();
      // B: 128 rows x 2 half-rows (4 packed words each) -> 8 fp16 chunks
      for (int i = pt; i < BN * 2; i += NPROD) {
        const int r = i >> 1, hh = i & 1;
        const int wr = wrow(r);
        const uint4 w4 = ldg_nc_v4(We + (size_t)wr * KW + g * 8 + hh * 4);
        __half2 s2 = __halves2half2(__ushort_as_half(0), __ushort_as_half(0));
        if (!I8) {
          const __half sh = __float2half_rn(bf2f(ste[(size_t)g * P.N + wr]));
          s2 = __halves2half2(sh, sh);
        }
        const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = hh * 4 + j;
          *reinterpret_cast<uint4*>(sB + r * 128 + ((c ^ (r & 7)) << 4)) = widen8(ws[j], !I8, s2);
        }
      }
      // per-group scalars
      for (int i = pt; i < 2 * BM + 2 * BN; i += NPROD) {
        float v = 0.0f;
        if (i < 2 * BM) {
          const int r = i & (BM - 1);
          int rr = row0 + r;
          if (rr >= rowend) rr = row0;
          const int arow = P.a_rows ? P.a_rows[rr] / P.a_div : rr;
          const float* arr = (i < BM) ? P.asc : P.ars;
          if (I8 || i >= BM) v = arr[(size_t)arow * P.s_r + (size_t)g * P.s_g];
        } else {
          const int c = (i - 2 * BM) & (BN - 1);
          const int wr = wrow(c);
          const float sv = bf2f(ste[(size_t)g * P.N + wr]);
          if (i < 2 * BM + BN) {
            v = __fmul_rn(sv, 1.0f);
          } else {
            const float bb = __fadd_rn(bf2f(bte[(size_t)g * P.N + wr]), __fmul_rn(8.0f, sv));
            v = I8 ? bfround(bb) : bb;
          }
        }
        sc[i] = v;
      }
      cp_async_wait<0>();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(full0 + 8 * s);
    }
    cp_async_wait<0>();
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;                      // TMEM lane quadrant
    const int half = (warp - 4) >> 2;            // column half
    const int lr = q * 32 + lane;                // tile row of this thread
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    float acc[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) acc[c] = 0.0f;
    bool ok = true;
    for (int g = 0; g < G && ok; ++g) {
      const int s = g % NST;
      const uint32_t ph = (g / NST) & 1;
      if (!mbar_wait(full0 + 8 * s, ph, abort_flag)) { ok = false; break; }
      const float* sc = reinterpret_cast<const float*>(smem + s * STAGE + A_BYTES + B_BYTES);
      const float xs = sc[lr], xr = sc[BM + lr];
      const float* cs = sc + 2 * BM + 64 * half;
      const float* cb = sc + 2 * BM + BN + 64 * half;
      if (I8) {
        const int b = g & 1;
        if (!mbar_wait(tfull0 + 8 * b, (g >> 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        float d[64];
        const uint32_t ta = tmem + lane_addr + (uint32_t)(b * BN + 64 * half);
        tmem_ld16(ta, d);
        tmem_ld16(ta + 16, d + 16);
        tmem_ld16(ta + 32, d + 32);
        tmem_ld16(ta + 48, d + 48);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty0 + 8 * b);
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float t1 = __fmul_rn(d[c], cs[c]);
          acc[c] = __fmaf_rn(t1, xs, acc[c]);
          acc[c] = __fmaf_rn(xr, cb[c], acc[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) acc[c] = __fmaf_rn(xr, cb[c], acc[c]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(sempty0 + 8 * s);
    }
    if (!I8 && ok) {
      if (mbar_wait(tfull0, 0, abort_flag)) {
        tc_fence_after();
        float d[64];
        const uint32_t ta = tmem + lane_addr + (uint32_t)(64 * half);
        tmem_ld16(ta, d);
        tmem_ld16(ta + 16, d + 16);
        tmem_ld16(ta + 32, d + 32);
        tmem_ld16(ta + 48, d + 48);
        tmem_wait_ld();
        tc_fence_before();
#pragma unroll
        for (int c = 0; c < 64; ++c) acc[c] = __fadd_rn(d[c], acc[c]);
      } else {
        ok = false;
      }
    }
    const int row = row0 + lr;
    const bool live = ok && row < rowend;
    if constexpr (EPI == kEpiStore) {
      if (live) {
        const int orow = P.y_rows ? P.y_rows[row] : row;
        uint4* dst = reinterpret_cast<uint4*>(P.Y + (size_t)orow * P.N + n0 + 64 * half);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          uint4 pk;
          pk.x = (uint32_t)f2bf(acc[8 * v + 0]) | ((uint32_t)f2bf(acc[8 * v + 1]) << 16);
          pk.y = (uint32_t)f2bf(acc[8 * v + 2]) | ((uint32_t)f2bf(acc[8 * v + 3]) << 16);
          pk.z = (uint32_t)f2bf(acc[8 * v + 4]) | ((uint32_t)f2bf(acc[8 * v + 5]) << 16);
          pk.w = (uint32_t)f2bf(acc[8 * v + 6]) | ((uint32_t)f2bf(acc[8 * v + 7]) << 16);
          dst[v] = pk;
        }
      }
    } else {
      // SwiGLU of the 32 (gate, up) pairs this thread holds; h columns
      // n0 + 32*half + j.  The 64-column quantisation group spans the two
      // halves: pair sums and amax are exchanged through shared memory.
      float h[32];
      float am = 0.0f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        h[j] = swiglu_bf16(bfround(acc[j]), bfround(acc[32 + j]));
        am = fmaxf(am, fabsf(h[j]));
      }
#pragma unroll
      for (int l = 0; l < 16; ++l) xch[lr * 36 + 16 * half + l] = __fadd_rn(h[2 * l], h[2 * l + 1]);
      xch[lr * 36 + 32 + half] = am;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      const float amax = fmaxf(xch[lr * 36 + 32], xch[lr * 36 + 33]);
      const float sum = serial_butterfly32(xch + lr * 36, 1);
      const float scl = __fdiv_rn(fmaxf(amax, 1e-30f), 127.0f);
      const float inv = __fdiv_rn(1.0f, scl);
      if (live) {
        const size_t o = (size_t)blockIdx.x * P.Rpad_h + row;
        if (half == 0) {
          if (EPI == kEpiSwigluQ8) P.hsc[o] = scl;
          P.hrs[o] = sum;
        }
        uint16_t* dst = P.h16p + (size_t)row * Ih + n0 + 32 * half;
#pragma unroll
        for (int cch = 0; cch < 4; ++cch) {
          uint16_t v[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            float val = h[8 * cch + k];
            if (EPI == kEpiSwigluQ8)
              val = __fadd_rn(fminf(fmaxf(__fadd_rn(rintf(__fmul_rn(val, inv)), 128.0f), 0.0f), 255.0f),
                              -128.0f);
            v[p8(k)] = __half_as_ushort(__float2half_rn(val));
          }
          uint4 pk;
          pk.x = v[0] | ((uint32_t)v[1] << 16);
          pk.y = v[2] | ((uint32_t)v[3] << 16);
          pk.z = v[4] | ((uint32_t)v[5] << 16);
          pk.w = v[6] | ((uint32_t)v[7] << 16);
          reinterpret_cast<uint4*>(dst)[cch] = pk;
        }
        if (P.hbf) {
#pragma unroll
          for (int j = 0; j < 32; ++j) P.hbf[(size_t)row * Ih + n0 + 32 * half + j] = f2bf(h[j]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    if (*abort_flag) {
      // let any issued MMA drain before the columns are released (bounded)
      if (lane == 0) {
        mma_commit(drain);
        for (uint32_t i = 0; i < kSpinLimit && !mbar_try(drain, 0); ++i) __nanosleep(128);
      }
      __syncwarp();
    }
    tc_fence_after();
    const uint32_t ncols = I8 ? 2 * BN : BN;
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
  }
}

template <bool I8, int EPI>
static cudaError_t launch_tc05_one(const GemmParams& P, int maxt, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    cudaError_t err = cudaFuncSetAttribute(gemm_tc05_kernel<I8, EPI>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (err != cudaSuccess) return err;
    attr = true;
  }
  const int gx = (EPI == kEpiStore) ? P.N / BN : (P.N / 2) / 64;
  gemm_tc05_kernel<I8, EPI><<<dim3(gx, maxt), NTHREADS, SMEM, s>>>(P);
  return cudaGetLastError();
}

cudaError_t launch_gemm_tc05(bool int8, int epi, const GemmParams& P, int maxt, cudaStream_t s) {
  if (maxt <= 0) return cudaSuccess;
  if (int8) {
    if (epi == kEpiStore) return launch_tc05_one<true, kEpiStore>(P, maxt, s);
    if (epi == kEpiSwigluQ8) return launch_tc05_one<true, kEpiSwigluQ8>(P, maxt, s);
    return launch_tc05_one<true, kEpiSwigluH16>(P, maxt, s);
  }
  if (epi == kEpiStore) return launch_tc05_one<false, kEpiStore>(P, maxt, s);
  if (epi == kEpiSwigluQ8) return launch_tc05_one<false, kEpiSwigluQ8>(P, maxt, s);
  return launch_tc05_one<false, kEpiSwigluH16>(P, maxt, s);
}

// Operand prep for the tcgen05 GEMMs: one warp per (row, 64-group), lane l
// holds elements 2l, 2l+1.  QUANT: the int8 codes xu - 128 as fp16 plus the
// per-group scale and exact sum; otherwise x itself in fp16 plus the sum.
// Elements are stored in the (0,4,1,5,2,6,3,7) order of every 8-chunk.
template <bool QUANT>
__global__ void __launch_bounds__(256) prep_a16_kernel(const uint16_t* __restrict__ x, int R, int K,
                                                        uint16_t* __restrict__ a16,
                                                        float* __restrict__ xsc,
                                                        float* __restrict__ xrs) {
  const int lane = threadIdx.x & 31;
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int G = K / kGroup;
  if (w >= (long long)R * G) return;
  const int m = (int)(w / G), g = (int)(w % G);
  const uint32_t pr = *reinterpret_cast<const uint32_t*>(x + (size_t)m * K + g * kGroup + 2 * lane);
  float a = bf2f((uint16_t)(pr & 0xffffu)), b = bf2f((uint16_t)(pr >> 16));
  const float sum = warp_butterfly_sum(__fadd_rn(a, b));
  if (QUANT) {
    const float amax = warp_max(fmaxf(fabsf(a), fabsf(b)));
    const float sc = __fdiv_rn(fmaxf(amax, 1e-30f), 127.0f);
    const float inv = __fdiv_rn(1.0f, sc);
    a = __fadd_rn(fminf(fmaxf(__fadd_rn(rintf(__fmul_rn(a, inv)), 128.0f), 0.0f), 255.0f), -128.0f);
    b = __fadd_rn(fminf(fmaxf(__fadd_rn(rintf(__fmul_rn(b, inv)), 128.0f), 0.0f), 255.0f), -128.0f);
    if (lane == 0) xsc[(size_t)m * G + g] = sc;
  }
  if (lane == 0) xrs[(size_t)m * G + g] = sum;
  uint16_t* dst = a16 + (size_t)m * K + g * kGroup;
  const int k0 = 2 * lane;
  dst[p8(k0)] = __half_as_ushort(__float2half_rn(a));
  dst[p8(k0 + 1)] = __half_as_ushort(__float2half_rn(b));
}

cudaError_t launch_prep_a16(const uint16_t* x, int R, int K, bool quant, uint16_t* a16, float* xsc,
                            float* xrs, cudaStream_t s) {
  const long long warps = (long long)R * (K / kGroup);
  if (warps <= 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((warps * 32 + 255) / 256);
  if (quant)
    prep_a16_kernel<true><<<blocks, 256, 0, s>>>(x, R, K, a16, xsc, xrs);
  else
    prep_a16_kernel<false><<<blocks, 256, 0, s>>>(x, R, K, a16, xsc, xrs);
  return cudaGetLastError();
}

int tc05_error_flag() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc05_error, sizeof(int));
  return v;
}

}  // namespace tmoe
