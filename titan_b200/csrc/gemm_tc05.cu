// Expert-sorted grouped GEMM on the 5th-generation tensor cores (tcgen05,
// TMEM accumulators), sm_100a.
//
// One CTA computes a 128-row x 128-column tile of one expert over the K
// dimension, one 64-wide quantisation group per pipeline stage.  Roles
// (512 threads):
//   warp 0      allocates TMEM, issues tcgen05.mma (one elected lane) and
//               commits stage / accumulator barriers;
//   warps 1-7   producers: cp.async copies of the A rows (gathered through
//               a_rows), the packed int4 B rows and the scalars, LAG groups
//               ahead; then widen the current group's B rows into fp16, both
//               operands in the 128B-swizzled K-major layout that the MMA
//               descriptors address;
//   warps 8-15  epilogue: two warps per TMEM lane quadrant, 64 columns each.
//
// Two arithmetic modes, both on kind::f16 with fp32 accumulation:
//   INT8  — the reference's int8 x int4 algebra: A holds the activation codes
//           xu - 128 and B the re-centred nibbles q - 8, both exact in fp16,
//           so each group's MMA sum is the exact integer
//           sum (xu-128)(q-8) (|sum| < 2^24).  The accumulator is
//           double-buffered in TMEM per group and rescaled by the epilogue:
//           acc = fma(D*s, xsc, acc); acc = fma(xrs, bf16(b + 8s), acc) — the
//           arithmetic of the mma.sync kernel and the oracle's re-centred
//           order, bit for bit.  When every scale of the CTA's columns lies in
//           fp16's normal range, B carries (q-8)*s instead (still exact) and
//           the MMA returns D*s itself, saving one multiply per element per
//           group with identical bits.  (kind::i8 would halve the MMA time but its
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
#include "tc05.cuh"
#include "tmoe_internal.h"

namespace tmoe {

__device__ int g_tc05_error = 0;

namespace tc {

constexpr int BM = 128, BN = 128;
constexpr int NST = 5;                            // pipeline stages
constexpr int LAG = 3;                            // groups in flight ahead of the widening
constexpr int A_BYTES = BM * 128;                 // 64 fp16 per row per group
constexpr int B_BYTES = BN * 128;
constexpr int SC_BYTES = (2 * BM + 2 * BN) * 4;   // xsc, xrs, s, bv (fp32)
constexpr int RAWB_BYTES = BN * 32;               // packed int4 rows of the group
constexpr int RAWT_BYTES = 2 * BN * 2;            // bf16 scales and biases of the group
constexpr int STAGE = 39936;                      // A + B + SC + RAWB + RAWT rounded to 1 KB
static_assert(A_BYTES + B_BYTES + SC_BYTES + RAWB_BYTES + RAWT_BYTES <= STAGE &&
                  STAGE % 1024 == 0, "stage layout");
static_assert(LAG < NST, "the producer refills a stage the MMA finished two groups ago");
constexpr int BAR_OFF = NST * STAGE;
constexpr int AROW_OFF = BAR_OFF + 256;           // source row of each tile row
constexpr int XCH_OFF = AROW_OFF + BM * 4;
constexpr int SMEM = XCH_OFF + BM * 36 * 4 + 1024;
static_assert(SMEM <= 232448, "shared memory per CTA");
constexpr int NTHREADS = 512;
constexpr int NPROD = 224;                       // warps 1-7
// Bounded wait recording into this kernel's error flag.
TMOE_DEV bool mbar_wait(uint32_t a, uint32_t parity, volatile int* abort_flag) {
  return tc::mbar_wait(a, parity, abort_flag, &g_tc05_error);
}

// Named barrier over the producer warps that also ANDs a predicate.
TMOE_DEV bool producers_and(bool v) {
  uint32_t r;
  asm volatile(
      "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.and.pred q, 2, %2, p; selp.u32 %0, 1, 0, q; }"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(NPROD)
      : "memory");
  return r != 0;
}

// kind::f16, f16 x f16 -> f32, K-major A and B, M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

TMOE_DEV void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  tc::mma_f16(tmem_d, adesc, bdesc, kIdesc, accumulate);
}

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
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + NST);
  const uint32_t tfull0 = smem_u32(bars + 3 * NST), tempty0 = smem_u32(bars + 3 * NST + 2);
  const uint32_t drain = smem_u32(bars + 3 * NST + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * NST + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * NST + 6);
  int* prescale_flag = reinterpret_cast<int*>(bars + 3 * NST + 7);
  float* xch = reinterpret_cast<float*>(smem + XCH_OFF);           // [128][36]

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(full0 + 8 * s, NPROD);
      mbar_init(empty0 + 8 * s, 9);         // the MMA commit + the 8 epilogue warps
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
  } else if (warp < 8) {
    // --------------------------------------------------------------- producers
    // Copies for group g + LAG are issued (cp.async: A rows, packed B rows,
    // row scalars, column tables) before group g is widened, so LAG groups of
    // loads are in flight behind the one being converted.
    const int pt = tid - 32;
    const size_t KW = (size_t)(P.K / 8);
    const uint32_t* We = P.W + (size_t)e * P.N * KW;
    const uint16_t* ste = P.st + (size_t)e * G * P.N;
    const uint16_t* bte = P.bt + (size_t)e * G * P.N;
    const uint16_t* A = static_cast<const uint16_t*>(P.A);
    int* arow_s = reinterpret_cast<int*>(smem + AROW_OFF);
    for (int r = pt; r < BM; r += NPROD) {
      int rr = row0 + r;
      if (rr >= rowend) rr = row0;           // rows past the expert's end: any valid row
      arow_s[r] = !P.a_rows ? rr : (P.a_map ? P.a_map[P.a_rows[rr]] : P.a_rows[rr] / P.a_div);
    }
    // INT8: B can carry the scale, (q - 8) * s exact in fp16, when every scale
    // of the tile is 0 or inside [2^-14, 2^12): then the MMA returns D * s
    // exactly (|D| <= 2^16, so D * s needs at most 24 bits).  One flag per CTA.
    bool safe = true;
    {
      for (int i = pt; i < G * 16; i += NPROD) {
        const int g = i >> 4, cc = i & 15;
        const uint4 v = *reinterpret_cast<const uint4*>(ste + (size_t)g * P.N + wrow(cc * 8));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t b = (w[j >> 1] >> (16 * (j & 1))) & 0xffffu;
          const uint32_t ex = (b >> 7) & 0xffu;
          safe = safe && (((b & 0x7fffu) == 0u) || (ex >= 113u && ex <= 138u));
        }
      }
    }
    const bool prescale = producers_and(safe);
    if (pt == 0) *prescale_flag = prescale ? 1 : 0;
    // STOCK accumulates every group in TMEM, so B must carry the scale: a
    // tile whose scales fall outside fp16's exact range is reported (error 2,
    // tmoe_device_status) — the swap-AB kernel with row normalisers has
    // no such limit.
    if (!I8 && !prescale && pt == 0) atomicExch(&g_tc05_error, 2);
    const bool scale_b = !I8 || prescale;

    // Per-thread copy plan, fixed across groups (addresses advance per group).
    constexpr int NA = (BM * 8 + NPROD - 1) / NPROD;
    constexpr int NB = (BN * 2 + NPROD - 1) / NPROD;
    constexpr int NS = (2 * BM + NPROD - 1) / NPROD;
    const uint16_t* a_src[NA];
    uint32_t a_dst[NA];
#pragma unroll
    for (int j = 0; j < NA; ++j) {
      const int i = min(pt + j * NPROD, BM * 8 - 1);
      const int r = i >> 3, c = i & 7;
      a_src[j] = A + (size_t)arow_s[r] * P.K + c * 8;
      a_dst[j] = r * 128 + ((c ^ (r & 7)) << 4);
    }
    const uint32_t* b_src[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      const int i = min(pt + j * NPROD, BN * 2 - 1);
      b_src[j] = We + (size_t)wrow(i >> 1) * KW + (i & 1) * 4;
    }
    const float* s_src[NS];
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const int i = min(pt + j * NPROD, 2 * BM - 1);
      const float* arr = (i < BM) ? P.asc : P.ars;
      s_src[j] = (arr ? arr : P.ars) + (size_t)arow_s[i & (BM - 1)] * P.s_r;
    }
    const uint16_t* t_src = (pt < 32) ? ((pt >> 4) ? bte : ste) + wrow((pt & 15) * 8) : ste;

    auto issue = [&](int g) {
      uint8_t* sA = smem + (g % NST) * STAGE;
      float* sc = reinterpret_cast<float*>(sA + A_BYTES + B_BYTES);
      uint8_t* raw = reinterpret_cast<uint8_t*>(sc) + SC_BYTES;
      uint8_t* rawt = raw + RAWB_BYTES;
#pragma unroll
      for (int j = 0; j < NA; ++j)
        if (pt + j * NPROD < BM * 8) cp_async16(sA + a_dst[j], a_src[j] + g * 64);
#pragma unroll
      for (int j = 0; j < NB; ++j)
        if (pt + j * NPROD < BN * 2) cp_async16_l2pf(raw + (pt + j * NPROD) * 16, b_src[j] + g * 8);
#pragma unroll
      for (int j = 0; j < NS; ++j) {
        const int i = pt + j * NPROD;
        if (i < 2 * BM && (I8 || i >= BM)) cp_async4(sc + i, s_src[j] + (size_t)g * P.s_g);
      }
      if (pt < 32) cp_async16(rawt + pt * 16, t_src + (size_t)g * P.N);
    };
    auto stage_free = [&](int g) -> bool {
      const int s = g % NST;
      const uint32_t ph = ((g / NST) & 1) ^ 1;
      return mbar_wait(empty0 + 8 * s, ph, abort_flag);
    };

    for (int g = 0; g < LAG; ++g) {   // the first NST stages start free; one
      if (g < G) issue(g);             // commit group per group index keeps the
      cp_async_commit();               // wait_group<LAG> count exact when G < LAG
    }
    for (int g = 0; g < G; ++g) {
      const int gi = g + LAG;
      bool ok = true;
      if (gi < G) {
        ok = stage_free(gi);
        if (ok) issue(gi);
      }
      cp_async_commit();
      cp_async_wait<LAG>();                    // this thread's copies of group g landed
      if (!producers_and(ok && !*abort_flag)) break;   // ... and every producer's
      const int s = g % NST;
      uint8_t* sB = smem + s * STAGE + A_BYTES;
      float* sc = reinterpret_cast<float*>(sB + B_BYTES);
      const uint8_t* raw = reinterpret_cast<const uint8_t*>(sc) + SC_BYTES;
      const uint16_t* rawt = reinterpret_cast<const uint16_t*>(raw + RAWB_BYTES);
      // B: 128 rows x 2 half-rows (4 packed words each) -> 8 fp16 chunks
      for (int i = pt; i < BN * 2; i += NPROD) {
        const int r = i >> 1, hh = i & 1;
        const uint4 w4 = *reinterpret_cast<const uint4*>(raw + r * 32 + hh * 16);
        const __half sh = __float2half_rn(bf2f(rawt[r]));
        const __half2 s2 = __halves2half2(sh, sh);
        const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = hh * 4 + j;
          *reinterpret_cast<uint4*>(sB + r * 128 + ((c ^ (r & 7)) << 4)) = widen8(ws[j], scale_b, s2);
        }
      }
      // column scalars: s and the folded bias b + 8s
      for (int c = pt; c < BN; c += NPROD) {
        const float sv = bf2f(rawt[c]);
        const float bb = __fadd_rn(bf2f(rawt[BN + c]), __fmul_rn(8.0f, sv));
        sc[2 * BM + c] = sv;
        sc[2 * BM + BN + c] = I8 ? bfround(bb) : bb;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(full0 + 8 * s);
    }
    cp_async_wait<0>();
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;                      // TMEM lane quadrant
    const int half = (warp - 8) >> 2;            // column half
    const int lr = q * 32 + lane;                // tile row of this thread
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    float acc[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) acc[c] = 0.0f;
    bool ok = true;
    bool prescaled = false;
    for (int g = 0; g < G && ok; ++g) {
      const int s = g % NST;
      const uint32_t ph = (g / NST) & 1;
      if (!mbar_wait(full0 + 8 * s, ph, abort_flag)) { ok = false; break; }
      if (g == 0) prescaled = *reinterpret_cast<volatile int*>(prescale_flag) != 0;
      const float* sc = reinterpret_cast<const float*>(smem + s * STAGE + A_BYTES + B_BYTES);
      const float xs = sc[lr], xr = sc[BM + lr];
      const float* cs = sc + 2 * BM + 64 * half;
      const float* cb = sc + 2 * BM + BN + 64 * half;
      if (I8) {
        const int b = g & 1;
        if (!mbar_wait(tfull0 + 8 * b, (g >> 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ta = tmem + lane_addr + (uint32_t)(b * BN + 64 * half);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {       // two 32-column halves: fewer registers
          float d[32];
          tmem_ld16(ta + 32 * hh, d);
          tmem_ld16(ta + 32 * hh + 16, d + 16);
          tmem_wait_ld();
          if (hh == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty0 + 8 * b);
          }
          // column scalars read 4 at a time (16-byte aligned in the stage)
          const float4* cb4 = reinterpret_cast<const float4*>(cb + 32 * hh);
          const float4* cs4 = reinterpret_cast<const float4*>(cs + 32 * hh);
          if (prescaled) {                     // d = D * s already (exact)
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
              const float4 b4 = cb4[c4];
              const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int c = 4 * c4 + q;
                acc[32 * hh + c] = __fmaf_rn(d[c], xs, acc[32 * hh + c]);
                acc[32 * hh + c] = __fmaf_rn(xr, bv[q], acc[32 * hh + c]);
              }
            }
          } else {
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
              const float4 b4 = cb4[c4], s4 = cs4[c4];
              const float bv[4] = {b4.x, b4.y, b4.z, b4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int c = 4 * c4 + q;
                const float t1 = __fmul_rn(d[c], sv[q]);
                acc[32 * hh + c] = __fmaf_rn(t1, xs, acc[32 * hh + c]);
                acc[32 * hh + c] = __fmaf_rn(xr, bv[q], acc[32 * hh + c]);
              }
            }
          }
        }
      } else {
        const float4* cb4 = reinterpret_cast<const float4*>(cb);
#pragma unroll
        for (int c4 = 0; c4 < 16; ++c4) {
          const float4 b4 = cb4[c4];
          acc[4 * c4] = __fmaf_rn(xr, b4.x, acc[4 * c4]);
          acc[4 * c4 + 1] = __fmaf_rn(xr, b4.y, acc[4 * c4 + 1]);
          acc[4 * c4 + 2] = __fmaf_rn(xr, b4.z, acc[4 * c4 + 2]);
          acc[4 * c4 + 3] = __fmaf_rn(xr, b4.w, acc[4 * c4 + 3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * s);
    }
    if (!I8 && ok) {
      if (mbar_wait(tfull0, 0, abort_flag)) {
        tc_fence_after();
        const uint32_t ta = tmem + lane_addr + (uint32_t)(64 * half);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float d[32];
          tmem_ld16(ta + 32 * hh, d);
          tmem_ld16(ta + 32 * hh + 16, d + 16);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) acc[32 * hh + c] = __fadd_rn(d[c], acc[32 * hh + c]);
        }
        tc_fence_before();
      } else {
        ok = false;
      }
    }
    const int row = row0 + lr;
    const bool live = ok && row < rowend;
    if constexpr (EPI == kEpiStore) {
      if (live) {
        const int orow = P.y_rows ? P.y_rows[row] : row;
        uint16_t* yrow = P.y_ptr ? P.y_ptr[orow] : P.Y + (size_t)orow * P.N;
        uint4* dst = reinterpret_cast<uint4*>(yrow + n0 + 64 * half);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          uint4 pk;
          pk.x = (uint32_t)f2bf(acc[8 * v + 0]) | ((uint32_t)f2bf(acc[8 * v + 1]) << 16);
          pk.y = (uint32_t)f2bf(acc[8 * v + 2]) | ((uint32_t)f2bf(acc[8 * v + 3]) << 16);
          pk.z = (uint32_t)f2bf(acc[8 * v + 4]) | ((uint32_t)f2bf(acc[8 * v + 5]) << 16);
          pk.w = (uint32_t)f2bf(acc[8 * v + 6]) | ((uint32_t)f2bf(acc[8 * v + 7]) << 16);
          dst[v] = pk;
        }
        // stores into other GPUs' memory (the expert-parallel return) are
        // performed at system scope before this kernel ends, ahead of the
        // flag the next launch posts
        if (P.y_ptr) __threadfence_system();
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
  cudaError_t err = ensure_smem_attr((const void*)gemm_tc05_kernel<I8, EPI>, SMEM);
  if (err != cudaSuccess) return err;
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
  if (!QUANT) {
    // x itself becomes the fp16 operand: it overflows past 65504, and a group
    // lying wholly below fp16's normal range keeps too few bits
    const float gm = warp_max(fmaxf(fabsf(a), fabsf(b)));
    if (lane == 0 && (gm >= 65504.0f || (gm > 0.0f && gm < 6.103515625e-05f)))
      atomicExch(&g_tc05_error, 2);
  }
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
