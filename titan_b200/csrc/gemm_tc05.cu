// Expert-sorted grouped GEMM on the 5th-generation tensor cores (tcgen05,
// TMEM accumulators), sm_100a.
//
// One CTA computes a 128-row x 128-column tile of one expert over the K
// dimension, one 64-wide quantisation group per pipeline stage.  Roles
// (512 threads):
//   warp 0      loader, LAG groups ahead: TMA loads (no multicast) of the
//               packed int4 weight rows and of the group's scale / bias
//               segments; cp.async copies of the gathered A rows (through
//               a_rows) into the 128B-swizzled K-major layout and of the row
//               scalars;
//   warp 1      allocates TMEM, issues tcgen05.mma (one elected lane) and
//               commits stage / accumulator barriers;
//   warps 2-7   converters: widen the group's packed rows into fp16 B (same
//               swizzled layout) and write the fp32 column scalars;
//   warps 8-15  epilogue: two warps per TMEM lane quadrant, 64 columns each;
//               the per-group rescale issues as packed f32x2 FMAs.
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
constexpr int NA = 3;                             // activation tiles (one group each)
constexpr int NB = 3;                             // widened weight tiles (one group each)
constexpr int NQ = 2;                             // packed stages (4 groups each)
constexpr int ND = 4;                             // TMEM accumulator buffers (128 columns each)
constexpr int NCS = 8;                            // column-scalar slots (one group each)
constexpr int kMaxG = 48;                         // K <= 3072: scale / bias tables held whole
constexpr int A_BYTES = BM * 128;                 // 128 rows x 64 fp16, 128B-swizzled
constexpr int B_BYTES = BN * 128;
constexpr int CS_BYTES = 2 * BN * 4;              // column s and b + 8s (fp32) of a group
constexpr int QW_BYTES = 4 * 32 * 128;            // 4 segments x [32 rows][4 groups x 32 B], SW128
constexpr int QS_BYTES = BM * 16;                 // one row scalar x [128 rows][4 groups]
constexpr int Q_BYTES = QW_BYTES + 2 * QS_BYTES;  // + xsc, xrs
constexpr int A_OFF = 0;
constexpr int B_OFF = A_OFF + NA * A_BYTES;
constexpr int Q_OFF = B_OFF + NB * B_BYTES;
constexpr int CS_OFF = Q_OFF + NQ * Q_BYTES;
constexpr int TB_OFF = CS_OFF + NCS * CS_BYTES;    // 2 x 8 table boxes [G][32] bf16 (s x 4, b x 4)
constexpr int TB_BYTES = 8 * 64 * kMaxG;          // one work item's tables
constexpr int XCH_OFF = TB_OFF + 2 * TB_BYTES;
constexpr int BAR_OFF = XCH_OFF + BM * 36 * 4;
constexpr int SMEM = BAR_OFF + 512 + 1024;        // + alignment slack
static_assert(A_OFF % 1024 == 0 && B_OFF % 1024 == 0 && Q_OFF % 1024 == 0 && Q_BYTES % 1024 == 0 &&
                  CS_OFF % 128 == 0 && TB_OFF % 128 == 0 && BAR_OFF % 8 == 0,
              "TMA / UMMA tiles 1024-byte aligned, other TMA destinations 128-byte aligned");
static_assert(SMEM <= 232448, "shared memory per CTA");
constexpr int NTHREADS = 512;
constexpr int NCONV = 128;                        // converter warps 4-7 (one per SM sub-partition)
// barrier indices (uint64 each) at BAR_OFF
constexpr int B_AF = 0, B_AE = B_AF + NA, B_BF = B_AE + NA, B_BE = B_BF + NB, B_QF = B_BE + NB,
              B_QE = B_QF + NQ, B_CSF = B_QE + NQ, B_CSE = B_CSF + NCS, B_TF = B_CSE + NCS,
              B_TE = B_TF + ND, B_TBF = B_TE + ND,
              B_TBE = B_TBF + 2, B_DRAIN = B_TBE + 2, B_SLOT = B_DRAIN + 1,
              B_ABORT = B_SLOT + 1, B_PRESCALE = B_ABORT + 1;   // 4 prescale flags (ints)
static_assert((B_PRESCALE + 2) * 8 <= 512, "barrier area");
// Bounded wait recording into this kernel's error flag.
TMOE_DEV bool mbar_wait(uint32_t a, uint32_t parity, volatile int* abort_flag) {
  return tc::mbar_wait(a, parity, abort_flag, &g_tc05_error);
}

// Named barrier over the converter warps that also ANDs a predicate.
TMOE_DEV bool converters_and(bool v) {
  uint32_t r;
  asm volatile(
      "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.and.pred q, 2, %2, p; selp.u32 %0, 1, 0, q; }"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(NCONV)
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

struct Tc05Maps {
  CUtensorMap a;    // [rows][K] fp16 operand, box 64 x 128, 128B swizzle
  CUtensorMap xs;   // [rows][srow] fp32 row scales, box 4 x 128
  CUtensorMap xr;   // [rows][srow] fp32 row sums, box 4 x 128
  CUtensorMap w;    // [E*N][K/8] packed int4 words, box 32 x 32, 128B swizzle
  CUtensorMap s;    // [E*G][N] bf16 scales, box 32 x G
  CUtensorMap b;    // [E*G][N] bf16 biases, box 32 x G
};

template <bool I8, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_tc05_kernel(const __grid_constant__ GemmParams P, const __grid_constant__ Tc05Maps M) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = P.K / kGroup;
  constexpr bool SW = EPI != kEpiStore;
  const int Ih = P.N / 2;
  const int gx = SW ? Ih / 64 : P.N / BN;     // column blocks per tile
  const int nitems = P.ntiles[0] * gx;        // work items: (row tile, column block)
  const int TBS = (64 * G + 127) & ~127;      // bytes per table box, 128-byte aligned

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  auto bar = [&](int i) -> uint32_t { return smem_u32(bars + i); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_SLOT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + B_ABORT);
  int* prescale_flag = reinterpret_cast<int*>(bars + B_PRESCALE);   // [4], by item
  float* xch = reinterpret_cast<float*>(smem + XCH_OFF);           // [128][36]

  if (tid == 0) {
    for (int i = 0; i < NA; ++i) {
      mbar_init(bar(B_AF + i), 1);          // the loader's expect_tx + the tile's bytes
      mbar_init(bar(B_AE + i), 1);          // MMA commit
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(bar(B_BF + i), NCONV / 32); // one arrival per converter warp
      mbar_init(bar(B_BE + i), 1);          // MMA commit
    }
    for (int i = 0; i < NCS; ++i) {
      mbar_init(bar(B_CSF + i), NCONV / 32);  // converters wrote the group's column scalars
      mbar_init(bar(B_CSE + i), 8);           // the 8 epilogue warps read them
    }
    for (int i = 0; i < ND; ++i) {
      mbar_init(bar(B_TF + i), 1);
      mbar_init(bar(B_TE + i), 8);
    }
    for (int i = 0; i < NQ; ++i) {
      mbar_init(bar(B_QF + i), 1);
      mbar_init(bar(B_QE + i), NCONV / 32 + 8);   // converters (packed rows), epilogue (row scalars)
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(B_TBF + b), 1);
      mbar_init(bar(B_TBE + b), NCONV / 32);
    }
    mbar_init(bar(B_DRAIN), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&M.a);
    tma_prefetch_desc(&M.w);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)), "r"(ND * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // weight row of B-tile row c of column block nb: the SwiGLU tiles
  // interleave 32-row segments (gate lo, up lo, gate hi, up hi) so that each
  // epilogue half holds matching gate and up columns
  auto wrow = [&](int nb, int c) -> int {
    const int n0 = nb * (SW ? 64 : BN);
    if (!SW) return n0 + c;
    const int q = c >> 5;
    const int j = c & 31;
    return ((q & 1) ? Ih : 0) + n0 + ((q >> 1) << 5) + j;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- loader
    // One thread issues every copy, all TMA (no multicast): per work item the
    // scale / bias tables (double-buffered across items), per group the 16 KB
    // activation tile, per 4 groups the packed weight rows (4 x 4 KB) and the
    // row scalars (2 x 2 KB).  x of every box is a multiple of 16 bytes; rows
    // past the operand's end read zeros.  Ring phases count across items.
    if (lane == 0) {
      const uint32_t qtx = (uint32_t)QW_BYTES + (I8 ? 2u : 1u) * (uint32_t)QS_BYTES;
      int ga = 0, gq = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++it) {
        const int tile = item / gx, nb = item - tile * gx;
        const int e = P.tile_exp[tile], row0 = P.tile_row[tile];
        const int tb = it & 1;
        if (!(ok = mbar_wait(bar(B_TBE + tb), ((it >> 1) & 1) ^ 1, abort_flag))) break;
        mbar_expect_tx(bar(B_TBF + tb), 8u * 64u * (uint32_t)G);
        uint8_t* tbs = smem + TB_OFF + tb * TB_BYTES;
        for (int seg = 0; seg < 4; ++seg) {
          const int wr = wrow(nb, seg * 32);
          tma_load_2d(smem_u32(tbs + seg * TBS), &M.s, wr, e * G, bar(B_TBF + tb));
          tma_load_2d(smem_u32(tbs + (4 + seg) * TBS), &M.b, wr, e * G, bar(B_TBF + tb));
        }
        for (int g = 0; g < G && ok; ++g) {
          if ((g & 3) == 0) {
            const int sq = gq % NQ;
            if (!(ok = mbar_wait(bar(B_QE + sq), ((gq / NQ) & 1) ^ 1, abort_flag))) break;
            const uint32_t qb = bar(B_QF + sq);
            uint8_t* qs = smem + Q_OFF + sq * Q_BYTES;
            mbar_expect_tx(qb, qtx);
            for (int seg = 0; seg < 4; ++seg)
              tma_load_2d(smem_u32(qs + seg * 4096), &M.w, (g >> 2) * 32,
                          e * P.N + wrow(nb, seg * 32), qb);
            if (I8) tma_load_2d(smem_u32(qs + QW_BYTES), &M.xs, (g >> 2) * 4, row0, qb);
            tma_load_2d(smem_u32(qs + QW_BYTES + QS_BYTES), &M.xr, (g >> 2) * 4, row0, qb);
            ++gq;
          }
          const int sa = ga % NA;
          if (!(ok = mbar_wait(bar(B_AE + sa), ((ga / NA) & 1) ^ 1, abort_flag))) break;
          mbar_expect_tx(bar(B_AF + sa), A_BYTES);
          tma_load_2d(smem_u32(smem + A_OFF + sa * A_BYTES), &M.a, g * 64, row0, bar(B_AF + sa));
          ++ga;
        }
      }
      // copies still in flight (after an abort) land before the CTA exits
      auto drain_wait = [&](uint32_t b, uint32_t par) {
        for (uint32_t i = 0; i < kSpinLimit && !mbar_try(b, par); ++i) __nanosleep(128);
      };
      for (int i = it > 2 ? it - 2 : 0; i < it; ++i) drain_wait(bar(B_TBF + (i & 1)), (i >> 1) & 1);
      for (int g = ga > NA ? ga - NA : 0; g < ga; ++g) drain_wait(bar(B_AF + g % NA), (g / NA) & 1);
      for (int q = gq > NQ ? gq - NQ : 0; q < gq; ++q) drain_wait(bar(B_QF + q % NQ), (q / NQ) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int ga = 0, gb = 0, gt = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
        if (!I8) {   // STOCK: one accumulator buffer per item
          if (!(ok = mbar_wait(bar(B_TE + gt % ND), ((gt / ND) & 1) ^ 1, abort_flag))) break;
        }
        for (int g = 0; g < G; ++g) {
          const int sa = ga % NA, sb = gb % NB;
          if (!(ok = mbar_wait(bar(B_AF + sa), (ga / NA) & 1, abort_flag))) break;
          if (!(ok = mbar_wait(bar(B_BF + sb), (gb / NB) & 1, abort_flag))) break;
          if (I8 && !(ok = mbar_wait(bar(B_TE + gt % ND), ((gt / ND) & 1) ^ 1, abort_flag))) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + A_OFF + sa * A_BYTES);
          const uint32_t b_base = smem_u32(smem + B_OFF + sb * B_BYTES);
          const uint32_t d = tmem + (uint32_t)((gt % ND) * BN);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16(d, sw128_desc(a_base + kk * 32), sw128_desc(b_base + kk * 32),
                    (kk > 0 || (!I8 && g > 0)) ? 1u : 0u);
          mma_commit(bar(B_AE + sa));
          mma_commit(bar(B_BE + sb));
          ++ga;
          ++gb;
          if (I8) {
            mma_commit(bar(B_TF + gt % ND));
            ++gt;
          }
        }
        if (!I8 && ok) {
          mma_commit(bar(B_TF + gt % ND));
          ++gt;
        }
      }
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------- converters
    // Thread ct widens B-tile row ct of each group: its 8 packed words (two
    // 16-byte loads from the swizzled packed stage), one scale, eight fp16
    // chunks into the 128B-swizzled K-major B tile — conflict-free on both
    // sides (8 consecutive rows touch 8 different 16-byte slots) — and the
    // fp32 scalars of column ct.  Warps 2-3 stay idle.
    const int ct = tid - 128;
    int gb = 0, gq = 0, it = 0;
    bool ok = true;
    // Every converter thread reaches the same named barriers in the same
    // order: a failed wait only ends the item, and the next item's barrier
    // ends the loop for all of them at once.
    for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++it) {
      const int tb = it & 1;
      const bool tok = ok && mbar_wait(bar(B_TBF + tb), (it >> 1) & 1, abort_flag);
      if (!converters_and(tok)) {
        ok = false;
        break;
      }
      const uint8_t* tbs = smem + TB_OFF + tb * TB_BYTES;
      auto tab = [&](int which, int g, int c) -> uint16_t {   // which: 0 = s, 1 = b
        return *reinterpret_cast<const uint16_t*>(tbs + (which * 4 + (c >> 5)) * TBS + g * 64 +
                                                  (c & 31) * 2);
      };
      // INT8: B can carry the scale, (q - 8) * s exact in fp16, when every
      // scale of the item is 0 or inside [2^-14, 2^12): then the MMA returns
      // D * s exactly (|D| <= 2^16, so D * s needs at most 24 bits).
      bool safe = true;
      for (int g = 0; g < G; ++g) {
        const uint32_t bv = tab(0, g, ct);
        const uint32_t ex = (bv >> 7) & 0xffu;
        safe = safe && (((bv & 0x7fffu) == 0u) || (ex >= 113u && ex <= 138u));
      }
      const bool prescale = converters_and(safe);
      if (ct == 0) prescale_flag[it & 3] = prescale ? 1 : 0;
      // STOCK accumulates every group in TMEM, so B must carry the scale: an
      // item whose scales fall outside fp16's exact range is reported (error
      // 2, tmoe_device_status) — the swap-AB kernel with row normalisers has
      // no such limit.
      if (!I8 && !prescale && ct == 0) atomicExch(&g_tc05_error, 2);
      const bool scale_b = !I8 || prescale;
      const int r = ct, r7 = r & 7;
      const uint32_t qrow = (r >> 5) * 4096 + (r & 31) * 128;   // row in the packed stage
      for (int g = 0; g < G; ++g) {
        const int sq = gq % NQ, sb = gb % NB, gg = g & 3;
        if (!(ok = mbar_wait(bar(B_QF + sq), (gq / NQ) & 1, abort_flag))) break;
        if (!(ok = mbar_wait(bar(B_BE + sb), ((gb / NB) & 1) ^ 1, abort_flag))) break;
        const int sc = gb % NCS;
        if (!(ok = mbar_wait(bar(B_CSE + sc), ((gb / NCS) & 1) ^ 1, abort_flag))) break;
        const uint8_t* qs = smem + Q_OFF + sq * Q_BYTES + qrow;
        uint8_t* sB = smem + B_OFF + sb * B_BYTES + r * 128;
        const uint4 w0 = *reinterpret_cast<const uint4*>(qs + (((2 * gg) ^ r7) << 4));
        const uint4 w1 = *reinterpret_cast<const uint4*>(qs + (((2 * gg + 1) ^ r7) << 4));
        const uint16_t sbits = tab(0, g, r);
        const __half sh = __float2half_rn(bf2f(sbits));
        const __half2 s2 = __halves2half2(sh, sh);
        const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(sB + ((c ^ r7) << 4)) = widen8(wv[c], scale_b, s2);
        // column scalars: s and the folded bias b + 8s
        {
          const float sv = bf2f(sbits);
          const float bb = __fadd_rn(bf2f(tab(1, g, r)), __fmul_rn(8.0f, sv));
          float* cs = reinterpret_cast<float*>(smem + CS_OFF + sc * CS_BYTES);
          cs[r] = sv;
          cs[BN + r] = I8 ? bfround(bb) : bb;
        }
        // each writer makes its stores visible to the async proxy; one
        // arrival per warp
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar(B_BF + sb));
          mbar_arrive(bar(B_CSF + sc));
          if (gg == 3 || g == G - 1) mbar_arrive(bar(B_QE + sq));
          if (g == G - 1) mbar_arrive(bar(B_TBE + tb));   // this item's tables consumed
        }
        ++gb;
        if (gg == 3 || g == G - 1) ++gq;
      }
    }
  } else if (warp >= 8) {
    // ---------------------------------------------------------------- epilogue
    // Every epilogue warp walks every item (after a failed wait it skips the
    // waits and stores nothing), so the named barriers of the SwiGLU tail are
    // reached by all 256 threads the same number of times.
    const int q = warp & 3;                      // TMEM lane quadrant
    const int half = (warp - 8) >> 2;            // column half
    const int lr = q * 32 + lane;                // tile row of this thread
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    int gb = 0, gq = 0, gt = 0, it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++it) {
      const int tile = item / gx, nb = item - tile * gx;
      const int e = P.tile_exp[tile], row0 = P.tile_row[tile], rowend = P.offsets[e + 1];
      const int n0 = nb * (SW ? 64 : BN);
      // accumulators as column pairs: the per-group rescale issues as packed
      // f32x2 FMAs (each component rounds exactly as a scalar fma.rn)
      float2 acc2[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) acc2[c] = make_float2(0.0f, 0.0f);
      auto acc = [&](int c) -> float { return (c & 1) ? acc2[c >> 1].y : acc2[c >> 1].x; };
      bool prescaled = false;
      for (int g = 0; g < G; ++g) {
        const int sq = gq % NQ, sc = gb % NCS, gg = g & 3;
        const bool qend = gg == 3 || g == G - 1;
        // row scalars of the packed stage (TMA), column scalars of the group
        // (converters)
        if (ok) ok = mbar_wait(bar(B_QF + sq), (gq / NQ) & 1, abort_flag) &&
                     mbar_wait(bar(B_CSF + sc), (gb / NCS) & 1, abort_flag);
        if (ok) {
          if (g == 0) prescaled = reinterpret_cast<volatile int*>(prescale_flag)[it & 3] != 0;
          const float* qsc = reinterpret_cast<const float*>(smem + Q_OFF + sq * Q_BYTES + QW_BYTES);
          const float xs = I8 ? qsc[lr * 4 + gg] : 0.0f;
          const float xr = qsc[BM * 4 + lr * 4 + gg];
          const float* csb = reinterpret_cast<const float*>(smem + CS_OFF + sc * CS_BYTES);
          const float* cs = csb + 64 * half;
          const float* cb = csb + BN + 64 * half;
          if (I8) {
            const int b = gt % ND;
            ok = mbar_wait(bar(B_TF + b), (gt / ND) & 1, abort_flag);
            if (ok) {
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
                  if (lane == 0) mbar_arrive(bar(B_TE + b));
                }
                // column scalars read 4 at a time (16-byte aligned)
                const float4* cb4 = reinterpret_cast<const float4*>(cb + 32 * hh);
                const float4* cs4 = reinterpret_cast<const float4*>(cs + 32 * hh);
                const float2 xs2 = make_float2(xs, xs), xr2 = make_float2(xr, xr);
                float2* a2 = acc2 + 16 * hh;
                if (prescaled) {                     // d = D * s already (exact)
#pragma unroll
                  for (int c4 = 0; c4 < 8; ++c4) {
                    const float4 b4 = cb4[c4];
                    a2[2 * c4] = __ffma2_rn(make_float2(d[4 * c4], d[4 * c4 + 1]), xs2, a2[2 * c4]);
                    a2[2 * c4] = __ffma2_rn(xr2, make_float2(b4.x, b4.y), a2[2 * c4]);
                    a2[2 * c4 + 1] =
                        __ffma2_rn(make_float2(d[4 * c4 + 2], d[4 * c4 + 3]), xs2, a2[2 * c4 + 1]);
                    a2[2 * c4 + 1] = __ffma2_rn(xr2, make_float2(b4.z, b4.w), a2[2 * c4 + 1]);
                  }
                } else {
#pragma unroll
                  for (int c4 = 0; c4 < 8; ++c4) {
                    const float4 b4 = cb4[c4], s4 = cs4[c4];
                    const float2 t0 = __fmul2_rn(make_float2(d[4 * c4], d[4 * c4 + 1]),
                                                 make_float2(s4.x, s4.y));
                    const float2 t1 = __fmul2_rn(make_float2(d[4 * c4 + 2], d[4 * c4 + 3]),
                                                 make_float2(s4.z, s4.w));
                    a2[2 * c4] = __ffma2_rn(t0, xs2, a2[2 * c4]);
                    a2[2 * c4] = __ffma2_rn(xr2, make_float2(b4.x, b4.y), a2[2 * c4]);
                    a2[2 * c4 + 1] = __ffma2_rn(t1, xs2, a2[2 * c4 + 1]);
                    a2[2 * c4 + 1] = __ffma2_rn(xr2, make_float2(b4.z, b4.w), a2[2 * c4 + 1]);
                  }
                }
              }
            }
          } else {
            const float4* cb4 = reinterpret_cast<const float4*>(cb);
            const float2 xr2 = make_float2(xr, xr);
#pragma unroll
            for (int c4 = 0; c4 < 16; ++c4) {
              const float4 b4 = cb4[c4];
              acc2[2 * c4] = __ffma2_rn(xr2, make_float2(b4.x, b4.y), acc2[2 * c4]);
              acc2[2 * c4 + 1] = __ffma2_rn(xr2, make_float2(b4.z, b4.w), acc2[2 * c4 + 1]);
            }
          }
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(bar(B_CSE + sc));
            if (qend) mbar_arrive(bar(B_QE + sq));
          }
        }
        ++gb;
        if (qend) ++gq;
        if (I8) ++gt;
      }
      if (!I8) {   // STOCK: the whole K sum is in this item's TMEM buffer
        const int b = gt % ND;
        if (ok) ok = mbar_wait(bar(B_TF + b), (gt / ND) & 1, abort_flag);
        if (ok) {
          tc_fence_after();
          const uint32_t ta = tmem + lane_addr + (uint32_t)(b * BN + 64 * half);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float d[32];
            tmem_ld16(ta + 32 * hh, d);
            tmem_ld16(ta + 32 * hh + 16, d + 16);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c)
              acc2[16 * hh + c] = make_float2(__fadd_rn(d[2 * c], acc2[16 * hh + c].x),
                                              __fadd_rn(d[2 * c + 1], acc2[16 * hh + c].y));
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B_TE + b));
        }
        ++gt;
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
            pk.x = (uint32_t)f2bf(acc(8 * v + 0)) | ((uint32_t)f2bf(acc(8 * v + 1)) << 16);
            pk.y = (uint32_t)f2bf(acc(8 * v + 2)) | ((uint32_t)f2bf(acc(8 * v + 3)) << 16);
            pk.z = (uint32_t)f2bf(acc(8 * v + 4)) | ((uint32_t)f2bf(acc(8 * v + 5)) << 16);
            pk.w = (uint32_t)f2bf(acc(8 * v + 6)) | ((uint32_t)f2bf(acc(8 * v + 7)) << 16);
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
        for (int j = 0; j < 32; j += 2) {
          const float2 hv = swiglu_bf16x2(bfround2(acc2[j >> 1]), bfround2(acc2[16 + (j >> 1)]));
          h[j] = hv.x;
          h[j + 1] = hv.y;
          am = fmaxf(am, fmaxf(fabsf(hv.x), fabsf(hv.y)));
        }
#pragma unroll
        for (int l = 0; l < 16; ++l) xch[lr * 36 + 16 * half + l] = __fadd_rn(h[2 * l], h[2 * l + 1]);
        xch[lr * 36 + 32 + half] = am;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        const float amax = fmaxf(xch[lr * 36 + 32], xch[lr * 36 + 33]);
        const float sum = serial_butterfly32(xch + lr * 36, 1);
        asm volatile("bar.sync 1, 256;" ::: "memory");   // xch is rewritten by the next item
        const float scl = __fdiv_rn(fmaxf(amax, 1e-30f), 127.0f);
        const float inv = __fdiv_rn(1.0f, scl);
        if (live) {
          const size_t o = (size_t)row * P.h_srow + nb;   // row-major, padded stride
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
                val = __fadd_rn(
                    fminf(fmaxf(__fadd_rn(rintf(__fmul_rn(val, inv)), 128.0f), 0.0f), 255.0f),
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
  }

  // stores into other GPUs' memory (the expert-parallel return) are performed
  // at system scope before this kernel ends, ahead of the flag the next
  // launch posts: one fence per storing thread, after its last item
  if (EPI == kEpiStore && P.y_ptr && warp >= 8) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (*abort_flag) {
      // let any issued MMA drain before the columns are released (bounded)
      if (lane == 0) {
        mma_commit(bar(B_DRAIN));
        for (uint32_t i = 0; i < kSpinLimit && !mbar_try(bar(B_DRAIN), 0); ++i) __nanosleep(128);
      }
      __syncwarp();
    }
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ND * BN));
  }
}

template <bool I8, int EPI>
static cudaError_t launch_tc05_one(const GemmParams& P, const Tc05Maps& M, int maxt, cudaStream_t s) {
  cudaError_t err = ensure_smem_attr((const void*)gemm_tc05_kernel<I8, EPI>, SMEM);
  if (err != cudaSuccess) return err;
  // persistent: one CTA per SM walks (row tile, column block) items
  const long long items = (long long)maxt * ((EPI == kEpiStore) ? P.N / BN : (P.N / 2) / 64);
  const int sms = device_sm_count();
  const int grid = (int)(items < sms ? items : sms);
  gemm_tc05_kernel<I8, EPI><<<grid, NTHREADS, SMEM, s>>>(P, M);
  return cudaGetLastError();
}

bool gemm_tc05_supported(int K, int N) {
  return K > 0 && K % kGroup == 0 && K / kGroup <= kMaxG && N > 0 && N % BN == 0;
}

cudaError_t launch_gemm_tc05(bool int8, int epi, const GemmParams& P, int maxt, cudaStream_t s) {
  if (maxt <= 0) return cudaSuccess;
  const int G = P.K / kGroup;
  // A: expert-sorted contiguous rows; row scalars row-major with a stride of
  // whole 4-group boxes; the SwiGLU epilogues write h scalars the same way
  if (!gemm_tc05_supported(P.K, P.N) || P.E <= 0 || P.a_nrows <= 0 || P.a_rows || P.a_map ||
      P.s_g != 1 || P.s_r < G || P.s_r % 4 != 0 || (int8 && !P.asc) || !P.ars ||
      (epi != kEpiStore && (P.h_srow < P.N / 128 || P.h_srow % 4 != 0)))
    return cudaErrorInvalidValue;
  Tc05Maps M;
  const unsigned long long rows = (unsigned long long)P.a_nrows;
  const float* xs = P.asc ? P.asc : P.ars;
  if (!encode_2d(&M.a, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, P.A, (unsigned long long)P.K, rows, 64,
                 BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&M.xs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, xs, (unsigned long long)P.s_r, rows, 4,
                 BM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_2d(&M.xr, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, P.ars, (unsigned long long)P.s_r, rows,
                 4, BM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_2d(&M.w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, P.W, (unsigned long long)P.K / 8,
                 (unsigned long long)P.E * P.N, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&M.s, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, P.st, (unsigned long long)P.N,
                 (unsigned long long)P.E * G, 32, G, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_2d(&M.b, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, P.bt, (unsigned long long)P.N,
                 (unsigned long long)P.E * G, 32, G, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  if (int8) {
    if (epi == kEpiStore) return launch_tc05_one<true, kEpiStore>(P, M, maxt, s);
    if (epi == kEpiSwigluQ8) return launch_tc05_one<true, kEpiSwigluQ8>(P, M, maxt, s);
    return launch_tc05_one<true, kEpiSwigluH16>(P, M, maxt, s);
  }
  if (epi == kEpiStore) return launch_tc05_one<false, kEpiStore>(P, M, maxt, s);
  if (epi == kEpiSwigluQ8) return launch_tc05_one<false, kEpiSwigluQ8>(P, M, maxt, s);
  return launch_tc05_one<false, kEpiSwigluH16>(P, M, maxt, s);
}

// Operand prep for the tcgen05 GEMMs: one warp per output row, four 64-groups
// per step; lane l handles the 8-element chunk l % 8 of group l / 8, so every
// load and store of the warp is 512 contiguous bytes.  QUANT: the int8 codes
// xu - 128 as fp16 plus the per-group scale and exact sum; otherwise x itself
// in fp16 plus the sum.  Elements are stored in the (0,4,1,5,2,6,3,7) order of
// every 8-chunk.  Output row m reads x row m, or (gathered, expert-sorted) x
// row a_map[a_rows[m]] / a_rows[m] / a_div; its scalars sit at m * srow + g.
// The group sum is the pair sums (2j, 2j+1) reduced by the xor tree
// 16, 8, 4, 2, 1 (p[j] += p[j + off] for j < off) — the order of a butterfly
// over 32 lanes holding one pair each — evaluated across the group's 8 lanes.
template <bool QUANT>
__global__ void __launch_bounds__(256) prep_a16_kernel(const uint16_t* __restrict__ x, int R, int K,
                                                        const int32_t* __restrict__ a_rows,
                                                        const int32_t* __restrict__ a_map,
                                                        int a_div, int srow,
                                                        uint16_t* __restrict__ a16,
                                                        float* __restrict__ xsc,
                                                        float* __restrict__ xrs) {
  const int lane = threadIdx.x & 31;
  const long long m = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (m >= R) return;
  const int G = K / kGroup;
  const int src = !a_rows ? (int)m : (a_map ? a_map[a_rows[m]] : a_rows[m] / a_div);
  const int sub = lane >> 3, c = lane & 7;
  for (int g0 = 0; g0 < G; g0 += 4) {
    const int g = g0 + sub;
    const bool act = g < G;
    float v[8];
    if (act) {
      unpack8_bf16(__ldg(reinterpret_cast<const uint4*>(x + (size_t)src * K + g * kGroup + c * 8)),
                   v);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
    float p[4];
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p[i] = __fadd_rn(v[2 * i], v[2 * i + 1]);
      am = fmaxf(am, fmaxf(fabsf(v[2 * i]), fabsf(v[2 * i + 1])));
    }
    // pairs j = 4c + i: off 16, 8, 4 cross lanes (c + 4, c + 2, c + 1), off 2, 1 stay in lane 0
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __fadd_rn(p[i], __shfl_down_sync(0xffffffffu, p[i], 4, 8));
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __fadd_rn(p[i], __shfl_down_sync(0xffffffffu, p[i], 2, 8));
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __fadd_rn(p[i], __shfl_down_sync(0xffffffffu, p[i], 1, 8));
    p[0] = __fadd_rn(p[0], p[2]);
    p[1] = __fadd_rn(p[1], p[3]);
    const float sum = __fadd_rn(p[0], p[1]);          // meaningful in lane c == 0
#pragma unroll
    for (int off = 4; off >= 1; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off, 8));
    if (!act) continue;
    if (!QUANT) {
      // x itself becomes the fp16 operand: it overflows past 65504, and a
      // group lying wholly below fp16's normal range keeps too few bits
      if (c == 0 && (am >= 65504.0f || (am > 0.0f && am < 6.103515625e-05f)))
        atomicExch(&g_tc05_error, 2);
    }
    // element pairs (i, i + 4): the stored order 0,4,1,5,2,6,3,7
    float2 pr[4];
    if (QUANT) {
      const float sc = __fdiv_rn(fmaxf(am, 1e-30f), 127.0f);
      const float inv = __fdiv_rn(1.0f, sc);
      // xu - 128 = clamp(rint(v / sc) + 128, 0, 255) - 128, two lanes at a
      // time.  The products stay scalar (__fmul_rn is never fused into the
      // add after it); rint is (t + 1.5*2^23) - 1.5*2^23, exact for |t| < 2^22
      // (here |t| <= 127).
      const float2 big = make_float2(12582912.0f, 12582912.0f),
                   nbig = make_float2(-12582912.0f, -12582912.0f);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 t = make_float2(__fmul_rn(v[i], inv), __fmul_rn(v[i + 4], inv));
        const float2 q = __fadd2_rn(__fadd2_rn(__fadd2_rn(t, big), nbig), make_float2(128.0f, 128.0f));
        pr[i] = __fadd2_rn(make_float2(fminf(fmaxf(q.x, 0.0f), 255.0f), fminf(fmaxf(q.y, 0.0f), 255.0f)),
                           make_float2(-128.0f, -128.0f));
      }
      if (c == 0) xsc[(size_t)m * srow + g] = sc;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) pr[i] = make_float2(v[i], v[i + 4]);
    }
    if (c == 0) xrs[(size_t)m * srow + g] = sum;
    auto h2 = [](float2 f) {                         // .x in the low half
      const __half2 hh = __float22half2_rn(f);
      return *reinterpret_cast<const uint32_t*>(&hh);
    };
    uint4 pk;
    pk.x = h2(pr[0]);
    pk.y = h2(pr[1]);
    pk.z = h2(pr[2]);
    pk.w = h2(pr[3]);
    *reinterpret_cast<uint4*>(a16 + (size_t)m * K + g * kGroup + c * 8) = pk;
  }
}

cudaError_t launch_prep_a16_rows(const uint16_t* x, int R, int K, bool quant, const int32_t* a_rows,
                                 const int32_t* a_map, int a_div, int srow, uint16_t* a16,
                                 float* xsc, float* xrs, cudaStream_t s) {
  if (R <= 0 || K <= 0) return cudaSuccess;
  const unsigned blocks = (unsigned)(((long long)R * 32 + 255) / 256);
  if (quant)
    prep_a16_kernel<true><<<blocks, 256, 0, s>>>(x, R, K, a_rows, a_map, a_div, srow, a16, xsc, xrs);
  else
    prep_a16_kernel<false><<<blocks, 256, 0, s>>>(x, R, K, a_rows, a_map, a_div, srow, a16, xsc,
                                                  xrs);
  return cudaGetLastError();
}

cudaError_t launch_prep_a16(const uint16_t* x, int R, int K, bool quant, uint16_t* a16, float* xsc,
                            float* xrs, cudaStream_t s) {
  return launch_prep_a16_rows(x, R, K, quant, nullptr, nullptr, 1, K / kGroup, a16, xsc, xrs, s);
}

int tc05_error_flag() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc05_error, sizeof(int));
  return v;
}

}  // namespace tmoe
