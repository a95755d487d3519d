// Persistent swap-AB grouped GEMM on tcgen05 (sm_100a): the prefill routed
// experts, the shared expert and the expert-parallel owner side.
//
// Shape.  One work item = one tile of up to 64 routed rows of one expert (the
// route plan's tiles) x two 128-row tiles of that expert's weight rows
// (store: 256 consecutive output columns; SwiGLU: 128 gate rows and the 128
// matching up rows).  The weight rows sit on the MMA's M = 128 side and the
// routed rows on N = 16..64 (rounded up to 16), so an expert with 40 routed
// rows costs 48 columns, not a 128-row M tile.  One CTA per SM walks the
// items (tile-major, weight tiles minor, so the items running at once share
// their activation tiles in L2 and read each expert's weights once).
//
// Arithmetic: the reference's int8 x int4 algebra in its re-centred fp32
// order, bit for bit.  Per 64-wide group g the MMA computes, exactly,
//   D'[n, t] = sum_k (q - 8)[n, k] * s'[n, g] * code[t, k]
// with A = (q - 8) * s' widened in shared memory (s' = s * 2^Ew(n), a power of
// two that keeps every scaled weight an fp16 normal number: exact) and B = the
// activation codes xu - 128 (exact in fp16); |D| <= 2^16 and s' has 8
// significant bits, so every partial sum is exact in fp32.  The epilogue then
// applies, group by group in the reference's order,
//   acc = fma(D', xsc[t, g], acc);  acc = fma(xrs[t, g], bv[n, g] * 2^Ew, acc)
// (bv = bf16(b + 8s)) and finally multiplies by 2^-Ew: scaling every operand
// and the accumulator by the same power of two changes no rounding, so the
// result equals acc = fma(D * s, xsc, acc); acc = fma(xrs, bv, acc) exactly.
// The stock (bf16-activation) semantics run the same pipeline with B = x *
// 2^-Et (exact), xsc -> 2^Et and bv = b + 8s in fp32.
//
// Roles (512 threads, 16 warps):
//   warp 0      TMA: packed int4 rows (SW128) and the transposed scale and
//               bias tables, 256 K per stage, two stages in flight;
//   warp 1      TMEM allocation (4 group buffers x 2 weight tiles x 64
//               columns) and the MMA issue (one elected lane);
//   warps 2-3   activation rows (codes) by cp.async, gathered through the
//               routing permutation, into SW128 stages of 64 K, and each
//               row's per-group scale and exact sum;
//   warps 4-7   one thread per weight-row pair (row r of both tiles):
//               nibbles -> scaled fp16 A stages, and each row's folded bias
//               per group for the epilogue;
//   warps 8-15  epilogue: thread = one weight row of both tiles x 32 routed
//               rows: the per-group fp32 FMAs, then the bf16 store or SwiGLU.
// Every wait is bounded; on a timeout the kernel records g_sw_error, every
// role leaves its loop, TMA and MMA work in flight is drained (bounded) and
// TMEM is released.
#include "tc05.cuh"
#include "tmoe_internal.h"

namespace tmoe {

__device__ int g_sw_error = 0;

namespace sw {

using namespace tc;

constexpr int NTHREADS = 512;
constexpr int NP = 2;                       // packed stages (256 K each)
constexpr int NA = 2;                       // converted A stages (one group each)
constexpr int NB = 6;                       // activation stages (one group each)
constexpr int NES = 8;                      // per-group row biases, converter -> epilogue
constexpr int MAX_ITEMS = 1024;             // item table in shared memory (more: from global)
constexpr int KP = 256;                     // K per packed stage
constexpr int W_BYTES = 128 * 128;          // one weight tile's packed rows of a stage
constexpr int T_BYTES = 4 * 128 * 2;        // one tile's scales (or biases) of a stage
constexpr int PK_STAGE = 2 * W_BYTES + 4 * T_BYTES;   // 36 KB
constexpr int A_STAGE = 2 * 128 * 128;      // two weight tiles x 128 rows x 128 B
constexpr int B_STAGE = kSwTileN * 128;     // 64 routed rows x 64 codes (fp16)
constexpr int CS_STAGE = 2 * kSwTileN * 4;  // per routed row: xsc (or 2^Et), xrs
constexpr int ND = 4;                       // TMEM group buffers (MMA runs ND groups ahead)
constexpr int TMEM_COLS = ND * 2 * kSwTileN;
// An activation stage is posted LAG stages after it was issued (its copies
// have landed by then).  Posting depends on the slot LAG - NB stages back
// being free, which the epilogue releases: LAG <= NB - ND keeps that no
// tighter than the MMA's own ND-group lead over the epilogue.
constexpr int PK_OFF = 0;
constexpr int A_OFF = PK_OFF + NP * PK_STAGE;
constexpr int B_OFF = A_OFF + NA * A_STAGE;
constexpr int CS_OFF = B_OFF + NB * B_STAGE;
constexpr int ES_OFF = CS_OFF + NB * CS_STAGE;        // [NES][256] fp32 row biases
constexpr int IT_OFF = ES_OFF + NES * 256 * 4;        // [MAX_ITEMS] int4 item table
constexpr int BAR_OFF = IT_OFF + MAX_ITEMS * 16;
constexpr int SMEM = BAR_OFF + 512 + 1024;            // + alignment slack
static_assert(SMEM <= 232448, "shared memory per CTA");
static_assert(PK_STAGE % 1024 == 0 && A_STAGE % 1024 == 0 && B_STAGE % 1024 == 0, "1 KB stages");
static_assert(TMEM_COLS == 512, "TMEM allocation is a power of two >= 32");
constexpr uint32_t PK_TX = PK_STAGE;        // bytes every packed stage's TMA completes

// barrier indices (uint64 each, at BAR_OFF)
constexpr int BAR_PKF = 0, BAR_PKE = BAR_PKF + NP, BAR_AF = BAR_PKE + NP, BAR_AE = BAR_AF + NA,
              BAR_BF = BAR_AE + NA, BAR_BE = BAR_BF + NB, BAR_CE = BAR_BE + NB,
              BAR_DF = BAR_CE + NB, BAR_DE = BAR_DF + ND, BAR_EF = BAR_DE + ND,
              BAR_EE = BAR_EF + NES, BAR_DRAIN = BAR_EE + NES, BAR_N = BAR_DRAIN + 1;
static_assert(BAR_N * 8 + 16 <= 512, "barrier area");

TMOE_DEV bool wait_bar(uint32_t a, uint32_t parity, volatile int* abort_flag) {
  return tc::mbar_wait(a, parity, abort_flag, &g_sw_error);
}

// A wait that ignores the abort flag (teardown: let copies in flight land).
TMOE_DEV void drain_bar(uint32_t a, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit && !mbar_try(a, parity); ++i) __nanosleep(128);
}

// Every lane of the warp waits; the warp proceeds only if all succeeded.
TMOE_DEV bool warp_wait(uint32_t a, uint32_t parity, volatile int* abort_flag) {
  return __all_sync(0xffffffffu, wait_bar(a, parity, abort_flag));
}

struct Item {
  int e, row0, ntok, mp;
};

// Item `it` of the CTA walk: tile-major, weight tiles minor.
TMOE_DEV Item item_at(const SwParams& P, int it, int nmp) {
  Item t;
  const int tile = it / nmp;
  t.mp = it - tile * nmp;
  t.e = P.tile_exp[tile];
  t.row0 = P.tile_row[tile];
  const int end = P.offsets[t.e + 1];
  t.ntok = min(kSwTileN, end - t.row0);
  return t;
}

// The CTA's k-th item: from the shared-memory table when it holds it.
TMOE_DEV Item item_k(const SwParams& P, const int4* tab, int k, int it, int nmp) {
  if (k < MAX_ITEMS) {
    const int4 v = tab[k];
    return Item{v.x, v.y, v.z, v.w};
  }
  return item_at(P, it, nmp);
}

// First weight row of weight tile m (0 or 1) of item mp.
TMOE_DEV int wrow0(int epi, int Nw, int mp, int m) {
  if (epi == kEpiStore) return mp * 256 + m * 128;
  return m * (Nw / 2) + mp * 128;
}

// The activation row that routed (sorted) row r reads.
TMOE_DEV int brow_of(const SwParams& P, int r) {
  return !P.b_rows ? r : (P.b_map ? P.b_map[P.b_rows[r]] : P.b_rows[r] / P.b_div);
}

}  // namespace sw
}  // namespace tmoe

namespace tmoe {

using namespace sw;

template <int EPI>
__global__ void __launch_bounds__(sw::NTHREADS, 1)
    gemm_sw_kernel(const __grid_constant__ SwParams P, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_b) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  auto bar = [&](int i) -> uint32_t { return smem_u32(bars + i); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + BAR_N);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + BAR_N) + 1;

  const int G = P.K / kGroup;
  const int npk = (G + 3) / 4;                 // packed stages per item
  const int nmp = P.Nw / 256;                  // weight-tile pairs per routed tile
  const int nitems = P.ntiles[0] * nmp;

  if (tid == 0) {
    for (int i = 0; i < NP; ++i) {
      mbar_init(bar(BAR_PKF + i), 1);
      mbar_init(bar(BAR_PKE + i), 4);          // the 4 converter warps
    }
    for (int i = 0; i < NA; ++i) {
      mbar_init(bar(BAR_AF + i), 4);
      mbar_init(bar(BAR_AE + i), 1);           // MMA commit
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(bar(BAR_BF + i), 2);           // the 2 activation warps (codes and scalars)
      mbar_init(bar(BAR_BE + i), 1);           // MMA commit: the codes consumed
      mbar_init(bar(BAR_CE + i), 8);           // the 8 epilogue warps: the scalars consumed
    }
    for (int i = 0; i < ND; ++i) {
      mbar_init(bar(BAR_DF + i), 1);           // MMA commit: group sums ready
      mbar_init(bar(BAR_DE + i), 8);           // the 8 epilogue warps: buffer read
    }
    for (int i = 0; i < NES; ++i) {
      mbar_init(bar(BAR_EF + i), 4);           // the 4 converter warps: row biases written
      mbar_init(bar(BAR_EE + i), 8);           // the 8 epilogue warps: read
    }
    mbar_init(bar(BAR_DRAIN), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // this CTA's items (e, first row, rows, weight pair), read once here
  int4* tab = reinterpret_cast<int4*>(smem + IT_OFF);
  for (int k = tid; k < MAX_ITEMS; k += NTHREADS) {
    const int it = blockIdx.x + k * gridDim.x;
    if (it >= nitems) break;
    const Item t = item_at(P, it, nmp);
    tab[k] = make_int4(t.e, t.row0, t.ntok, t.mp);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
        smem_u32(tmem_slot)), "n"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_s);
    tma_prefetch_desc(&tm_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      uint32_t pc = 0;
      bool ok = true;
      for (int it = blockIdx.x, kk_ = 0; ok && it < nitems; it += gridDim.x, ++kk_) {
        const Item t = item_k(P, tab, kk_, it, nmp);
        if (t.ntok <= 0) continue;
        for (int p = 0; p < npk; ++p) {
          const int s = pc % NP;
          if (!wait_bar(bar(BAR_PKE + s), ((pc / NP) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t base = smem_u32(smem + PK_OFF + s * PK_STAGE);
          const uint32_t full = bar(BAR_PKF + s);
          mbar_expect_tx(full, PK_TX);
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            const int wr = wrow0(EPI, P.Nw, t.mp, m);
            tma_load_2d(base + m * W_BYTES, &tm_w, p * (KP / 8), t.e * P.Nw + wr, full);
            tma_load_2d(base + 2 * W_BYTES + m * T_BYTES, &tm_s, wr, t.e * G + 4 * p, full);
            tma_load_2d(base + 2 * W_BYTES + (2 + m) * T_BYTES, &tm_b, wr, t.e * G + 4 * p, full);
          }
          ++pc;
        }
      }
      // every issued stage lands before the CTA may exit (consumed ones already have)
      for (uint32_t q = pc > (uint32_t)NP ? pc - NP : 0; q < pc; ++q)
        drain_bar(bar(BAR_PKF + q % NP), (q / NP) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    // group g of an item: D[g % 2][m] = A(tile m) x B over the group's 64 K
    if (lane == 0) {
      uint32_t ac = 0, bc = 0;
      bool ok = true;
      for (int it = blockIdx.x, kk_ = 0; ok && it < nitems; it += gridDim.x, ++kk_) {
        const Item t = item_k(P, tab, kk_, it, nmp);
        if (t.ntok <= 0) continue;
        const uint32_t idesc = idesc_f16(128, (t.ntok + 15) & ~15);
        for (int j = 0; j < G; ++j) {
          const int sa = ac % NA, sb = bc % NB, d = bc % ND;
          if (!wait_bar(bar(BAR_DE + d), ((bc / ND) & 1) ^ 1, abort_flag) ||
              !wait_bar(bar(BAR_AF + sa), (ac / NA) & 1, abort_flag) ||
              !wait_bar(bar(BAR_BF + sb), (bc / NB) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t abase = smem_u32(smem + A_OFF + sa * A_STAGE);
          const uint32_t bbase = smem_u32(smem + B_OFF + sb * B_STAGE);
          const uint32_t d0 = tmem + (uint32_t)(d * 2 * kSwTileN);
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f16(d0 + m * kSwTileN, sw128_desc(abase + m * 16384 + kk * 32),
                      sw128_desc(bbase + kk * 32), idesc, kk > 0 ? 1u : 0u);
          mma_commit(bar(BAR_AE + sa));
          mma_commit(bar(BAR_BE + sb));
          mma_commit(bar(BAR_DF + d));
          ++ac;
          ++bc;
        }
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------ activation rows
    // Stage j of an item: codes [64j, 64j + 64) of the tile's rows, and each
    // row's scale and exact sum of group j.  A stage's full barrier is posted
    // LAG stages later, once this thread's copies of it have landed.
    constexpr int LAG = NB - ND;
    static_assert(LAG >= 1, "activation ring too shallow");
    const int pt = tid - 64;                   // routed row pt of a tile
    uint32_t bc = 0;
    bool ok = true;
    auto post = [&](uint32_t q) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_BF + q % NB));
    };
    for (int it = blockIdx.x, kk_ = 0; ok && it < nitems; it += gridDim.x, ++kk_) {
      const Item t = item_k(P, tab, kk_, it, nmp);
      if (t.ntok <= 0) continue;
      const uint16_t* src = nullptr;
      const float *s1 = nullptr, *s2 = nullptr;
      if (pt < t.ntok) {
        const size_t br = (size_t)brow_of(P, t.row0 + pt);
        src = P.B + br * P.K;
        s1 = P.c1 + br * G;
        s2 = P.c2 + br * G;
      }
      for (int j = 0; j < G; ++j) {
        const int sb = bc % NB;
        const uint32_t par = ((bc / NB) & 1) ^ 1;
        if (!warp_wait(bar(BAR_BE + sb), par, abort_flag) ||
            !warp_wait(bar(BAR_CE + sb), par, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* dst = smem + B_OFF + sb * B_STAGE + pt * 128;
        float* cs = reinterpret_cast<float*>(smem + CS_OFF + sb * CS_STAGE);
        if (src) {
#pragma unroll
          for (int c = 0; c < 8; ++c)
            cp_async16(dst + ((c ^ (pt & 7)) << 4), src + j * 64 + c * 8);
          cp_async4(cs + pt, s1 + j);
          cp_async4(cs + kSwTileN + pt, s2 + j);
        } else {
          cs[pt] = 0.0f;
          cs[kSwTileN + pt] = 0.0f;
        }
        cp_async_commit();
        if (bc >= (uint32_t)LAG) {
          cp_async_wait<LAG>();
          post(bc - LAG);
        }
        ++bc;
      }
    }
    cp_async_wait<0>();
    if (ok)
      for (uint32_t q = bc > (uint32_t)LAG ? bc - LAG : 0; q < bc; ++q) post(q);
  }
  else if (warp < 8) {
    // ------------------------------------------------ weight rows -> A stages
    // Thread lr converts row lr of both weight tiles, group by group:
    // (q - 8) * s * 2^Ew in fp16 (exact), in the operand layout of B; and
    // hands the epilogue each row's folded bias bv * 2^Ew per group.
    const int lr = tid - 128;
    uint32_t pc = 0, ac = 0;
    bool ok = true;
    float mult[2] = {0.0f, 0.0f};
    if (blockIdx.x < nitems) {                 // the first item's row normalisers
      const Item t = item_k(P, tab, 0, blockIdx.x, nmp);
#pragma unroll
      for (int m = 0; m < 2; ++m)
        mult[m] = P.rscale[(size_t)t.e * P.Nw + wrow0(EPI, P.Nw, t.mp, m) + lr];
    }
    for (int it = blockIdx.x, kk_ = 0; ok && it < nitems; it += gridDim.x, ++kk_) {
      const Item t = item_k(P, tab, kk_, it, nmp);
      float nmult[2] = {0.0f, 0.0f};             // the next item's, loaded ahead
      if (it + (int)gridDim.x < nitems) {
        const Item tn = item_k(P, tab, kk_ + 1, it + gridDim.x, nmp);
#pragma unroll
        for (int m = 0; m < 2; ++m)
          nmult[m] = P.rscale[(size_t)tn.e * P.Nw + wrow0(EPI, P.Nw, tn.mp, m) + lr];
      }
      if (t.ntok > 0) {
        for (int p = 0; p < npk; ++p) {
          const int s = pc % NP;
          if (!warp_wait(bar(BAR_PKF + s), (pc / NP) & 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint8_t* stg = smem + PK_OFF + s * PK_STAGE;
          __half s16[2][4];
          float bvs[2][4];
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            const uint16_t* stab = reinterpret_cast<const uint16_t*>(stg + 2 * W_BYTES + m * T_BYTES);
            const uint16_t* btab =
                reinterpret_cast<const uint16_t*>(stg + 2 * W_BYTES + (2 + m) * T_BYTES);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float sv = bf2f(stab[j * 128 + lr]);
              float bv = __fadd_rn(bf2f(btab[j * 128 + lr]), __fmul_rn(8.0f, sv));
              if (P.bias_bf16) bv = bfround(bv);
              s16[m][j] = __float2half_rn(__fmul_rn(sv, mult[m]));
              bvs[m][j] = __fmul_rn(bv, mult[m]);
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (4 * p + j >= G) break;
            const int sa = ac % NA, se = ac % NES;
            if (!warp_wait(bar(BAR_AE + sa), ((ac / NA) & 1) ^ 1, abort_flag) ||
                !warp_wait(bar(BAR_EE + se), ((ac / NES) & 1) ^ 1, abort_flag)) {
              ok = false;
              break;
            }
            float* es = reinterpret_cast<float*>(smem + ES_OFF + se * 1024);
            es[lr] = bvs[0][j];
            es[128 + lr] = bvs[1][j];
#pragma unroll
            for (int m = 0; m < 2; ++m) {
              const uint8_t* prow = stg + m * W_BYTES + lr * 128;
              const uint4 w0 = *reinterpret_cast<const uint4*>(prow + (((2 * j) ^ (lr & 7)) << 4));
              const uint4 w1 =
                  *reinterpret_cast<const uint4*>(prow + (((2 * j + 1) ^ (lr & 7)) << 4));
              const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
              const __half2 s2 = __halves2half2(s16[m][j], s16[m][j]);
              uint8_t* arow = smem + A_OFF + sa * A_STAGE + m * 16384 + lr * 128;
#pragma unroll
              for (int i = 0; i < 8; ++i)
                *reinterpret_cast<uint4*>(arow + ((i ^ (lr & 7)) << 4)) = widen8(ws[i], true, s2);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
              mbar_arrive(bar(BAR_AF + sa));
              mbar_arrive(bar(BAR_EF + se));
            }
            ++ac;
          }
          if (!ok) break;
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(BAR_PKE + s));
          ++pc;
        }
      }
      mult[0] = nmult[0];
      mult[1] = nmult[1];
    }
  } else {
    // ------------------------------------------------------------- epilogue
    // Warp (q, h): TMEM lanes 32q..32q+31 (weight row lr of both tiles) x
    // routed rows [32h, 32h + 32) of the item; per group the reference's two
    // fp32 FMAs per element, in group order.
    const int q = warp & 3, h = (warp - 8) >> 2;
    const int lr = q * 32 + lane;
    const int Ih = P.Nw / 2;
    uint32_t bc = 0;
    bool ok = true;
    for (int it = blockIdx.x, kk_ = 0; ok && it < nitems; it += gridDim.x, ++kk_) {
      const Item t = item_k(P, tab, kk_, it, nmp);
      if (t.ntok <= 0) continue;
      const bool active = 32 * h < t.ntok;          // warp-uniform
      // lane i's output row pointer for routed row 32h + i, and this thread's
      // row normalisers: loaded now, used after the last group
      uint16_t* myrow = nullptr;
      {
        const int col = 32 * h + lane;
        if (col < t.ntok) {
          const int rr = t.row0 + col;
          if (EPI == kEpiStore) {
            const int orow = P.y_rows ? P.y_rows[rr] : rr;
            myrow = P.y_ptr ? P.y_ptr[orow] : P.Y + (size_t)orow * P.Nw;
          } else {
            myrow = P.H + (size_t)rr * Ih;
          }
        }
      }
      const int wr0 = wrow0(EPI, P.Nw, t.mp, 0) + lr, wr1 = wrow0(EPI, P.Nw, t.mp, 1) + lr;
      const float rs0 = P.rscale[(size_t)t.e * P.Nw + wr0];
      const float rs1 = P.rscale[(size_t)t.e * P.Nw + wr1];
      // accumulators as token-column pairs: the per-group rescale issues as
      // packed f32x2 FMAs (each component rounds exactly as a scalar fma.rn)
      float2 acc0[16], acc1[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc0[i] = acc1[i] = make_float2(0.0f, 0.0f);
      for (int g = 0; g < G; ++g) {
        const int d = bc % ND, sb = bc % NB, se = bc % NES;
        if (!warp_wait(bar(BAR_DF + d), (bc / ND) & 1, abort_flag) ||
            !warp_wait(bar(BAR_BF + sb), (bc / NB) & 1, abort_flag) ||
            !warp_wait(bar(BAR_EF + se), (bc / NES) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (active) {
          const float* es = reinterpret_cast<const float*>(smem + ES_OFF + se * 1024);
          const float bv0 = es[lr], bv1 = es[128 + lr];
          const float* c1 = reinterpret_cast<const float*>(smem + CS_OFF + sb * CS_STAGE) + 32 * h;
          const float* c2 = c1 + kSwTileN;
          const uint32_t ta =
              tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(d * 2 * kSwTileN + 32 * h);
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            float2* acc = m ? acc1 : acc0;
            const float bv = m ? bv1 : bv0;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {          // 16 columns at a time: fewer registers
              float v[16];
              tmem_ld16(ta + m * kSwTileN + 16 * hh, v);
              tmem_wait_ld();
#pragma unroll
              for (int c4 = 0; c4 < 4; ++c4) {
                const float4 a1 = *reinterpret_cast<const float4*>(c1 + 16 * hh + 4 * c4);
                const float4 a2 = *reinterpret_cast<const float4*>(c2 + 16 * hh + 4 * c4);
                const float2 bv2 = make_float2(bv, bv);
                const int c = (16 * hh + 4 * c4) >> 1;
                acc[c] = __ffma2_rn(make_float2(v[4 * c4], v[4 * c4 + 1]), make_float2(a1.x, a1.y),
                                    acc[c]);
                acc[c] = __ffma2_rn(make_float2(a2.x, a2.y), bv2, acc[c]);
                acc[c + 1] = __ffma2_rn(make_float2(v[4 * c4 + 2], v[4 * c4 + 3]),
                                        make_float2(a1.z, a1.w), acc[c + 1]);
                acc[c + 1] = __ffma2_rn(make_float2(a2.z, a2.w), bv2, acc[c + 1]);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar(BAR_DE + d));
          mbar_arrive(bar(BAR_CE + sb));
          mbar_arrive(bar(BAR_EE + se));
        }
        ++bc;
      }
      if (!ok) break;
      if (active) {
        const float inv0 = __fdiv_rn(1.0f, rs0), inv1 = __fdiv_rn(1.0f, rs1);
        const int n = min(32, t.ntok - 32 * h);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          uint16_t* dst0 = reinterpret_cast<uint16_t*>(
              __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(myrow), i));
          uint16_t* dst1 = reinterpret_cast<uint16_t*>(
              __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(myrow), i + 1));
          const float2 a = acc0[i >> 1], b = acc1[i >> 1];
          if (EPI == kEpiStore) {
            if (i < n) {
              dst0[wr0] = f2bf(__fmul_rn(a.x, inv0));
              dst0[wr1] = f2bf(__fmul_rn(b.x, inv1));
            }
            if (i + 1 < n) {
              dst1[wr0] = f2bf(__fmul_rn(a.y, inv0));
              dst1[wr1] = f2bf(__fmul_rn(b.y, inv1));
            }
          } else if (i < n) {
            const float2 gt = bfround2(__fmul2_rn(a, make_float2(inv0, inv0)));
            const float2 ut = bfround2(__fmul2_rn(b, make_float2(inv1, inv1)));
            const float2 hv = swiglu_bf16x2(gt, ut);
            dst0[t.mp * 128 + lr] = f2bf(hv.x);
            if (i + 1 < n) dst1[t.mp * 128 + lr] = f2bf(hv.y);
          }
        }
      }
    }
  }

  // stores into other GPUs' memory (the expert-parallel return) are performed
  // at system scope before the kernel ends: one fence per storing thread,
  // after its last item
  if (EPI == kEpiStore && P.y_ptr && warp >= 8) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (*abort_flag) {
      // let issued MMAs finish before their columns are released (bounded)
      if (lane == 0) {
        mma_commit(bar(BAR_DRAIN));
        drain_bar(bar(BAR_DRAIN), 0);
      }
      __syncwarp();
    }
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(TMEM_COLS));
  }
}

}  // namespace tmoe

// ------------------------------------------------------------ operand prep

namespace tmoe {

// One warp per row; lane l holds elements 2l, 2l+1 of every 64-group, stored
// at their (0,4,1,5,2,6,3,7)-order positions (the order the widened weights
// use).  The group sum is the pair sums then the butterfly (the quantiser's
// canonical order); QUANT's scale and codes are those of the reference's
// quantiser.
template <bool QUANT>
__global__ void __launch_bounds__(256) prep_rows_kernel(const uint16_t* __restrict__ x, int R, int K,
                                                        uint16_t* __restrict__ out,
                                                        float* __restrict__ c1,
                                                        float* __restrict__ c2,
                                                        const int32_t* __restrict__ rows_limit) {
  const int lane = threadIdx.x & 31;
  const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= R || (rows_limit && row >= *rows_limit)) return;
  const int G = K / kGroup;
  const uint16_t* xr = x + (size_t)row * K;
  uint16_t* o = out + (size_t)row * K;
  float inv = 1.0f, scl = 1.0f;
  if (!QUANT) {                                     // one power of two for the row
    float am = 0.0f;
    for (int g = 0; g < G; ++g) {
      const uint32_t pr = *reinterpret_cast<const uint32_t*>(xr + g * kGroup + 2 * lane);
      am = fmaxf(am, fmaxf(fabsf(bf2f((uint16_t)(pr & 0xffffu))), fabsf(bf2f((uint16_t)(pr >> 16)))));
    }
    am = warp_max(am);
    int ex = 0;
    if (am > 0.0f && am <= 3.0e38f) frexpf(am, &ex);          // am in [2^(ex-1), 2^ex)
    const int et = am > 0.0f ? max(-126, min(126, ex - 9)) : 0;  // am * 2^-et in [2^8, 2^9)
    inv = ldexpf(1.0f, -et);
    scl = ldexpf(1.0f, et);
  }
  for (int g = 0; g < G; ++g) {
    const uint32_t pr = *reinterpret_cast<const uint32_t*>(xr + g * kGroup + 2 * lane);
    float a = bf2f((uint16_t)(pr & 0xffffu)), b = bf2f((uint16_t)(pr >> 16));
    const float sum = warp_butterfly_sum(__fadd_rn(a, b));
    if (QUANT) {
      const float amax = warp_max(fmaxf(fabsf(a), fabsf(b)));
      scl = __fdiv_rn(fmaxf(amax, 1e-30f), 127.0f);
      const float isc = __fdiv_rn(1.0f, scl);
      a = __fadd_rn(fminf(fmaxf(__fadd_rn(rintf(__fmul_rn(a, isc)), 128.0f), 0.0f), 255.0f), -128.0f);
      b = __fadd_rn(fminf(fmaxf(__fadd_rn(rintf(__fmul_rn(b, isc)), 128.0f), 0.0f), 255.0f), -128.0f);
    } else {
      a = __fmul_rn(a, inv);
      b = __fmul_rn(b, inv);
    }
    const int k0 = g * kGroup + 2 * lane;
    o[tc::p8(k0)] = __half_as_ushort(__float2half_rn(a));
    o[tc::p8(k0 + 1)] = __half_as_ushort(__float2half_rn(b));
    if (lane == 0) {
      c1[(size_t)row * G + g] = scl;
      c2[(size_t)row * G + g] = sum;
    }
  }
}

// One thread per weight row: the power of two that brings the row's largest
// scaled nibble 8|s| into [2^13, 2^14), so (q - 8) * s * 2^Ew is an exact fp16
// for every group whose scale lies within 2^24 of the row's largest.
__global__ void row_scale_kernel(const uint16_t* __restrict__ scales, long long rows, int G,
                                 float* __restrict__ rscale) {
  const long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float m = 0.0f;
  for (int g = 0; g < G; ++g) m = fmaxf(m, fabsf(__fmul_rn(8.0f, bf2f(scales[r * G + g]))));
  int ex = 0;
  if (m > 0.0f && m <= 3.0e38f) frexpf(m, &ex);              // m in [2^(ex-1), 2^ex)
  const int ew = m > 0.0f ? max(-126, min(126, 14 - ex)) : 0;  // m * 2^ew in [2^13, 2^14)
  rscale[r] = ldexpf(1.0f, ew);
}

cudaError_t launch_prep_rows(const uint16_t* x, int R, int K, bool quant, uint16_t* out,
                             float* c1, float* c2, const int32_t* rows_limit, cudaStream_t s) {
  if (R <= 0) return cudaSuccess;
  const unsigned blocks = (unsigned)(((long long)R * 32 + 255) / 256);
  if (quant)
    prep_rows_kernel<true><<<blocks, 256, 0, s>>>(x, R, K, out, c1, c2, rows_limit);
  else
    prep_rows_kernel<false><<<blocks, 256, 0, s>>>(x, R, K, out, c1, c2, rows_limit);
  return cudaGetLastError();
}

cudaError_t launch_row_scale(const uint16_t* scales, const uint16_t* biases, long long rows, int K,
                             float* rscale, cudaStream_t s) {
  (void)biases;
  if (rows <= 0) return cudaSuccess;
  row_scale_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(scales, rows, K / kGroup, rscale);
  return cudaGetLastError();
}

// ------------------------------------------------------------ launch

bool gemm_sw_supported(int epi, int K, int Nw) {
  (void)epi;
  return K > 0 && K % kGroup == 0 && Nw > 0 && Nw % 256 == 0;
}

cudaError_t launch_gemm_sw(int epi, const SwParams& P, cudaStream_t s) {
  if (P.maxt <= 0) return cudaSuccess;
  if (!gemm_sw_supported(epi, P.K, P.Nw)) return cudaErrorInvalidValue;
  const int G = P.K / kGroup;
  CUtensorMap mw, ms, mb;
  if (!encode_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, P.W, (unsigned long long)P.K / 8,
                 (unsigned long long)P.E * P.Nw, sw::KP / 8, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&ms, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, P.st, (unsigned long long)P.Nw,
                 (unsigned long long)P.E * G, 128, 4, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, P.bt, (unsigned long long)P.Nw,
                 (unsigned long long)P.E * G, 128, 4, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  const long long items = (long long)P.maxt * (P.Nw / 256);
  const int sms = device_sm_count();
  const int grid = (int)(items < sms ? items : sms);
  const void* k = epi == kEpiStore ? (const void*)gemm_sw_kernel<kEpiStore>
                                   : (const void*)gemm_sw_kernel<kEpiSwigluH16>;
  cudaError_t err = ensure_smem_attr(k, sw::SMEM);
  if (err != cudaSuccess) return err;
  if (epi == kEpiStore)
    gemm_sw_kernel<kEpiStore><<<grid, sw::NTHREADS, sw::SMEM, s>>>(P, mw, ms, mb);
  else
    gemm_sw_kernel<kEpiSwigluH16><<<grid, sw::NTHREADS, sw::SMEM, s>>>(P, mw, ms, mb);
  return cudaGetLastError();
}

int sw_error_flag() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_sw_error, sizeof(int));
  return v;
}

}  // namespace tmoe
