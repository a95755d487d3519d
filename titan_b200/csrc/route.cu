// Routing plan: the stable sort of the flat (token, slot) expert ids
// (switch_layers.py:13-25, _gather_sort / _scatter_unsort), expert segment
// offsets and the ragged (row_start, expert) tile list of
// moe_gather_ws.py:133-202 (build_tiles), plus the list of distinct experts
// the decode kernels iterate over.  No host synchronisation: every count
// stays on the device and the consumers read it there.
//
// Small plans (R <= kSmallRows) are one CTA; large plans are three kernels:
// per-block histograms, a per-expert scan across blocks, and a stable
// scatter that ranks equal ids within a block with __match_any_sync.  The
// per-expert offsets, tile starts and distinct-expert slots come from one
// block-wide exclusive scan of a packed (count, tiles, present) word.
//
// route_decode fuses, for decode batches (T <= 32), the router's top-k, the
// plan and the activation prep into a single CTA.
//
// Also here: the per-(token, 64-group) int8 activation quantiser
// (moe_gather_int8.py:132-165).  It runs once per token; the grouped GEMM
// gathers the quantised token rows of each expert tile itself.
#include "common.cuh"
#include "tmoe_internal.h"

namespace tmoe {

namespace {

constexpr int kFieldBits = 21;                      // count | tiles | present
constexpr uint64_t kFieldMask = (1ull << kFieldBits) - 1;

// Block-wide exclusive scan of one 64-bit value per thread (blockDim <= 1024).
// ws: shared scratch of 32 words.  Returns the exclusive prefix; *total gets
// the block total.
TMOE_DEV uint64_t block_scan_excl(uint64_t v, uint64_t* ws, uint64_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  uint64_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) ws[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    uint64_t w = lane < nw ? ws[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    ws[lane] = w;
  }
  __syncthreads();
  const uint64_t excl = inc - v + (warp > 0 ? ws[warp - 1] : 0);
  *total = ws[nw - 1];
  __syncthreads();
  return excl;
}

// From per-expert counts (smem cnt[E]) build offsets (smem off[E+1] and the
// plan), the tile list and the distinct-expert list.  All threads call it.
TMOE_DEV void plan_from_counts(const int32_t* cnt, int32_t* off, int E, int R, int tile_m,
                               int maxt, const RoutePlan& plan, uint64_t* ws) {
  for (int e0 = 0; e0 < E; e0 += blockDim.x) {
    const int e = e0 + threadIdx.x;
    uint64_t v = 0;
    if (e < E) {
      const uint64_t n = (uint64_t)cnt[e];
      v = n | ((uint64_t)((n + tile_m - 1) / tile_m) << kFieldBits) |
          ((uint64_t)(n > 0) << (2 * kFieldBits));
    }
    uint64_t total;
    const uint64_t ex = block_scan_excl(v, ws, &total);
    __shared__ uint64_t carry;
    if (e0 == 0 && threadIdx.x == 0) carry = 0;
    __syncthreads();
    const uint64_t base = carry;
    const uint64_t p = base + ex;
    if (e < E) {
      const int o = (int)(p & kFieldMask);
      const int t0 = (int)((p >> kFieldBits) & kFieldMask);
      const int u = (int)(p >> (2 * kFieldBits));
      const int n = cnt[e];
      off[e] = o;
      plan.offsets[e] = o;
      if (plan.tile_row) {
        int t = t0;
        for (int r = 0; r < n; r += tile_m, ++t)
          if (t < maxt) {
            plan.tile_row[t] = o + r;
            plan.tile_exp[t] = e;
          }
      }
      if (plan.uexp && n > 0) {
        plan.uexp[u] = e;
        plan.ustart[u] = o;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) carry = base + total;
    __syncthreads();
  }
}

// Totals of the tile and distinct-expert counts and the closing entries of
// the offsets and distinct-expert lists.
TMOE_DEV void plan_totals(const int32_t* cnt, int E, int R, int tile_m, int maxt,
                          const RoutePlan& plan) {
  __shared__ int s_tiles, s_uniq;
  if (threadIdx.x == 0) {
    s_tiles = 0;
    s_uniq = 0;
  }
  __syncthreads();
  int tl = 0, un = 0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    tl += (cnt[e] + tile_m - 1) / tile_m;
    un += cnt[e] > 0;
  }
  atomicAdd(&s_tiles, tl);
  atomicAdd(&s_uniq, un);
  __syncthreads();
  if (threadIdx.x == 0) {
    plan.offsets[E] = R;
    if (plan.ntiles) plan.ntiles[0] = s_tiles < maxt ? s_tiles : maxt;
    if (plan.nuniq) plan.nuniq[0] = s_uniq;
    if (plan.ustart) plan.ustart[s_uniq] = R;
  }
}

}  // namespace

// ---------------------------------------------------------------- small plan
// One CTA of 1024 threads; R <= kSmallRows, E <= 1024.
__global__ void __launch_bounds__(1024) route_plan_small(
    const int32_t* __restrict__ idx, int R, int E, int tile_m, int maxt, RoutePlan plan) {
  extern __shared__ int32_t sm[];
  int32_t* sidx = sm;               // [R]
  int32_t* cnt = sidx + R;          // [E]
  int32_t* off = cnt + E;           // [E+1]
  __shared__ uint64_t ws[32];
  const int tid = threadIdx.x;
  for (int i = tid; i < R; i += blockDim.x) sidx[i] = idx[i];
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < R; i += blockDim.x) atomicAdd(&cnt[sidx[i]], 1);
  __syncthreads();
  plan_from_counts(cnt, off, E, R, tile_m, maxt, plan, ws);
  plan_totals(cnt, E, R, tile_m, maxt, plan);
  __syncthreads();
  for (int i = tid; i < R; i += blockDim.x) {
    const int e = sidx[i];
    int rank = 0;
    for (int j = 0; j < i; ++j) rank += (sidx[j] == e);
    const int pos = off[e] + rank;
    plan.order[pos] = i;
    plan.inv[i] = pos;
    if (plan.sorted_ids) plan.sorted_ids[pos] = e;
  }
}

// ---------------------------------------------------------------- large plan
constexpr int kBlk = 1024;

__global__ void __launch_bounds__(kBlk) route_hist(const int32_t* __restrict__ idx, int R, int E,
                                                   int32_t* __restrict__ blockhist) {
  extern __shared__ int32_t h[];
  for (int e = threadIdx.x; e < E; e += kBlk) h[e] = 0;
  __syncthreads();
  const int i = blockIdx.x * kBlk + threadIdx.x;
  if (i < R) atomicAdd(&h[idx[i]], 1);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kBlk) blockhist[(size_t)blockIdx.x * E + e] = h[e];
}

// One CTA: per-expert exclusive scan over blocks (in place), then the expert
// offsets, tile list and distinct-expert list.
__global__ void __launch_bounds__(1024) route_scan(int32_t* __restrict__ blockhist, int nb, int R,
                                                   int E, int tile_m, int maxt, RoutePlan plan) {
  extern __shared__ int32_t sm[];
  int32_t* tot = sm;            // [E]
  int32_t* off = tot + E;       // [E+1]
  __shared__ uint64_t ws[32];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int b = 0; b < nb; ++b) {
      const int v = blockhist[(size_t)b * E + e];
      blockhist[(size_t)b * E + e] = run;
      run += v;
    }
    tot[e] = run;
  }
  __syncthreads();
  plan_from_counts(tot, off, E, R, tile_m, maxt, plan, ws);
  plan_totals(tot, E, R, tile_m, maxt, plan);
}

// Stable scatter: rank = offsets[e] + (ids of e in earlier blocks) +
// (ids of e in earlier warps of this block) + (earlier lanes of this warp).
__global__ void __launch_bounds__(kBlk) route_scatter(const int32_t* __restrict__ idx, int R, int E,
                                                      const int32_t* __restrict__ blockoff,
                                                      RoutePlan plan) {
  extern __shared__ int32_t wc[];  // [32][E]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 32 * E; i += kBlk) wc[i] = 0;
  __syncthreads();
  const int i = blockIdx.x * kBlk + tid;
  const bool ok = i < R;
  const int e = ok ? idx[i] : -1 - lane;  // distinct dummies never match
  const unsigned mask = __match_any_sync(0xffffffffu, e);
  const int rank_w = __popc(mask & ((1u << lane) - 1u));
  if (ok && rank_w == 0) wc[warp * E + e] = __popc(mask);
  __syncthreads();
  for (int ee = tid; ee < E; ee += kBlk) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int v = wc[w * E + ee];
      wc[w * E + ee] = run;
      run += v;
    }
  }
  __syncthreads();
  if (ok) {
    const int pos =
        plan.offsets[e] + blockoff[(size_t)blockIdx.x * E + e] + wc[warp * E + e] + rank_w;
    plan.order[pos] = i;
    plan.inv[i] = pos;
    if (plan.sorted_ids) plan.sorted_ids[pos] = e;
  }
}

size_t route_plan_scratch_bytes(int R, int E) {
  if (R <= kSmallRows) return 0;
  const size_t nb = (size_t)(R + kBlk - 1) / kBlk;
  return nb * (size_t)E * sizeof(int32_t);
}

void route_init_attributes() {
  static bool done = false;
  if (!done) {
    cudaFuncSetAttribute(route_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    done = true;
  }
}

cudaError_t launch_route_plan(const int32_t* idx, int R, int E, int tile_m, int maxt,
                              const RoutePlan& plan, void* scratch, cudaStream_t s) {
  if (R <= kSmallRows) {
    const size_t smem = sizeof(int32_t) * ((size_t)R + 2 * (size_t)E + 1);
    route_plan_small<<<1, 1024, smem, s>>>(idx, R, E, tile_m, maxt, plan);
    return cudaGetLastError();
  }
  route_init_attributes();
  const int nb = (R + kBlk - 1) / kBlk;
  int32_t* bh = static_cast<int32_t*>(scratch);
  route_hist<<<nb, kBlk, sizeof(int32_t) * E, s>>>(idx, R, E, bh);
  route_scan<<<1, 1024, sizeof(int32_t) * (2 * (size_t)E + 1), s>>>(bh, nb, R, E, tile_m, maxt,
                                                                     plan);
  route_scatter<<<nb, kBlk, sizeof(int32_t) * 32 * (size_t)E, s>>>(idx, R, E, bh, plan);
  return cudaGetLastError();
}

// ------------------------------------------------------------ decode routing
// One CTA of 1024 threads for T <= 32 tokens: (a) warp t computes token t's
// softmax + top-k from the router logits (the canonical order of
// router_topk_kernel), (b) the routing plan over the T*k pairs, (c) the fp16
// operand copy and exact group sums of x for the decode GEMVs.
template <int PER>
__global__ void __launch_bounds__(1024) route_decode_kernel(
    const uint16_t* __restrict__ logits, int T, int E, int k, int32_t* __restrict__ idx,
    uint16_t* __restrict__ scores, const uint16_t* __restrict__ x, int H,
    uint16_t* __restrict__ x16p, float* __restrict__ xsum, RoutePlan plan,
    int32_t* __restrict__ counters, int ncounters) {
  __shared__ int32_t sidx[1024];
  __shared__ int32_t cnt[1024];
  __shared__ int32_t off[1025];
  __shared__ uint64_t ws[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int R = T * k;
  for (int i = threadIdx.x; i < ncounters; i += blockDim.x) counters[i] = 0;
  // (c) activation prep, one warp per (token, group)
  {
    const int G = H / kGroup;
    for (int task = warp; task < T * G; task += 32) {
      const int m = task / G, g = task % G;
      const uint16_t* src = x + (size_t)m * H + g * kGroup;
      const uint32_t pr = *reinterpret_cast<const uint32_t*>(src + 2 * lane);
      const float a = bf2f((uint16_t)(pr & 0xffffu)), b = bf2f((uint16_t)(pr >> 16));
      const float s = warp_butterfly_sum(__fadd_rn(a, b));
      uint16_t* dst = x16p + (size_t)m * H + g * kGroup;
      const int k0 = 2 * lane;
      const int hi = k0 & 8, r0 = k0 & 7, r1 = (k0 + 1) & 7;
      dst[(k0 & ~15) + hi + ((r0 & 3) << 1) + (r0 >> 2)] = __half_as_ushort(__float2half_rn(a));
      dst[((k0 + 1) & ~15) + ((k0 + 1) & 8) + ((r1 & 3) << 1) + (r1 >> 2)] =
          __half_as_ushort(__float2half_rn(b));
      if (lane == 0) xsum[(size_t)m * G + g] = s;
    }
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  // (a) top-k, warp t -> token t
  if (warp < T) {
    const int t = warp;
    float lv[PER];
    float m = -__int_as_float(0x7f800000);
#pragma unroll
    for (int c = 0; c < PER; ++c) {
      const int e = 32 * c + lane;
      lv[c] = (e < E) ? bf2f(logits[(size_t)t * E + e]) : -__int_as_float(0x7f800000);
      m = fmaxf(m, lv[c]);
    }
    m = warp_max(m);
    float ex[PER];
    float part = 0.0f;
#pragma unroll
    for (int c = 0; c < PER; ++c) {
      const int e = 32 * c + lane;
      if (e < E) {
        ex[c] = cexp(__fsub_rn(lv[c], m));
        part = __fadd_rn(part, ex[c]);
      } else {
        ex[c] = 0.0f;
      }
    }
    const float inv = __fdiv_rn(1.0f, warp_butterfly_sum(part));
    uint32_t pb[PER];
#pragma unroll
    for (int c = 0; c < PER; ++c) pb[c] = f2bf(__fmul_rn(ex[c], inv));
    uint32_t taken = 0, my_p = 0;
    int my_e = 0;
    float ssum = 0.0f;
    for (int j = 0; j < k; ++j) {
      uint32_t best = 0;
#pragma unroll
      for (int c = 0; c < PER; ++c) {
        const int e = 32 * c + lane;
        if (e < E && !((taken >> c) & 1u)) {
          const uint32_t key = (pb[c] << 16) | (uint32_t)(0xffff - e);
          best = key > best ? key : best;
        }
      }
      const uint32_t win = __reduce_max_sync(0xffffffffu, best);
      const int e_sel = 0xffff - (int)(win & 0xffffu);
      const uint32_t p_sel = win >> 16;
      if ((e_sel & 31) == lane) taken |= 1u << (e_sel >> 5);
      ssum = __fadd_rn(ssum, bf2f((uint16_t)p_sel));
      if (lane == j) {
        my_p = p_sel;
        my_e = e_sel;
      }
    }
    const float sb = bfround(ssum);
    if (lane < k) {
      idx[(size_t)t * k + lane] = my_e;
      sidx[t * k + lane] = my_e;
      scores[(size_t)t * k + lane] = f2bf(__fdiv_rn(bf2f((uint16_t)my_p), sb));
    }
  }
  __syncthreads();
  // (b) plan
  for (int i = threadIdx.x; i < R; i += blockDim.x) atomicAdd(&cnt[sidx[i]], 1);
  __syncthreads();
  plan_from_counts(cnt, off, E, R, 1, 0, plan, ws);
  plan_totals(cnt, E, R, 1, 0, plan);
  __syncthreads();
  for (int i = threadIdx.x; i < R; i += blockDim.x) {
    const int e = sidx[i];
    int rank = 0;
    for (int j = 0; j < i; ++j) rank += (sidx[j] == e);
    const int pos = off[e] + rank;
    plan.order[pos] = i;
    plan.inv[i] = pos;
  }
}

cudaError_t launch_route_decode(const uint16_t* logits, int T, int E, int k, int32_t* idx,
                                uint16_t* scores, const uint16_t* x, int H, uint16_t* x16p,
                                float* xsum, const RoutePlan& plan, int32_t* counters,
                                int ncounters, cudaStream_t s) {
  const int per = (E + 31) / 32;
#define TMOE_RD(P)                                                                          \
  route_decode_kernel<P><<<1, 1024, 0, s>>>(logits, T, E, k, idx, scores, x, H, x16p, xsum, \
                                            plan, counters, ncounters)
  if (per <= 4) TMOE_RD(4);
  else if (per <= 8) TMOE_RD(8);
  else if (per <= 16) TMOE_RD(16);
  else TMOE_RD(32);
#undef TMOE_RD
  return cudaGetLastError();
}

// ------------------------------------------------------- activation quantiser
// One warp per (row, group); lane l holds elements 2l, 2l+1 of the group.
// Writes signed codes xs = xu - 128, scale, and the exact-order group sum.
__global__ void __launch_bounds__(256) quantize_rows_kernel(
    const uint16_t* __restrict__ x, int R, int K, int8_t* __restrict__ xq, float* __restrict__ xsc,
    float* __restrict__ xrs) {
  const int lane = threadIdx.x & 31;
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int G = K / kGroup;
  if (w >= (long long)R * G) return;
  const int m = (int)(w / G), g = (int)(w % G);
  const uint32_t pr = *reinterpret_cast<const uint32_t*>(x + (size_t)m * K + g * kGroup + 2 * lane);
  const float a = bf2f((uint16_t)(pr & 0xffffu)), b = bf2f((uint16_t)(pr >> 16));
  const float amax = warp_max(fmaxf(fabsf(a), fabsf(b)));
  const float sum = warp_butterfly_sum(__fadd_rn(a, b));
  const float sc = __fdiv_rn(fmaxf(amax, 1e-30f), 127.0f);
  const float inv = __fdiv_rn(1.0f, sc);
  float qa = fminf(fmaxf(__fadd_rn(rintf(__fmul_rn(a, inv)), 128.0f), 0.0f), 255.0f);
  float qb = fminf(fmaxf(__fadd_rn(rintf(__fmul_rn(b, inv)), 128.0f), 0.0f), 255.0f);
  const int8_t ca = (int8_t)((int)qa - 128), cb = (int8_t)((int)qb - 128);
  const uint16_t packed = (uint16_t)((uint8_t)ca | ((uint16_t)(uint8_t)cb << 8));
  *reinterpret_cast<uint16_t*>(xq + (size_t)m * K + g * kGroup + 2 * lane) = packed;
  if (lane == 0) {
    xsc[(size_t)m * G + g] = sc;
    xrs[(size_t)m * G + g] = sum;
  }
}

cudaError_t launch_quantize_rows(const uint16_t* x, int R, int K, int8_t* xq, float* xsc,
                                 float* xrs, cudaStream_t s) {
  const long long warps = (long long)R * (K / kGroup);
  const long long blocks = (warps * 32 + 255) / 256;
  if (blocks > 0) quantize_rows_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, R, K, xq, xsc, xrs);
  return cudaGetLastError();
}

}  // namespace tmoe
