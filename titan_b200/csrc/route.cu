// Routing plan: the stable sort of the flat (token, slot) expert ids
// (switch_layers.py:13-25, _gather_sort / _scatter_unsort), expert segment
// offsets and the ragged (row_start, expert) tile list of
// moe_gather_ws.py:133-202 (build_tiles), plus the list of distinct experts
// the decode kernels iterate over.  No host synchronisation: every count
// stays on the device and the consumers read it there.
//
// Small plans (R <= kSmallRows) are one CTA; large plans are three kernels:
// per-block histograms, a per-expert scan across blocks, and a stable
// scatter that ranks equal ids within a block with __match_any_sync.
//
// Also here: the per-(token, 64-group) int8 activation quantiser
// (moe_gather_int8.py:132-165).  It runs once per token; the grouped GEMM
// gathers the quantised token rows of each expert tile itself.
#include "common.cuh"
#include "tmoe_internal.h"

namespace tmoe {

// ---------------------------------------------------------------- small plan
// One CTA of 1024 threads; R <= kSmallRows, E <= 1024.
__global__ void __launch_bounds__(1024) route_plan_small(
    const int32_t* __restrict__ idx, int R, int E, int tile_m, int maxt, RoutePlan plan) {
  extern __shared__ int32_t sm[];
  int32_t* sidx = sm;               // [R]
  int32_t* cnt = sidx + R;          // [E]
  int32_t* off = cnt + E;           // [E+1]
  int32_t* tcnt = off + E + 1;      // [E+1] tile offsets
  int32_t* ucnt = tcnt + E + 1;     // [E+1] unique offsets
  const int tid = threadIdx.x;
  for (int i = tid; i < R; i += blockDim.x) sidx[i] = idx[i];
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < R; i += blockDim.x) atomicAdd(&cnt[sidx[i]], 1);
  __syncthreads();
  if (tid == 0) {
    int a = 0, b = 0, c = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = a;
      tcnt[e] = b;
      ucnt[e] = c;
      a += cnt[e];
      b += (cnt[e] + tile_m - 1) / tile_m;
      c += cnt[e] > 0 ? 1 : 0;
    }
    off[E] = a;
    tcnt[E] = b;
    ucnt[E] = c;
  }
  __syncthreads();
  for (int e = tid; e <= E; e += blockDim.x) plan.offsets[e] = off[e];
  for (int i = tid; i < R; i += blockDim.x) {
    const int e = sidx[i];
    int rank = 0;
    for (int j = 0; j < i; ++j) rank += (sidx[j] == e);
    const int pos = off[e] + rank;
    plan.order[pos] = i;
    plan.inv[i] = pos;
    if (plan.sorted_ids) plan.sorted_ids[pos] = e;
  }
  for (int e = tid; e < E; e += blockDim.x) {
    const int n = cnt[e];
    if (plan.tile_row) {
      int t0 = tcnt[e];
      for (int r = 0; r < n; r += tile_m) {
        if (t0 < maxt) {
          plan.tile_row[t0] = off[e] + r;
          plan.tile_exp[t0] = e;
        }
        ++t0;
      }
    }
    if (plan.uexp && n > 0) {
      plan.uexp[ucnt[e]] = e;
      plan.ustart[ucnt[e]] = off[e];
    }
  }
  if (tid == 0) {
    if (plan.ntiles) plan.ntiles[0] = tcnt[E] < maxt ? tcnt[E] : maxt;
    if (plan.nuniq) plan.nuniq[0] = ucnt[E];
    if (plan.ustart) plan.ustart[ucnt[E]] = R;
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
  int32_t* tcnt = off + E + 1;  // [E+1]
  int32_t* ucnt = tcnt + E + 1; // [E+1]
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int b = 0; b < nb; ++b) {
      int v = blockhist[(size_t)b * E + e];
      blockhist[(size_t)b * E + e] = run;
      run += v;
    }
    tot[e] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int a = 0, b = 0, c = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = a;
      tcnt[e] = b;
      ucnt[e] = c;
      a += tot[e];
      b += (tot[e] + tile_m - 1) / tile_m;
      c += tot[e] > 0 ? 1 : 0;
    }
    off[E] = a;
    tcnt[E] = b;
    ucnt[E] = c;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) plan.offsets[e] = off[e];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int n = tot[e];
    if (plan.tile_row) {
      int t0 = tcnt[e];
      for (int r = 0; r < n; r += tile_m) {
        if (t0 < maxt) {
          plan.tile_row[t0] = off[e] + r;
          plan.tile_exp[t0] = e;
        }
        ++t0;
      }
    }
    if (plan.uexp && n > 0) {
      plan.uexp[ucnt[e]] = e;
      plan.ustart[ucnt[e]] = off[e];
    }
  }
  if (threadIdx.x == 0) {
    if (plan.ntiles) plan.ntiles[0] = tcnt[E] < maxt ? tcnt[E] : maxt;
    if (plan.nuniq) plan.nuniq[0] = ucnt[E];
    if (plan.ustart) plan.ustart[ucnt[E]] = R;
  }
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
      int v = wc[w * E + ee];
      wc[w * E + ee] = run;
      run += v;
    }
  }
  __syncthreads();
  if (ok) {
    const int pos = plan.offsets[e] + blockoff[(size_t)blockIdx.x * E + e] + wc[warp * E + e] + rank_w;
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

cudaError_t launch_route_plan(const int32_t* idx, int R, int E, int tile_m, int maxt,
                              const RoutePlan& plan, void* scratch, cudaStream_t s) {
  if (R <= kSmallRows) {
    const size_t smem = sizeof(int32_t) * ((size_t)R + 4 * (size_t)E + 3);
    route_plan_small<<<1, 1024, smem, s>>>(idx, R, E, tile_m, maxt, plan);
    return cudaGetLastError();
  }
  const int nb = (R + kBlk - 1) / kBlk;
  int32_t* bh = static_cast<int32_t*>(scratch);
  route_hist<<<nb, kBlk, sizeof(int32_t) * E, s>>>(idx, R, E, bh);
  route_scan<<<1, 1024, sizeof(int32_t) * (4 * (size_t)E + 3), s>>>(bh, nb, R, E, tile_m, maxt,
                                                                     plan);
  const size_t smem = sizeof(int32_t) * 32 * (size_t)E;
  static bool attr_done = false;
  if (!attr_done) {
    cudaFuncSetAttribute(route_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    attr_done = true;
  }
  route_scatter<<<nb, kBlk, smem, s>>>(idx, R, E, bh, plan);
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
