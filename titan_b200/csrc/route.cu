// Routing plan: the stable sort of the flat (token, slot) expert ids
// (switch_layers.py:13-25, _gather_sort / _scatter_unsort), expert segment
// offsets and the ragged (row_start, expert) tile list of
// moe_gather_ws.py:133-202 (build_tiles), plus the list of distinct experts
// the decode kernels iterate over.  No host synchronisation: every count
// stays on the device and the consumers read it there.
//
// Negative ids are skipped: they get no sorted row (inv = -1) and the sorted
// rows end at offsets[E] = the number of non-negative ids.
//
// Small plans (R <= kSmallRows) are one CTA; large plans are three kernels:
// per-block histograms, a per-expert scan across blocks, and a stable
// scatter that ranks equal ids within a block with __match_any_sync.  The
// per-expert offsets, tile starts and distinct-expert slots come from one
// block-wide exclusive scan of a packed (count, tiles, present) word.
//
// decode_route fuses, for small decode batches, the router logits, the
// top-k and the plan into one launch (the last CTA to finish routes).
//
// Also here: the per-(token, 64-group) int8 activation quantiser
// (moe_gather_int8.py:132-165).  It runs once per token; the grouped GEMM
// gathers the quantised token rows of each expert tile itself.
#include "common.cuh"
#include "fragments.cuh"
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
// The sorted rows end at the number of placed ids (R unless some are
// negative).
TMOE_DEV void plan_totals(const int32_t* cnt, int E, int tile_m, int maxt,
                          const RoutePlan& plan) {
  __shared__ int s_tiles, s_uniq, s_rows;
  if (threadIdx.x == 0) {
    s_tiles = 0;
    s_uniq = 0;
    s_rows = 0;
  }
  __syncthreads();
  int tl = 0, un = 0, nr = 0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    tl += (cnt[e] + tile_m - 1) / tile_m;
    un += cnt[e] > 0;
    nr += cnt[e];
  }
  atomicAdd(&s_tiles, tl);
  atomicAdd(&s_uniq, un);
  atomicAdd(&s_rows, nr);
  __syncthreads();
  if (threadIdx.x == 0) {
    plan.offsets[E] = s_rows;
    if (plan.ntiles) plan.ntiles[0] = s_tiles < maxt ? s_tiles : maxt;
    if (plan.nuniq) plan.nuniq[0] = s_uniq;
    if (plan.ustart) plan.ustart[s_uniq] = s_rows;
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
  for (int i = tid; i < R; i += blockDim.x)
    if (sidx[i] >= 0) atomicAdd(&cnt[sidx[i]], 1);
  __syncthreads();
  plan_from_counts(cnt, off, E, R, tile_m, maxt, plan, ws);
  plan_totals(cnt, E, tile_m, maxt, plan);
  __syncthreads();
  for (int i = tid; i < R; i += blockDim.x) {
    const int e = sidx[i];
    if (e < 0) {
      plan.inv[i] = -1;
      continue;
    }
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
  if (i < R && idx[i] >= 0) atomicAdd(&h[idx[i]], 1);
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
  plan_totals(tot, E, tile_m, maxt, plan);
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
  const int id = i < R ? idx[i] : -1;
  const bool ok = id >= 0;                // negative ids are not placed
  if (i < R && !ok) plan.inv[i] = -1;
  const int e = ok ? id : -1 - lane;      // distinct dummies never match
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


cudaError_t launch_route_plan(const int32_t* idx, int R, int E, int tile_m, int maxt,
                              const RoutePlan& plan, void* scratch, cudaStream_t s) {
  if (R <= kSmallRows) {
    const size_t smem = sizeof(int32_t) * ((size_t)R + 2 * (size_t)E + 1);
    route_plan_small<<<1, 1024, smem, s>>>(idx, R, E, tile_m, maxt, plan);
    return cudaGetLastError();
  }
  const size_t scatter_smem = sizeof(int32_t) * 32 * (size_t)E;
  cudaError_t err = ensure_smem_attr((const void*)route_scatter, (int)scatter_smem);
  if (err != cudaSuccess) return err;
  const int nb = (R + kBlk - 1) / kBlk;
  int32_t* bh = static_cast<int32_t*>(scratch);
  route_hist<<<nb, kBlk, sizeof(int32_t) * E, s>>>(idx, R, E, bh);
  route_scan<<<1, 1024, sizeof(int32_t) * (2 * (size_t)E + 1), s>>>(bh, nb, R, E, tile_m, maxt,
                                                                     plan);
  route_scatter<<<nb, kBlk, scatter_smem, s>>>(idx, R, E, bh, plan);
  return cudaGetLastError();
}

// ------------------------------------------------------------ decode routing
// Decode router (T <= kDecodeRouteMaxT tokens) in one launch.  Each CTA of 4
// warps computes the logits of 8 rows (experts, plus the shared-expert gate as
// row E) for every token: 8 lanes per row, one per canonical partial, warps 0
// and 1 over tokens 0-3 and warps 2 and 3 over tokens 4-7 of each pass of 8,
// with the rows and the token vectors staged in shared
// memory by cp.async.  The last CTA to finish (a device-wide ticket; nobody
// waits) then routes the tokens, one warp per token (route_token: the same
// selection and tie order as router_topk_kernel), builds the routing plan over
// the T*k pairs, zeroes the decode combine counters and resets the ticket.
//
// counters[0] is the ticket; counters[1 .. ncounters] are the combine
// counters.  counters[0] must be zero when the kernel starts; it is zero again
// when the kernel ends.  The rows are requested before the wait for the
// previous kernel (they are constant); the next kernel is released only after
// that wait, so it may read this layer's input without waiting for us.
constexpr int kDrRows = 8;         // rows per CTA (4 per warp, warps 0-1)
constexpr int kDrTok = 8;          // tokens per pass

template <int PER>
__global__ void __launch_bounds__(128) decode_route_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr,
    const uint16_t* __restrict__ wg, int T, int H, int E, int k, uint16_t* __restrict__ logits,
    float* __restrict__ gate_logit, int32_t* __restrict__ idx, uint16_t* __restrict__ scores,
    RoutePlan plan, int32_t* __restrict__ counters, int ncounters) {
  extern __shared__ __align__(16) uint8_t smem_dr[];
  __shared__ int32_t sidx[1024];
  __shared__ int32_t cnt[1024];
  __shared__ int32_t off[1025];
  __shared__ uint64_t ws[32];
  __shared__ __align__(16) uint16_t lg_s[4][1024];    // one token's logits per warp
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nch = H >> 3;                              // 16-byte chunks per row
  const int nrows = E + (wg ? 1 : 0);
  const int r0 = blockIdx.x * kDrRows;
  uint4* wsm = reinterpret_cast<uint4*>(smem_dr);      // [8][nch]
  uint4* xsm = wsm + kDrRows * nch;                    // [8][nch]

  // ---- logits of rows r0 .. r0+7: constant rows requested before the wait
  for (int r = 2 * warp; r < 2 * warp + 2; ++r) {
    const int er = r0 + r;
    const bool ok = er < nrows;
    const uint16_t* row = ok ? ((er < E) ? wr + (size_t)er * H : wg) : wr;
    for (int c = lane; c < nch; c += 32) cp_async16_zfill(&wsm[r * nch + c], row + (size_t)c * 8, ok);
  }
  pdl_wait();                                          // x and the workspace are ours now
  pdl_trigger();
  const int p = lane & 7, sub = lane >> 3;
  // warps 0-1 take tokens 0..3 of a pass and warps 2-3 tokens 4..7 of the
  // same 8 rows, so no lane carries more than 4 tokens
  const int rl = (warp & 1) * 4 + sub, e = r0 + rl, half = warp >> 1;
  const uint4* wrow_s = wsm + rl * nch;
  for (int t0 = 0; t0 < T; t0 += kDrTok) {
    const int nt = min(kDrTok, T - t0);
    __syncthreads();                                   // previous pass done with xsm
    for (int tt = 0; tt < nt; ++tt)
      for (int c = tid; c < nch; c += 128)
        cp_async16(&xsm[tt * nch + c], x + (size_t)(t0 + tt) * H + (size_t)c * 8);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    const int nth = half == 0 ? min(nt, 4) : nt - 4;
    if (nth > 0) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const uint4* xs_h = xsm + half * 4 * nch;
      // token count rounded up to 1, 2 or 4: straight-line inner loops (the
      // extra accumulators read stale rows and are dropped)
      if (nth == 1)
        router_dots<1>(wrow_s, xs_h, nch, p, acc);
      else if (nth == 2)
        router_dots<2>(wrow_s, xs_h, nch, p, acc);
      else
        router_dots<4>(wrow_s, xs_h, nch, p, acc);
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        const float s8 = tree8(acc[tt]);
        if (e < nrows && p == tt && tt < nth) {
          const int tok = t0 + half * 4 + tt;
          if (e < E)
            logits[(size_t)tok * E + e] = f2bf(s8);
          else
            gate_logit[tok] = s8;
        }
      }
    }
  }

  // ---- the last CTA to finish routes every token
  __syncthreads();
  if (tid == 0) s_last = (ticket_acq_rel(&counters[0]) == (int)gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  const int R = T * k;
  for (int i = tid; i < ncounters; i += 128) counters[1 + i] = 0;
  if (R > 32)
    for (int i = tid; i < E; i += 128) cnt[i] = 0;
  // every warp routes its tokens (t = warp, warp + 4, ...) from a copy of the
  // token's logits in shared memory
  for (int t = warp; t < T; t += 4) {
    const uint16_t* lrow = logits + (size_t)t * E;
    uint16_t* lw = lg_s[warp];
    if ((E & 7) == 0) {
      for (int i = lane; i < E / 8; i += 32)
        reinterpret_cast<uint4*>(lw)[i] = __ldcg(reinterpret_cast<const uint4*>(lrow) + i);
    } else {
      for (int i = lane; i < E; i += 32) lw[i] = __ldcg(lrow + i);
    }
    __syncwarp();
    const RouteOut ro = route_token<PER>(lw, E, k, lane);
    if (lane < k) {
      idx[(size_t)t * k + lane] = ro.e;
      sidx[t * k + lane] = ro.e;
      scores[(size_t)t * k + lane] = ro.score;
    }
    __syncwarp();
  }
  __syncthreads();
  if (R <= 32) {
    // One warp: bitonic sort of (expert, pair) keys; the pair index makes the
    // order stable.  Sorted position j holds pair order[j]; the first position
    // of each expert starts a distinct-expert segment.
    if (warp == 0) {
      int key = lane < R ? (sidx[lane] << 6) | lane : 0x7fffffff;
#pragma unroll
      for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
        for (int j = kk >> 1; j > 0; j >>= 1) {
          const int other = __shfl_xor_sync(0xffffffffu, key, j);
          const bool up = (lane & kk) == 0, lower = (lane & j) == 0;
          key = (lower == up) ? min(key, other) : max(key, other);
        }
      }
      const int ee = key >> 6, flat = key & 63;
      const int prev = __shfl_up_sync(0xffffffffu, ee, 1);
      const bool first = lane < R && (lane == 0 || prev != ee);
      const uint32_t mask = __ballot_sync(0xffffffffu, first);
      if (lane < R) {
        plan.order[lane] = flat;
        plan.inv[flat] = lane;
      }
      if (first) {
        const int u = __popc(mask & ((1u << lane) - 1u));
        plan.uexp[u] = ee;
        plan.ustart[u] = lane;
      }
      if (lane == 0) {
        plan.nuniq[0] = __popc(mask);
        plan.ustart[__popc(mask)] = R;
      }
    }
  } else if (R <= 128) {
    // one thread per pair: its sorted position is the number of pairs with a
    // smaller (expert, pair) key; the first pair of an expert opens a segment
    int e = 0, pos = 0, first = 0;
    if (tid < R) {
      e = sidx[tid];
      first = 1;
      for (int j = 0; j < R; ++j) {
        const int ej = sidx[j];
        pos += (ej < e) || (ej == e && j < tid);
        if (ej == e && j < tid) first = 0;
      }
      plan.order[pos] = tid;
      plan.inv[tid] = pos;
      cnt[tid] = first;
    }
    __syncthreads();
    if (tid < R && first) {
      int u = 0;
      for (int j = 0; j < R; ++j) u += (cnt[j] && sidx[j] < e);
      plan.uexp[u] = e;
      plan.ustart[u] = pos;
    }
    if (tid == 0) {
      int n = 0;
      for (int j = 0; j < R; ++j) n += cnt[j];
      plan.nuniq[0] = n;
      plan.ustart[n] = R;
    }
  } else {
    for (int i = tid; i < R; i += 128) atomicAdd(&cnt[sidx[i]], 1);
    __syncthreads();
    plan_from_counts(cnt, off, E, R, 1, 0, plan, ws);
    plan_totals(cnt, E, 1, 0, plan);
    __syncthreads();
    for (int i = tid; i < R; i += 128) {
      const int ee = sidx[i];
      int rank = 0;
      for (int j = 0; j < i; ++j) rank += (sidx[j] == ee);
      const int pos = off[ee] + rank;
      plan.order[pos] = i;
      plan.inv[i] = pos;
    }
  }
  if (tid == 0) counters[0] = 0;
}

size_t decode_route_smem(int H) { return (size_t)(kDrRows + kDrTok) * H * 2; }

cudaError_t launch_decode_route(const uint16_t* x, const uint16_t* wr, const uint16_t* wg, int T,
                                int H, int E, int k, uint16_t* logits, float* gate_logit,
                                int32_t* idx, uint16_t* scores, const RoutePlan& plan,
                                int32_t* counters, int ncounters, cudaStream_t s) {
  const int per = (E + 31) / 32;
  const int nrows = E + (wg ? 1 : 0);
  const int grid = (nrows + kDrRows - 1) / kDrRows;
  const size_t smem = decode_route_smem(H);
  cudaError_t err = cudaSuccess;
#define TMOE_DR(P)                                                                              \
  do {                                                                                          \
    err = ensure_smem_attr((const void*)decode_route_kernel<P>, (int)smem);                     \
    if (err == cudaSuccess)                                                                     \
      err = launch_pdl(decode_route_kernel<P>, dim3(grid), dim3(128), smem, s, x, wr, wg, T, H, \
                       E, k, logits, gate_logit, idx, scores, plan, counters, ncounters);       \
  } while (0)
  if (per <= 4) TMOE_DR(4);
  else if (per <= 8) TMOE_DR(8);
  else if (per <= 16) TMOE_DR(16);
  else TMOE_DR(32);
#undef TMOE_DR
  if (err != cudaSuccess) return err;
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
