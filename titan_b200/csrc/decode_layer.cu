// Decode MoE layer in one launch (a few tokens, T <= kLayerMaxT).
//
// Same semantics as the three-launch decode pipeline (route.cu decode_route,
// decode.cu gate_up / down): router Linear with the canonical 8-partial dots,
// softmax + top-k by bf16 probability (lowest index on ties) and normalised
// scores (switch_layers.py / qwen3_5_moe/language.py:60-91), gate_up GEMV with
// fp32 h = silu(g) * u, down GEMV, and the ordered weighted sum plus the
// sigmoid-gated shared expert rounded to bf16 once
// (engine/patches/decode-fusion/fused_kernels.py:31-229).
//
// B200 mapping.  One CTA per SM, 8 warps, all CTAs resident at once, so CTAs
// may wait for each other's data.  There is no grid barrier:
//   * the logits carry the launch epoch in the same single-copy-atomic 64-bit
//     store as the value, and a reader re-loads a word until its tag is
//     current — one L2 round trip once the data is there (a barrier costs a
//     fence, an atomic and a poll before the data read even starts);
//   * h is published per gate_up tile by a release-increment of a 64-bit
//     counter that only grows; one thread per CTA polls that one word, then
//     the CTA reads h once (re-reading hot h lines from 148 SMs would crowd
//     the L2 slices that hold them).
// The epoch counter lives in the caller's workspace; CTA 0 advances it once
// every CTA has marked that it read it.  Every wait is bounded.
//   0. Before the dependency wait (programmatic dependent launch) each CTA
//      requests its router rows and the packed rows of its shared-expert
//      gate_up tiles: constant data, loaded while the previous layer ends.
//   1. x (T rows) is read once per CTA and kept in shared memory as bf16 (for
//      the router) and as the fp16 MMA operand with exact 64-group sums (for
//      gate_up).  Warp 0 computes the CTA's router rows and publishes them;
//      the other warps compute the shared expert's gate_up tiles meanwhile.
//   2. Every CTA waits for all logits and routes every token itself (one
//      warp per token) and builds the plan (pairs sorted by expert, distinct
//      experts): no second round trip.
//   3. The routed gate_up tiles (16 weight rows = 8 gate + 8 up rows over the
//      full K, one warp each) are spread over all CTAs, balanced against each
//      CTA's down work.  Every warp streams its tiles through a private ring
//      of 4.5 KB stages (16 rows x 512 K of packed int4 plus their bf16
//      scales and biases), cp.async issued NS-1 stages ahead, and publishes h
//      as the down projection's fp16 hi + lo operand.  The down rows of the
//      warp follow in the same ring, so they load while gate_up computes.
//   4. Each CTA waits for every gate_up tile, stages every pair's h with
//      exact group sums, computes the down tiles of its 16-row output slabs
//      for every selected expert and the shared expert, and folds them into y
//      in slot order plus the gated shared expert, inside the CTA: no ticket,
//      no partial sums in global memory.
//
// The phases run once per launch each, so the kernel's speed depends on how
// much of its code the SM's instruction cache holds: the tile MMA routine is
// out of line (one copy per variant) and loops that are not on a hot path
// stay rolled.
//
// MMA mapping (both GEMVs): m16n8k16, weights as A in exact fp16 (q - 8)
// (qpairs4), the token columns as B (n = 8, at most 8 columns per expert per
// call), fp32 accumulation; per 64-group acc += s * D + (b + 8s) * colsum.
// One warp owns a tile over the whole K, groups in ascending order.
#include "common.cuh"
#include "fragments.cuh"
#include "tmoe_internal.h"

namespace tmoe {

__device__ int g_layer_error = 0;

namespace {

constexpr int kLWarps = 8;
constexpr int kLThreads = kLWarps * 32;
constexpr int kChunkK = 512;                       // K per ring stage
constexpr int kRowStride = 256;                    // packed row slice (512 K); 16-byte chunk c of
                                                   // row r sits at chunk c ^ (r & 7): the
                                                   // fragment loads take the minimum 2 wavefronts
constexpr int kStageW = 16 * kRowStride;           // weights of one stage
constexpr int kStageBytes = kStageW + 2 * 16 * 16; // + bf16 scales and biases (16 rows x 8 groups)
constexpr int kMaxRowsPerCta = 8;                  // router rows per CTA
constexpr uint32_t kSpin = 1u << 17;               // polls before a wait gives up (~0.1 s)
constexpr uint32_t kFastPolls = 1u << 12;

// Exchanges between CTAs: relaxed single-copy-atomic accesses at GPU scope.
TMOE_DEV void st_tag32(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
TMOE_DEV void st_tag64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
TMOE_DEV uint32_t ld_tag32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
TMOE_DEV unsigned long long ld_tag64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// h as the down projection's operand: fp16 hi = h, lo = h - hi
TMOE_DEV uint32_t pack_h(float h) {
  const __half hi = __float2half_rn(h);
  const __half lo = __float2half_rn(__fsub_rn(h, __half2float(hi)));
  return (uint32_t)__half_as_ushort(hi) | ((uint32_t)__half_as_ushort(lo) << 16);
}
// n gate_up tiles' h are published: the warp's stores are ordered before the
// increment (warp barrier, then a release add by lane 0).
TMOE_DEV void publish_tiles(unsigned long long* cnt, unsigned long long n, int lane) {
  __syncwarp();
  if (lane == 0) asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(cnt), "l"(n) : "memory");
}
TMOE_DEV void spin_pause(uint32_t i) {
  if (i >= kFastPolls) __nanosleep(32);
}
// A wait that ran out: record it for the host and stop this CTA's other waits.
TMOE_DEV void wait_failed(volatile int* abort_flag) {
  *abort_flag = 1;
  atomicExch(&g_layer_error, 1);
}

template <int N>
TMOE_DEV void cp_async_wait_n() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

}  // namespace

// Shared-memory plan, identical on host and device.
struct LayerPlan {
  int ntp, rpc, R, spc, cs_r, cs_s, gi, gs;
  int off_xraw, off_x16, off_xs, off_rows, off_rt, off_bh, off_bl, off_bx, off_sh, off_sl, off_sx,
      off_res, off_ring, total;
  TMOE_HD LayerPlan(int T, int H, int E, int k, int I, int Is, int nct, int ns) {
    ntp = T <= 1 ? 1 : (T <= 2 ? 2 : 4);
    rpc = (E + 1 + nct - 1) / nct;
    R = T * k;
    spc = (H / 16 + nct - 1) / nct;
    cs_r = I * 2 + 16;
    cs_s = Is * 2 + 16;
    gi = I / 64;
    gs = Is / 64;
    int o = 0;
    off_xraw = o; o += ntp * H * 2;
    off_x16 = o;  o += T * H * 2;
    off_xs = o;   o += T * (H / 64) * 4;
    o = (o + 15) & ~15;
    off_rows = o; o += rpc * H * 2;
    off_rt = o;   o += (8 * R + 16) * 4;            // routing scratch (ints / floats)
    o = (o + 15) & ~15;
    // h operands: routed pairs, then the shared expert's T columns.  The
    // routing phase uses the same space first for the logits (T x E bf16).
    const int st0 = o;
    off_bh = o;   o += R * cs_r;
    off_bl = o;   o += R * cs_r;
    off_bx = o;   o += R * gi * 4;
    off_sh = o;   o += T * cs_s;
    off_sl = o;   o += T * cs_s;
    off_sx = o;   o += T * gs * 4;
    const int rt_end = st0 + T * E * 2;
    if (o < rt_end) o = rt_end;
    o = (o + 15) & ~15;
    off_res = o;  o += spc * (R + T) * 16 * 4;
    o = (o + 127) & ~127;
    off_ring = o; o += kLWarps * ns * kStageBytes;
    total = o;
  }
};

namespace {

struct Job {
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  int K, half_n, row0, kind;   // kind: 0 gate_up (8 gate + 8 up rows), 1 down (16 rows)
  int u;                       // distinct-expert slot; nuniq = the shared expert
  int slab;                    // down: local slab index
};

TMOE_DEV int job_row(const Job& jb, int r) {
  return jb.kind == 0 ? (r < 8 ? jb.row0 + r : jb.half_n + jb.row0 + (r - 8)) : jb.row0 + r;
}

// cp.async of stage `ch` (K range [512 ch, 512 ch + 512)) of a job: 16 rows x
// 256 B of packed weights (8 copies per lane) and 16 rows x 8 bf16 scales and
// biases (one copy per lane).
TMOE_DEV void issue_stage(uint8_t* st, const Job& jb, int ch, int lane) {
  const int KW = jb.K / 8, G = jb.K / 64;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int i = lane + 32 * m, r = i >> 4, c = i & 15;
    cp_async16(st + r * kRowStride + ((c ^ (r & 7)) << 4),
               jb.w + (size_t)job_row(jb, r) * KW + ch * 64 + c * 4);
  }
  const int r = lane & 15;
  const uint16_t* src = (lane < 16 ? jb.s : jb.b) + (size_t)job_row(jb, r) * G + ch * 8;
  cp_async16(st + kStageW + (lane >> 4) * 256 + r * 16, src);
}

// One stage of MMAs: 8 groups; B columns from bgh (+ bgl for fp32 sources
// split into hi + lo), column sums xs0 / xs1 for the thread's two D columns.
// Two groups per iteration and separate hi / lo accumulators, so four
// independent MMA chains are in flight (each MMA waits for the previous one
// on the same accumulator); out of line, one copy per variant.
template <bool LO>
__device__ __noinline__ float4 stage_mma(const uint8_t* st, int gbase, const uint8_t* bgh,
                                         const uint8_t* bgl, const float* xs0, const float* xs1,
                                         int g, int t, float4 acc4) {
  float acc[4] = {acc4.x, acc4.y, acc4.z, acc4.w};
  const uint8_t* wp = st + g * kRowStride + (t & 1) * 8;   // rows g and g + 8 share the swizzle
  const uint16_t* sp = reinterpret_cast<const uint16_t*>(st + kStageW);
  const uint16_t* bp = sp + 128;
#pragma unroll 1
  for (int j0 = 0; j0 < 8; j0 += 2) {
    float d[2][4], e[2][4];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int j = j0 + u;
      const int sw = ((2 * j + (t >> 1)) ^ g) << 4;          // chunk 2j + t/2 of rows g, g + 8
      const uint2 wl = *reinterpret_cast<const uint2*>(wp + sw);
      const uint2 wh = *reinterpret_cast<const uint2*>(wp + 8 * kRowStride + sw);
      const int gj = gbase + j;
      const uint4* hp = reinterpret_cast<const uint4*>(bgh + gj * 128 + t * 32);
      const uint4 h0 = hp[0], h1 = hp[1];
      uint4 l0 = h0, l1 = h1;
      if (LO) {
        const uint4* lp = reinterpret_cast<const uint4*>(bgl + gj * 128 + t * 32);
        l0 = lp[0];
        l1 = lp[1];
      }
      uint32_t qL[8], qH[8];
      qpairs4(wl.x, qL);
      qpairs4(wl.y, qL + 4);
      qpairs4(wh.x, qH);
      qpairs4(wh.y, qH + 4);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        d[u][q] = 0.0f;
        e[u][q] = 0.0f;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int pi = (kk >> 1) * 4 + (kk & 1) * 2;
        const uint32_t a0 = qL[pi], a1 = qH[pi], a2 = qL[pi + 1], a3 = qH[pi + 1];
        const uint4 hb = (kk < 2) ? h0 : h1;
        mma16816(d[u], a0, a1, a2, a3, (kk & 1) ? hb.z : hb.x, (kk & 1) ? hb.w : hb.y);
        if (LO) {
          const uint4 lb = (kk < 2) ? l0 : l1;
          mma16816(e[u], a0, a1, a2, a3, (kk & 1) ? lb.z : lb.x, (kk & 1) ? lb.w : lb.y);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int j = j0 + u, gj = gbase + j;
      if (LO) {
#pragma unroll
        for (int q = 0; q < 4; ++q) d[u][q] = __fadd_rn(d[u][q], e[u][q]);
      }
      const float sl = bf2f(sp[g * 8 + j]), sh = bf2f(sp[(g + 8) * 8 + j]);
      const float bl = __fadd_rn(bf2f(bp[g * 8 + j]), __fmul_rn(8.0f, sl));
      const float bh = __fadd_rn(bf2f(bp[(g + 8) * 8 + j]), __fmul_rn(8.0f, sh));
      const float x0 = xs0[gj], x1 = xs1[gj];
      acc[0] = __fmaf_rn(sl, d[u][0], __fmaf_rn(bl, x0, acc[0]));
      acc[1] = __fmaf_rn(sl, d[u][1], __fmaf_rn(bl, x1, acc[1]));
      acc[2] = __fmaf_rn(sh, d[u][2], __fmaf_rn(bh, x0, acc[2]));
      acc[3] = __fmaf_rn(sh, d[u][3], __fmaf_rn(bh, x1, acc[3]));
    }
  }
  return make_float4(acc[0], acc[1], acc[2], acc[3]);
}

}  // namespace

// Per-CTA job lists after routing (identical arithmetic in every CTA).
struct CtaWork {
  int nuniq, nu_dn, ngu, g0, g1, nslab_c, ndn;
};

TMOE_DEV CtaWork cta_work(int c, int nct, int nuniq, int T, int H, int I, int Is) {
  CtaWork w;
  w.nuniq = nuniq;
  w.nu_dn = nuniq + (Is > 0 ? 1 : 0);
  const int per_exp = I / 8;                          // gate_up tiles per expert
  w.ngu = nuniq * per_exp;
  const int nslab = H / 16;
  const int q = nslab / nct, rr = nslab % nct;
  w.nslab_c = q + (c < rr ? 1 : 0);
  w.ndn = w.nslab_c * w.nu_dn;
  // cost in stages: gate_up tile H/512, down tile I/512 (shared Is/512)
  const float cg = (float)(H / kChunkK);
  const float dslab = (float)(nuniq * (I / kChunkK) + (Is > 0 ? Is / kChunkK : 0));
  const float total = (float)w.ngu * cg + (float)nslab * dslab;
  const float target = total / (float)nct;
  const float capA = fmaxf(0.0f, target - (float)(q + 1) * dslab);
  const float capB = fmaxf(0.0f, target - (float)q * dslab);
  const float sumcap = (float)rr * capA + (float)(nct - rr) * capB;
  const float scale = sumcap > 0.0f ? (float)w.ngu * cg / sumcap : 0.0f;
  auto prefix = [&](int cc) -> int {
    if (cc >= nct) return w.ngu;
    const float p = scale * ((float)min(cc, rr) * capA + (float)max(0, cc - rr) * capB);
    const int v = (int)floorf(p / cg + 0.5f);
    return v < 0 ? 0 : (v > w.ngu ? w.ngu : v);
  };
  w.g0 = prefix(c);
  w.g1 = prefix(c + 1);
  if (w.g1 < w.g0) w.g1 = w.g0;
  return w;
}

template <int NS>
__global__ void __launch_bounds__(kLThreads, 1) decode_layer_kernel(LayerArgs A) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int c = blockIdx.x, nct = gridDim.x;
  const int T = A.T, H = A.H, E = A.E, k = A.k, I = A.I, Is = A.Is;
  const LayerPlan L(T, H, E, k, I, Is, nct, NS);
  const int R = L.R, G = H / 64;
  uint8_t* ring = sm + L.off_ring + warp * NS * kStageBytes;
  uint16_t* xraw = reinterpret_cast<uint16_t*>(sm + L.off_xraw);
  uint8_t* x16 = sm + L.off_x16;
  float* xs = reinterpret_cast<float*>(sm + L.off_xs);
  uint4* rows = reinterpret_cast<uint4*>(sm + L.off_rows);
  int32_t* rt = reinterpret_cast<int32_t*>(sm + L.off_rt);
  int32_t* s_idx = rt;                    // [R] expert of pair (token-major)
  int32_t* s_order = s_idx + R;           // [R] pair at sorted position
  int32_t* s_pos = s_order + R;           // [R] sorted position of pair
  int32_t* s_first = s_pos + R;           // [R]
  int32_t* s_uexp = s_first + R;          // [R + 1]
  int32_t* s_ustart = s_uexp + R + 1;     // [R + 2]
  float* s_score = reinterpret_cast<float*>(s_ustart + R + 2);   // [R] bf16 score as float
  int32_t* s_nuniq = reinterpret_cast<int32_t*>(s_score + R);
  float* s_gate = reinterpret_cast<float*>(s_nuniq + 1);         // [T] sigmoid(gate logit)
  const int nch_h = H / 8;                // 16-byte chunks of a router row

  // ---- 0: constant data before the dependency wait
  if (warp == 0) {
    for (int j = 0; j < L.rpc; ++j) {
      const int er = c + j * nct;
      const bool ok = er < E || (er == E && A.wg != nullptr);
      const uint16_t* row = ok ? ((er < E) ? A.wr + (size_t)er * H : A.wg) : A.wr;
      for (int cc = lane; cc < nch_h; cc += 32)
        cp_async16_zfill(&rows[j * nch_h + cc], row + (size_t)cc * 8, ok);
    }
    cp_async_commit();
  }
  // shared-expert gate_up tiles of this warp (warps 1..7): tile c + nct * (warp - 1 + 7 m)
  const int nsh_tiles = Is / 8;
  auto sh_job = [&](int m) -> Job {
    Job jb;
    const int st = c + nct * (warp - 1 + (kLWarps - 1) * m);
    jb.w = A.sguw;
    jb.s = A.sgus;
    jb.b = A.sgub;
    jb.K = H;
    jb.half_n = Is;
    jb.row0 = st * 8;
    jb.kind = 0;
    jb.u = -1;
    jb.slab = 0;
    return jb;
  };
  int n_sh = 0;
  if (warp > 0 && Is > 0) {
    const int first = c + nct * (warp - 1);
    if (first < nsh_tiles) n_sh = (nsh_tiles - 1 - first) / (nct * (kLWarps - 1)) + 1;
  }
  const int cgu = H / kChunkK;              // stages per gate_up tile
  // ring cursor over the shared gate_up stages of this warp
  int sh_issue = 0;
  const int sh_total = n_sh * cgu;
  auto sh_issue_next = [&]() {
    if (sh_issue < sh_total) {
      const Job jb = sh_job(sh_issue / cgu);
      issue_stage(ring + (sh_issue % NS) * kStageBytes, jb, sh_issue % cgu, lane);
    }
    cp_async_commit();
    ++sh_issue;
  };
  if (warp > 0)
    for (int i = 0; i < NS - 1; ++i) sh_issue_next();

  pdl_wait();
  pdl_trigger();
  // this launch's epoch: one more than the counter (CTA 0 advances it once
  // every CTA has read it); every CTA marks that it has seen it.  The gate_up
  // counter as it stands: no CTA adds to it before every CTA has published its
  // logits, which each does after this read.
  __shared__ int s_epoch;
  __shared__ int s_abort;
  __shared__ unsigned long long s_gubase;
  if (tid == 0) {
    s_abort = 0;
    s_gubase = ld_tag64(A.gucnt);
    const int ep = (int)ld_tag32(reinterpret_cast<const uint32_t*>(A.epoch)) + 1;
    s_epoch = ep;
    st_tag32(reinterpret_cast<uint32_t*>(A.tseen) + c, (uint32_t)ep);
  }

  // ---- 1: x -> bf16 copy (router) + fp16 operand with exact group sums
  {
    const int nblk = T * (H / 16);
    for (int base = 0; base < nblk; base += kLThreads) {
      const int b = base + tid;
      float sum = 0.0f, bmax = 0.0f;
      if (b < nblk) {
        const int tt = b / (H / 16), bb = b % (H / 16);
        const uint4* src = reinterpret_cast<const uint4*>(A.x + (size_t)tt * H + bb * 16);
        const uint4 u0 = __ldcg(src), u1 = __ldcg(src + 1);
        uint4* draw = reinterpret_cast<uint4*>(xraw + (size_t)tt * H + bb * 16);
        draw[0] = u0;
        draw[1] = u1;
        const uint32_t w8[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
        uint16_t hv[16];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float v0 = bf2f((uint16_t)(w8[q] & 0xffffu)), v1 = bf2f((uint16_t)(w8[q] >> 16));
          bmax = fmaxf(bmax, fmaxf(fabsf(v0), fabsf(v1)));
          const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
          hv[f16p_pos(2 * q)] = __half_as_ushort(h0);
          hv[f16p_pos(2 * q + 1)] = __half_as_ushort(h1);
          sum = __fadd_rn(sum, __half2float(h0));
          sum = __fadd_rn(sum, __half2float(h1));
        }
        uint4* dh = reinterpret_cast<uint4*>(x16 + ((size_t)tt * H + bb * 16) * 2);
        dh[0] = make_uint4(hv[0] | ((uint32_t)hv[1] << 16), hv[2] | ((uint32_t)hv[3] << 16),
                           hv[4] | ((uint32_t)hv[5] << 16), hv[6] | ((uint32_t)hv[7] << 16));
        dh[1] = make_uint4(hv[8] | ((uint32_t)hv[9] << 16), hv[10] | ((uint32_t)hv[11] << 16),
                           hv[12] | ((uint32_t)hv[13] << 16), hv[14] | ((uint32_t)hv[15] << 16));
      }
      sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
      sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
      bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));
      bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 2));
      if (b < nblk && (b & 3) == 0) {
        xs[(b / (H / 16)) * G + (b % (H / 16)) / 4] = sum;
        // x is staged as fp16: exact only inside fp16's normal range
        if (c == 0 && !fp16_group_ok(bmax)) atomicExch(&g_layer_error, 2);
      }
    }
  }
  __syncthreads();
  const int epoch = s_epoch;

  if (warp == 0) {
    // ---- router rows of this CTA: 4 rows per pass, 8 lanes (partials) each
    cp_async_wait_n<0>();
    __syncwarp();
    const int p = lane & 7, sub = lane >> 3;
    const uint4* xsm = reinterpret_cast<const uint4*>(xraw);
    for (int j0 = 0; j0 < L.rpc; j0 += 4) {
      const int j = j0 + sub;
      const int er = c + j * nct;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const uint4* wrow = rows + (j < L.rpc ? j : 0) * nch_h;
      if (L.ntp == 1)
        router_dots<1>(wrow, xsm, nch_h, p, acc);
      else if (L.ntp == 2)
        router_dots<2>(wrow, xsm, nch_h, p, acc);
      else
        router_dots<4>(wrow, xsm, nch_h, p, acc);
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        const float s8 = tree8(acc[tt]);
        if (j < L.rpc && p == tt && tt < T) {
          if (er < E)
            st_tag64(A.tlog + (size_t)tt * E + er,
                     (unsigned long long)f2bf(s8) | ((unsigned long long)(uint32_t)epoch << 32));
          else if (er == E && A.wg)
            st_tag64(A.tgate + tt, (unsigned long long)__float_as_uint(s8) |
                                       ((unsigned long long)(uint32_t)epoch << 32));
        }
      }
    }
  } else {
    // ---- the shared expert's gate_up tiles (independent of the routing)
    int seq = 0;
    for (int m = 0; m < n_sh; ++m) {
      const Job jb = sh_job(m);
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      const int c0 = min(2 * t, T - 1), c1 = min(2 * t + 1, T - 1);
      const uint8_t* bgh = x16 + (size_t)min(g, T - 1) * H * 2;
      for (int ch = 0; ch < cgu; ++ch, ++seq) {
        sh_issue_next();
        cp_async_wait_n<NS - 1>();
        __syncwarp();
        acc = stage_mma<false>(ring + (seq % NS) * kStageBytes, ch * 8, bgh, bgh, xs + c0 * G,
                               xs + c1 * G, g, t, acc);
        __syncwarp();
      }
      const int row = jb.row0 + g;
      if (2 * t < T) A.ths[(size_t)(2 * t) * Is + row] = pack_h(silu_mul_f32(acc.x, acc.z));
      if (2 * t + 1 < T) A.ths[(size_t)(2 * t + 1) * Is + row] = pack_h(silu_mul_f32(acc.y, acc.w));
    }
    cp_async_wait_n<0>();
    __syncwarp();
  }
  __syncthreads();

  // ---- 2: every thread waits for its words of this launch's logits (CTA 0
  // also for every CTA's start mark, after which it advances the epoch)
  uint16_t* lg_s = reinterpret_cast<uint16_t*>(sm + L.off_bh);
  {
    const int n = T * E;
    const int nseen = c == 0 ? nct : 0;
    for (int i = tid; i < n + T + nseen; i += kLThreads) {
      bool done = false;
      for (uint32_t it = 0; it < kSpin && !(it >= kFastPolls && *(volatile int*)&s_abort);
           ++it, spin_pause(it)) {
        if (i < n) {
          const unsigned long long w = ld_tag64(A.tlog + i);
          if ((int)(w >> 32) == epoch) {
            lg_s[i] = (uint16_t)(w & 0xffffu);
            done = true;
          }
        } else if (i < n + T) {
          if (!A.wg) {
            done = true;
          } else {
            const unsigned long long w = ld_tag64(A.tgate + (i - n));
            if ((int)(w >> 32) == epoch) {
              s_gate[i - n] = csigmoid(__uint_as_float((uint32_t)w));
              done = true;
            }
          }
        } else {
          done = (int)ld_tag32(reinterpret_cast<const uint32_t*>(A.tseen) + (i - n - T)) == epoch;
        }
        if (done) break;
      }
      if (!done) wait_failed(&s_abort);
    }
  }
  __syncthreads();
  if (c == 0 && tid == 0) st_tag32(reinterpret_cast<uint32_t*>(A.epoch), (uint32_t)epoch);
  // every CTA has read the gate_up counter by now: the shared-expert tiles of
  // phase 1 are counted from here
  if (n_sh > 0) publish_tiles(A.gucnt, (unsigned long long)n_sh, lane);
  // Routing: warp w routes token w (route_token: keys in registers, sorted
  // per lane, k rounds of warp max over the lane heads)
  if (warp < T) {
    const int tt = warp;
    const uint16_t* lg = lg_s + (size_t)tt * E;
    const int per = (E + 31) / 32;
    RouteOut ro;
    if (per <= 4)
      ro = route_token<4>(lg, E, k, lane);
    else if (per <= 8)
      ro = route_token<8>(lg, E, k, lane);
    else if (per <= 16)
      ro = route_token<16>(lg, E, k, lane);
    else
      ro = route_token<32>(lg, E, k, lane);
    if (lane < k) {
      s_idx[tt * k + lane] = ro.e;
      s_score[tt * k + lane] = bf2f(ro.score);
      if (c == 0) {
        A.idx[(size_t)tt * k + lane] = ro.e;
        A.scores[(size_t)tt * k + lane] = ro.score;
      }
    }
  }
  __syncthreads();
  // plan: stable sort of the pairs by expert, distinct experts in order
  if (tid < R) {
    const int e = s_idx[tid];
    const int key = e * 128 + tid;
    int pos = 0, first = 1;
    for (int j = 0; j < R; ++j) {
      const int ej = s_idx[j];
      pos += (ej * 128 + j) < key;
      if (ej == e && j < tid) first = 0;
    }
    s_order[pos] = tid;
    s_pos[tid] = pos;
    s_first[tid] = first;
  }
  __syncthreads();
  if (tid < R && s_first[tid]) {
    const int e = s_idx[tid];
    int u = 0;
    for (int j = 0; j < R; ++j) u += (s_first[j] && s_idx[j] < e);
    s_uexp[u] = e;
    s_ustart[u] = s_pos[tid];
  }
  if (tid == 0) {
    int n = 0;
    for (int j = 0; j < R; ++j) n += s_first[j];
    s_nuniq[0] = n;
    s_ustart[n] = R;
  }
  __syncthreads();

  // ---- 3: routed gate_up tiles, then the down tiles, through the warp's ring
  const int nuniq = s_nuniq[0];
  const CtaWork W = cta_work(c, nct, nuniq, T, H, I, Is);
  const int n_gu_c = W.g1 - W.g0;
  const int ngw = warp < n_gu_c ? (n_gu_c - 1 - warp) / kLWarps + 1 : 0;
  const int d0 = ((warp - n_gu_c) % kLWarps + kLWarps) % kLWarps;
  const int ndw = d0 < W.ndn ? (W.ndn - 1 - d0) / kLWarps + 1 : 0;
  const int njobs = ngw + ndw;
  const int per_exp = I / 8;
  auto make_job = [&](int q) -> Job {
    Job jb;
    if (q < ngw) {
      const int gt = W.g0 + warp + kLWarps * q;
      const int u = gt / per_exp;
      const int e = s_uexp[u];
      jb.w = A.guw + (size_t)e * 2 * I * (H / 8);
      jb.s = A.gus + (size_t)e * 2 * I * G;
      jb.b = A.gub + (size_t)e * 2 * I * G;
      jb.K = H;
      jb.half_n = I;
      jb.row0 = (gt % per_exp) * 8;
      jb.kind = 0;
      jb.u = u;
      jb.slab = 0;
    } else {
      const int d = d0 + kLWarps * (q - ngw);
      const int js = d / W.nu_dn, u = d % W.nu_dn;
      jb.slab = js;
      jb.row0 = (c + js * nct) * 16;
      jb.kind = 1;
      jb.u = u;
      jb.half_n = 0;
      if (u < nuniq) {
        const int e = s_uexp[u];
        jb.w = A.dnw + (size_t)e * H * (I / 8);
        jb.s = A.dns + (size_t)e * H * (I / 64);
        jb.b = A.dnb + (size_t)e * H * (I / 64);
        jb.K = I;
      } else {
        jb.w = A.sdnw;
        jb.s = A.sdns;
        jb.b = A.sdnb;
        jb.K = Is;
      }
    }
    return jb;
  };
  // issue cursor
  int iq = 0, ich = 0, issued = 0;
  Job ijob;
  if (njobs > 0) ijob = make_job(0);
  auto issue_next = [&]() {
    if (iq < njobs) {
      issue_stage(ring + (issued % NS) * kStageBytes, ijob, ich, lane);
      if (++ich == ijob.K / kChunkK) {
        ich = 0;
        if (++iq < njobs) ijob = make_job(iq);
      }
    }
    cp_async_commit();
    ++issued;
  };
  for (int i = 0; i < NS - 1; ++i) issue_next();
  int seq = 0;
  // gate_up
  for (int q = 0; q < ngw; ++q) {
    const Job jb = make_job(q);
    const int p0 = s_ustart[jb.u], nc = s_ustart[jb.u + 1] - p0;
    const int tg = s_order[p0 + min(g, nc - 1)] / k;
    const int tc0 = s_order[p0 + min(2 * t, nc - 1)] / k;
    const int tc1 = s_order[p0 + min(2 * t + 1, nc - 1)] / k;
    const uint8_t* bgh = x16 + (size_t)tg * H * 2;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int ch = 0; ch < cgu; ++ch, ++seq) {
      issue_next();
      cp_async_wait_n<NS - 1>();
      __syncwarp();
      acc = stage_mma<false>(ring + (seq % NS) * kStageBytes, ch * 8, bgh, bgh, xs + tc0 * G,
                             xs + tc1 * G, g, t, acc);
      __syncwarp();
    }
    const int row = jb.row0 + g;
    if (2 * t < nc) A.th[(size_t)s_order[p0 + 2 * t] * I + row] = pack_h(silu_mul_f32(acc.x, acc.z));
    if (2 * t + 1 < nc)
      A.th[(size_t)s_order[p0 + 2 * t + 1] * I + row] = pack_h(silu_mul_f32(acc.y, acc.w));
    publish_tiles(A.gucnt, 1ull, lane);
  }

  // ---- 4: wait until every gate_up tile of this launch is published (one
  // thread polls one counter), then stage h (routed pairs, then the shared
  // expert's tokens) as fp16 hi + lo with exact group sums of hi + lo; two
  // 16-element blocks per thread and pass, loaded before either is converted
  if (tid == 0) {
    const unsigned long long need = (unsigned long long)(nuniq * (I / 8) + (Is > 0 ? Is / 8 : 0));
    bool ok = false;
    for (uint32_t it = 0; it < kSpin; ++it, spin_pause(it))
      if (ld_tag64(A.gucnt) - s_gubase >= need) {
        ok = true;
        break;
      }
    if (!ok) wait_failed(&s_abort);
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
  }
  __syncthreads();
  {
    const int nb_r = R * (I / 16), nb_s = T * (Is / 16), nb = nb_r + nb_s;
    for (int base = 0; base < nb; base += 2 * kLThreads) {
      uint32_t hl[2][16];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int b = base + hh * kLThreads + tid;
        if (b < nb) {
          const bool shared = b >= nb_r;
          const int K = shared ? Is : I;
          const int bb = shared ? b - nb_r : b;
          const uint4* src = reinterpret_cast<const uint4*>(
              (shared ? A.ths : A.th) + (size_t)(bb / (K / 16)) * K + (bb % (K / 16)) * 16);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 w = __ldcg(src + q);
            hl[hh][4 * q] = w.x;
            hl[hh][4 * q + 1] = w.y;
            hl[hh][4 * q + 2] = w.z;
            hl[hh][4 * q + 3] = w.w;
          }
        }
      }
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int b = base + hh * kLThreads + tid;
        const bool ok = b < nb;
        const bool shared = b >= nb_r;
        const int K = shared ? Is : I;
        const int bb = shared ? b - nb_r : b;
        const int col = bb / (K / 16), blk = bb % (K / 16);
        float sum = 0.0f;
        if (ok) {
          uint16_t hv[16], lv[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const uint16_t hb = (uint16_t)(hl[hh][q] & 0xffffu), lb = (uint16_t)(hl[hh][q] >> 16);
            hv[f16p_pos(q)] = hb;
            lv[f16p_pos(q)] = lb;
            sum = __fadd_rn(sum, __fadd_rn(__half2float(__ushort_as_half(hb)),
                                           __half2float(__ushort_as_half(lb))));
          }
          const int cs = shared ? L.cs_s : L.cs_r;
          uint4* dh = reinterpret_cast<uint4*>(sm + (shared ? L.off_sh : L.off_bh) + (size_t)col * cs + blk * 32);
          uint4* dl = reinterpret_cast<uint4*>(sm + (shared ? L.off_sl : L.off_bl) + (size_t)col * cs + blk * 32);
          dh[0] = make_uint4(hv[0] | ((uint32_t)hv[1] << 16), hv[2] | ((uint32_t)hv[3] << 16),
                             hv[4] | ((uint32_t)hv[5] << 16), hv[6] | ((uint32_t)hv[7] << 16));
          dh[1] = make_uint4(hv[8] | ((uint32_t)hv[9] << 16), hv[10] | ((uint32_t)hv[11] << 16),
                             hv[12] | ((uint32_t)hv[13] << 16), hv[14] | ((uint32_t)hv[15] << 16));
          dl[0] = make_uint4(lv[0] | ((uint32_t)lv[1] << 16), lv[2] | ((uint32_t)lv[3] << 16),
                             lv[4] | ((uint32_t)lv[5] << 16), lv[6] | ((uint32_t)lv[7] << 16));
          dl[1] = make_uint4(lv[8] | ((uint32_t)lv[9] << 16), lv[10] | ((uint32_t)lv[11] << 16),
                             lv[12] | ((uint32_t)lv[13] << 16), lv[14] | ((uint32_t)lv[15] << 16));
        }
        sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
        sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
        if (ok && (blk & 3) == 0) {
          float* xsum = reinterpret_cast<float*>(sm + (shared ? L.off_sx : L.off_bx));
          xsum[col * (K / 64) + blk / 4] = sum;
        }
      }
    }
  }
  __syncthreads();
  // down tiles
  float* res = reinterpret_cast<float*>(sm + L.off_res);
  for (int q = ngw; q < njobs; ++q) {
    const Job jb = make_job(q);
    const bool shared = jb.u >= nuniq;
    const int p0 = shared ? 0 : s_ustart[jb.u];
    const int nc = shared ? T : s_ustart[jb.u + 1] - p0;
    auto col_of = [&](int cc) { return shared ? cc : s_order[p0 + cc]; };
    const int cg_ = col_of(min(g, nc - 1));
    const int cc0 = col_of(min(2 * t, nc - 1)), cc1 = col_of(min(2 * t + 1, nc - 1));
    const int cs = shared ? L.cs_s : L.cs_r;
    const uint8_t* bgh = sm + (shared ? L.off_sh : L.off_bh) + (size_t)cg_ * cs;
    const uint8_t* bgl = sm + (shared ? L.off_sl : L.off_bl) + (size_t)cg_ * cs;
    const float* xsum = reinterpret_cast<const float*>(sm + (shared ? L.off_sx : L.off_bx));
    const int gk = jb.K / 64;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const int nchk = jb.K / kChunkK;
    for (int ch = 0; ch < nchk; ++ch, ++seq) {
      issue_next();
      cp_async_wait_n<NS - 1>();
      __syncwarp();
      acc = stage_mma<true>(ring + (seq % NS) * kStageBytes, ch * 8, bgh, bgl, xsum + cc0 * gk,
                            xsum + cc1 * gk, g, t, acc);
      __syncwarp();
    }
    float* rs = res + (size_t)jb.slab * (R + T) * 16;
    const int base_col = shared ? R : 0;
    if (2 * t < nc) {
      const int cl = base_col + col_of(2 * t);
      rs[cl * 16 + g] = acc.x;
      rs[cl * 16 + g + 8] = acc.z;
    }
    if (2 * t + 1 < nc) {
      const int cl = base_col + col_of(2 * t + 1);
      rs[cl * 16 + g] = acc.y;
      rs[cl * 16 + g + 8] = acc.w;
    }
  }
  cp_async_wait_n<0>();
  __syncthreads();
  // weighted sum in slot order + the gated shared expert, per output slab; a
  // CTA whose wait gave up writes NaN, so its slabs cannot pass for a result
  const bool failed = *(volatile int*)&s_abort != 0;
  for (int js = 0; js < W.nslab_c; ++js) {
    const int slab = c + js * nct;
    const float* rs = res + (size_t)js * (R + T) * 16;
    for (int i = tid; i < T * 16; i += kLThreads) {
      const int tt = i >> 4, r = i & 15;
      float a = 0.0f;
      for (int j = 0; j < k; ++j) a = __fmaf_rn(s_score[tt * k + j], rs[(tt * k + j) * 16 + r], a);
      if (Is > 0) a = __fmaf_rn(s_gate[tt], rs[(R + tt) * 16 + r], a);
      A.y[(size_t)tt * H + slab * 16 + r] = failed ? (uint16_t)0x7fc0u : f2bf(a);
    }
  }
}

size_t decode_layer_smem(int T, int H, int E, int k, int I, int Is, int nct, int ns) {
  return (size_t)LayerPlan(T, H, E, k, I, Is, nct, ns).total;
}

// Largest ring depth whose plan fits in shared memory, or 0 when the layer
// cannot take the single-launch path.
int decode_layer_stages(int T, int H, int E, int k, int I, int Is, int nct) {
  if (T < 1 || T > kLayerMaxT || T * k > 128 || k > 32 || E > 1024 || E < k) return 0;
  if (nct > kLayerMaxCtas) return 0;
  if (H % kChunkK || I % kChunkK || (Is > 0 && Is % kChunkK)) return 0;
  if ((E + 1 + nct - 1) / nct > kMaxRowsPerCta) return 0;
  for (int ns = 4; ns >= 2; --ns)
    if (decode_layer_smem(T, H, E, k, I, Is, nct, ns) <= 232448 - 4096) return ns;   // + static
  return 0;
}

int decode_layer_ctas() { return device_sm_count(); }

cudaError_t launch_decode_layer(const LayerArgs& a, int ns, cudaStream_t s) {
  const int nct = decode_layer_ctas();
  const size_t smem = decode_layer_smem(a.T, a.H, a.E, a.k, a.I, a.Is, nct, ns);
  cudaError_t err = cudaSuccess;
  auto go = [&](auto kernel) {
    cudaError_t e = ensure_smem_attr((const void*)kernel, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kLThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;   // the CTAs could not all be resident
    // cooperative: the driver guarantees every CTA is resident at once (the
    // CTAs wait for each other's data) or refuses the launch
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nct);
    cfg.blockDim = dim3(kLThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, a);
  };
  if (ns == 4) err = go(decode_layer_kernel<4>);
  else if (ns == 3) err = go(decode_layer_kernel<3>);
  else err = go(decode_layer_kernel<2>);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

int layer_error_flag() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_layer_error, sizeof(int));
  return v;
}

}  // namespace tmoe
