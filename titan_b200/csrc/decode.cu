// Decode-shaped MoE (a handful of tokens): grouped GEMVs over the distinct
// experts the batch selected, on the tensor cores.
//
// Follows engine/patches/decode-fusion/fused_kernels.py:31-229 (gate_up_silu
// and down_wsum): fp32 accumulation, h = silu(g)*u kept in fp32, the routed
// weighted sum and the sigmoid-gated shared expert folded in fp32 and rounded
// to bf16 once.
//
// B200 mapping.  A CTA (4 warps) owns one (expert, 32-weight-row slab); the
// K dimension is split four ways, one contiguous quarter per warp, so a warp
// stages, converts and multiplies only its own quarter and no CTA barrier is
// taken before the final 4-way reduction.  Every warp first issues cp.async
// copies of its activation columns, then of its packed int4 rows in two
// halves and the loads of its scales; it converts the columns as soon as they
// land and multiplies the first half of its rows while the second half is
// still in flight.  Conversion: bf16 x -> fp16 (exact for
// normal-range values), or fp32 h -> fp16 hi + lo halves, each with exact fp32
// group sums of the operand it stored.  The MMAs are m16n8k16 with the weights
// as the A operand in exact fp16 (q - 8) (0x6400|q is 1024 + q: nine integer /
// half2 ops per eight weights) and the activations as B.  Per 64-group the
// fp32 MMA result is scaled on the CUDA cores:
// acc += s * D + (b + 8s) * sum(column over the group).
//
// Modes: 0 = gate_up rows (i, I + i) -> h = silu(g) * u fp32; 1 = down ->
// fp32 partial per (token, slot) and, in the last CTA to finish a 32-row
// output slab (a device-wide counter, nobody waits), the ordered weighted sum
// plus the gated shared expert -> bf16 y; 2 = plain bf16 output rows (the
// stock gather).
#include "common.cuh"
#include "fragments.cuh"
#include "tmoe_internal.h"

namespace tmoe {

__device__ int g_decode_range = 0;   // bf16 x outside fp16's exact range (sticky)

int decode_range_flag() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_decode_range, sizeof(int));
  return v;
}

namespace {

constexpr int kSlabRows = 32;   // weight rows per CTA (two m16 tiles)
constexpr int kCols = 8;        // activation columns per MMA pass (n = 8)
constexpr int kColsPerPass = 2; // columns staged per pass (at most kCols)
constexpr int kThreads = 128;   // 4 warps, one K quarter each
constexpr int kWarps = 4;
constexpr int kMaxGw = 12;      // groups per warp whose scales are held in registers

// Per-warp shared-memory plan, identical on host and device.
struct GemvPlan {
  int gw;                 // groups per warp (the largest quarter)
  int wstride;            // bytes per weight row slice (== 8 words mod 32: rows
                          // 0..3 of a fragment load hit distinct banks)
  int cstride;            // bytes per staged column slice (== 16 mod 128)
  int ncol;               // columns staged per pass
  int rstride;            // bytes per raw (source-format) column slice
  int w_off, sb_off, xh_off, xl_off, xs_off, raw_off, warp_bytes, red_off, total;
  TMOE_HD GemvPlan(int K, int ncol_, bool lo) {
    const int G = K / kGroup;
    gw = (G + kWarps - 1) / kWarps;
    const int words = gw * 8;
    wstride = (words + ((8 - words) % 32 + 32) % 32) * 4;
    cstride = gw * 128 + 16;
    ncol = ncol_;
    w_off = 0;
    sb_off = w_off + kSlabRows * wstride;
    xh_off = sb_off + gw * kSlabRows * 8;
    xl_off = xh_off + ncol * cstride;
    xs_off = xl_off + (lo ? ncol * cstride : 0);
    raw_off = (xs_off + ncol * gw * 4 + 15) & ~15;
    rstride = gw * 64 * (lo ? 4 : 2);
    warp_bytes = raw_off + ncol * rstride;
    red_off = kWarps * warp_bytes;
    total = red_off + kWarps * 2 * 32 * 16;
  }
};

// Columns [cb, cb + nc) of this warp's K quarter [k0, k0 + kq), in two steps
// so the loads can be issued ahead of the weights: issue_columns() starts
// cp.async copies of the source rows (bf16 x or fp32 h) into the raw area;
// after they land, convert_columns() writes the fp16 operand blocks (hi, and
// lo for fp32 sources) plus exact fp32 sums of the stored operands per
// 64-group.  Columns nc..ncol-1 are left alone (the MMA reads column nc-1 in
// their place).
template <int MODE>
TMOE_DEV void issue_columns(const StreamParams& P, const GemvPlan& L, uint8_t* wsm, bool shared,
                            int p0, int cb, int nc, int k0, int kq, int lane) {
  const int K = shared ? P.K_sh : P.K;
  constexpr int esz = MODE == 1 ? 4 : 2;
  const int chunks = kq * esz / 16;             // 16-byte chunks per column slice
  for (int c = 0; c < nc; ++c) {
    const int col = cb + c;
    const uint8_t* src;
    if (MODE == 1)
      src = reinterpret_cast<const uint8_t*>(shared ? P.h_sh + (size_t)col * K
                                                    : P.h + (size_t)P.order[p0 + col] * K);
    else  // one token: every column is row 0, no lookup of the plan's order
      src = reinterpret_cast<const uint8_t*>(
          P.x + (size_t)(shared || P.tokens == 1 ? (shared ? col : 0)
                                                  : P.order[p0 + col] / P.col_div) * K);
    src += (size_t)k0 * esz;
    for (int i = lane; i < chunks; i += 32)
      cp_async16(wsm + L.raw_off + c * L.rstride + i * 16, src + i * 16);
  }
}

template <int MODE>
TMOE_DEV void convert_columns(const GemvPlan& L, uint8_t* wsm, int nc, int kq, int lane) {
  const int nblk = kq / 16;                      // 16-element blocks in the quarter
  for (int c = 0; c < nc; ++c) {
    uint16_t* xh = reinterpret_cast<uint16_t*>(wsm + L.xh_off + c * L.cstride);
    uint16_t* xl = reinterpret_cast<uint16_t*>(wsm + L.xl_off + c * L.cstride);
    float* xs = reinterpret_cast<float*>(wsm + L.xs_off) + c * L.gw;
    const uint8_t* raw = wsm + L.raw_off + c * L.rstride;
    for (int b0 = 0; b0 < nblk; b0 += 32) {
      const int b = b0 + lane;
      float sum = 0.0f, bmax = 0.0f;
      if (b < nblk) {
        float v[16];
        if (MODE == 1) {
          const float4* s4 = reinterpret_cast<const float4*>(raw + b * 64);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 f = s4[q];
            v[4 * q] = f.x;
            v[4 * q + 1] = f.y;
            v[4 * q + 2] = f.z;
            v[4 * q + 3] = f.w;
          }
        } else {
          const uint4* s4 = reinterpret_cast<const uint4*>(raw + b * 32);
          const uint4 u0 = s4[0], u1 = s4[1];
          const uint32_t w8[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            v[2 * q] = bf2f((uint16_t)(w8[q] & 0xffffu));
            v[2 * q + 1] = bf2f((uint16_t)(w8[q] >> 16));
            bmax = fmaxf(bmax, fmaxf(fabsf(v[2 * q]), fabsf(v[2 * q + 1])));
          }
        }
        uint16_t hv[16], lv[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const __half h = __float2half_rn(v[q]);
          const float hf = __half2float(h);
          hv[f16p_pos(q)] = __half_as_ushort(h);
          if (MODE == 1) {
            const __half l = __float2half_rn(__fsub_rn(v[q], hf));
            lv[f16p_pos(q)] = __half_as_ushort(l);
            sum = __fadd_rn(sum, __fadd_rn(hf, __half2float(l)));
          } else {
            sum = __fadd_rn(sum, hf);
          }
        }
        uint4* dh = reinterpret_cast<uint4*>(xh + 16 * b);
        dh[0] = make_uint4(hv[0] | ((uint32_t)hv[1] << 16), hv[2] | ((uint32_t)hv[3] << 16),
                           hv[4] | ((uint32_t)hv[5] << 16), hv[6] | ((uint32_t)hv[7] << 16));
        dh[1] = make_uint4(hv[8] | ((uint32_t)hv[9] << 16), hv[10] | ((uint32_t)hv[11] << 16),
                           hv[12] | ((uint32_t)hv[13] << 16), hv[14] | ((uint32_t)hv[15] << 16));
        if (MODE == 1) {
          uint4* dl = reinterpret_cast<uint4*>(xl + 16 * b);
          dl[0] = make_uint4(lv[0] | ((uint32_t)lv[1] << 16), lv[2] | ((uint32_t)lv[3] << 16),
                             lv[4] | ((uint32_t)lv[5] << 16), lv[6] | ((uint32_t)lv[7] << 16));
          dl[1] = make_uint4(lv[8] | ((uint32_t)lv[9] << 16), lv[10] | ((uint32_t)lv[11] << 16),
                             lv[12] | ((uint32_t)lv[13] << 16), lv[14] | ((uint32_t)lv[15] << 16));
        }
      }
      // four consecutive blocks make one 64-group
      sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
      sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
      bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));
      bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 2));
      if (b < nblk && (lane & 3) == 0) {
        xs[b >> 2] = sum;
        // bf16 x is staged as one fp16 value: exact only inside fp16's range
        if (MODE != 1 && !fp16_group_ok(bmax)) atomicExch(&g_decode_range, 1);
      }
    }
  }
}

}  // namespace

size_t gemv_stream_smem(int K, int ncol, bool lo) { return (size_t)GemvPlan(K, ncol, lo).total; }

template <int MODE>
__global__ void __launch_bounds__(kThreads, 5) gemv_stream_kernel(StreamParams P, int ncol) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int u = blockIdx.x;
  const bool shared = P.Wsh != nullptr && u == P.umax;
  // Dependencies.  The shared expert's gate_up reads only the layer input,
  // which the router kernel released before triggering this launch.  With
  // plan_ready the routing was complete when this kernel was released (the
  // previous kernel triggers only after its own wait), so the expert's rows
  // can be requested before waiting for the activations.  Everything else
  // waits first.  This kernel releases the next one only once it is past
  // that wait, so the next one may read the routing early in turn.
  const bool independent = MODE == 0 && shared;
  const bool early_plan = MODE == 1 && P.plan_ready;
  if (independent) pdl_trigger();
  if (shared) {
    // the shared expert's rows do not depend on the routing: pull this slab
    // into L2 while the previous kernel finishes
    const int Ns = P.Nsh, rb = P.K_sh / 2;          // bytes per packed weight row
    const int s0 = blockIdx.y;
    if (MODE == 0 ? s0 * 16 < Ns / 2 : s0 * kSlabRows < Ns) {
      const uint8_t* base = reinterpret_cast<const uint8_t*>(P.Wsh);
      for (int i = tid; i < kSlabRows * (rb / 128); i += kThreads) {
        const int r = i / (rb / 128), c = i % (rb / 128);
        const int wr = MODE == 0 ? ((r < 16) ? s0 * 16 + r : Ns / 2 + s0 * 16 + r - 16)
                                 : s0 * kSlabRows + r;
        prefetch_l2(base + (size_t)wr * rb + c * 128);
      }
    }
  }
  if (!independent && !early_plan) {
    pdl_wait();
    pdl_trigger();
  }
  const int nuniq = independent ? 0 : P.nuniq[0];
  if (!shared && u >= nuniq) return;
  const int e = shared ? 0 : P.uexp[u];
  const int p0 = shared ? 0 : P.ustart[u];
  const int ncol_all = shared ? P.nsh : (P.ustart[u + 1] - p0);
  const int N = shared ? P.Nsh : P.N;
  const int K = shared ? P.K_sh : P.K;
  const int G = K / kGroup, KW = K / 8;
  const int slab = blockIdx.y;
  if (MODE == 0 ? slab * (kSlabRows / 2) >= N / 2 : slab * kSlabRows >= N) return;
  const GemvPlan L((P.Wsh && P.K_sh > P.K) ? P.K_sh : P.K, ncol, MODE == 1);
  const uint32_t* We = shared ? P.Wsh : P.W + (size_t)e * N * KW;
  const uint16_t* Se = shared ? P.Ssh : P.S + (size_t)e * N * G;
  const uint16_t* Be = shared ? P.Bsh : P.B + (size_t)e * N * G;

  // tile row r <-> weight row (mode 0: 16 gate rows, then the matching up rows)
  auto wrow_of = [&](int r) -> int {
    if (MODE == 0) return (r < 16) ? slab * 16 + r : N / 2 + slab * 16 + (r - 16);
    return slab * kSlabRows + r;
  };
  // this warp's K quarter
  const int g0 = (warp * G) / kWarps, g1 = ((warp + 1) * G) / kWarps, ng = g1 - g0;
  uint8_t* wsm = sm + warp * L.warp_bytes;

  // ---- copies, in the order they are needed: the first pass's activation
  // columns (one commit group), then the weight rows of the first half of the
  // quarter's groups and of the second half (two groups).  With early_plan the
  // weights go first and the columns follow the wait.
  const int ncol_first = min(ncol, ncol_all);
  const int nh = (ng + 1) / 2;                   // groups in the first weight half
  auto issue_weights = [&]() {
    for (int part = 0; part < 2; ++part) {
      // all lanes busy: (row, chunk) of copy i = lane + 32 j, stepped without division
      const int j0 = part ? nh : 0;
      const int chunks = ((part ? ng : nh) - j0) * 2;   // 16-byte chunks per row slice
      if (chunks > 0) {
        const int dr = 32 / chunks, dc = 32 % chunks;
        int r = lane / chunks, c = lane % chunks;
        for (; r < kSlabRows;) {
          cp_async16(wsm + L.w_off + r * L.wstride + j0 * 32 + c * 16,
                     We + (size_t)wrow_of(r) * KW + (g0 + j0) * 8 + c * 4);
          r += dr;
          c += dc;
          if (c >= chunks) {
            c -= chunks;
            ++r;
          }
        }
      }
      cp_async_commit();
    }
  };
  if (!early_plan) {
    issue_columns<MODE>(P, L, wsm, shared, p0, 0, ncol_first, g0 * kGroup, ng * kGroup, lane);
    cp_async_commit();
  }
  issue_weights();
  // ---- scales of row `lane`: loads issued now, converted after the first
  // activation columns are staged so both latencies overlap
  const size_t ro = (size_t)wrow_of(lane) * G + g0;
  uint32_t sbraw[kMaxGw];                       // (scale, bias) bf16 pairs
#pragma unroll
  for (int j = 0; j < kMaxGw; ++j)
    if (j < ng) sbraw[j] = (uint32_t)Se[ro + j] | ((uint32_t)Be[ro + j] << 16);
  auto store_scales = [&]() {
    float2* sb = reinterpret_cast<float2*>(wsm + L.sb_off);
#pragma unroll
    for (int j = 0; j < kMaxGw; ++j)
      if (j < ng) {
        const float sv = bf2f((uint16_t)(sbraw[j] & 0xffffu));
        sb[j * kSlabRows + lane] =
            make_float2(sv, __fadd_rn(bf2f((uint16_t)(sbraw[j] >> 16)), __fmul_rn(8.0f, sv)));
      }
    for (int j = kMaxGw; j < ng; ++j) {          // K beyond 64 * 4 * kMaxGw
      const float sv = bf2f(Se[ro + j]);
      sb[j * kSlabRows + lane] = make_float2(sv, __fadd_rn(bf2f(Be[ro + j]), __fmul_rn(8.0f, sv)));
    }
  };

  if (early_plan) {
    pdl_wait();                                  // the activations are ready now
    pdl_trigger();
    issue_columns<MODE>(P, L, wsm, shared, p0, 0, ncol_first, g0 * kGroup, ng * kGroup, lane);
    cp_async_commit();
  }

  const uint8_t* w0p = wsm + L.w_off + g * L.wstride + t * 8;
  const float2* sbp = reinterpret_cast<const float2*>(wsm + L.sb_off);
  const uint8_t* xhp = wsm + L.xh_off;
  const uint8_t* xlp = wsm + L.xl_off;
  const float* xsp = reinterpret_cast<const float*>(wsm + L.xs_off);
  float4* red = reinterpret_cast<float4*>(sm + L.red_off);

  for (int cb = 0; cb < ncol_all; cb += ncol) {
    const int nc = min(ncol, ncol_all - cb);
    if (cb > 0) {
      __syncthreads();                           // the previous pass's reduction is done
      issue_columns<MODE>(P, L, wsm, shared, p0, cb, nc, g0 * kGroup, ng * kGroup, lane);
      cp_async_commit();
      cp_async_wait<0>();
    } else if (early_plan) {
      cp_async_wait<0>();                        // weights and activation columns
    } else {
      cp_async_wait<2>();                        // the activation columns
    }
    __syncwarp();
    convert_columns<MODE>(L, wsm, nc, ng * kGroup, lane);
    if (cb == 0) store_scales();

    float acc[2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[m][q] = 0.0f;
    const int bcol = min(g, nc - 1);             // the B column this thread loads
    const int c0 = min(2 * t, nc - 1), c1 = min(2 * t + 1, nc - 1);
    auto group = [&](int j) {
      uint2 wv[4];
#pragma unroll
      for (int m = 0; m < 4; ++m)                // rows g, g+8, 16+g, 24+g
        wv[m] = *reinterpret_cast<const uint2*>(w0p + (8 * m) * L.wstride + j * 32);
      const uint4* bh = reinterpret_cast<const uint4*>(xhp + bcol * L.cstride + j * 128 + t * 32);
      const uint4 h0 = bh[0], h1 = bh[1];
      uint4 l0, l1;
      if (MODE == 1) {
        const uint4* bl = reinterpret_cast<const uint4*>(xlp + bcol * L.cstride + j * 128 + t * 32);
        l0 = bl[0];
        l1 = bl[1];
      }
      float d[2][4];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
#pragma unroll
        for (int q = 0; q < 4; ++q) d[m][q] = 0.0f;
        const uint2 wl = wv[2 * m], wh = wv[2 * m + 1];
        uint32_t qL[8], qH[8];                  // pairs of the row-g and row-g+8 words
        qpairs4(wl.x, qL);
        qpairs4(wl.y, qL + 4);
        qpairs4(wh.x, qH);
        qpairs4(wh.y, qH + 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int pi = (kk >> 1) * 4 + (kk & 1) * 2;
          const uint32_t a0 = qL[pi], a1 = qH[pi], a2 = qL[pi + 1], a3 = qH[pi + 1];
          const uint4 hb = (kk < 2) ? h0 : h1;
          const uint32_t b0 = (kk & 1) ? hb.z : hb.x, b1 = (kk & 1) ? hb.w : hb.y;
          mma16816(d[m], a0, a1, a2, a3, b0, b1);
          if (MODE == 1) {
            const uint4 lb = (kk < 2) ? l0 : l1;
            mma16816(d[m], a0, a1, a2, a3, (kk & 1) ? lb.z : lb.x, (kk & 1) ? lb.w : lb.y);
          }
        }
      }
      const float xs0 = xsp[c0 * L.gw + j], xs1 = xsp[c1 * L.gw + j];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const float2 lo = sbp[j * kSlabRows + 16 * m + g];
        const float2 hi = sbp[j * kSlabRows + 16 * m + g + 8];
        acc[m][0] = __fmaf_rn(lo.x, d[m][0], __fmaf_rn(lo.y, xs0, acc[m][0]));
        acc[m][1] = __fmaf_rn(lo.x, d[m][1], __fmaf_rn(lo.y, xs1, acc[m][1]));
        acc[m][2] = __fmaf_rn(hi.x, d[m][2], __fmaf_rn(hi.y, xs0, acc[m][2]));
        acc[m][3] = __fmaf_rn(hi.x, d[m][3], __fmaf_rn(hi.y, xs1, acc[m][3]));
      }
    };
    if (cb == 0 && !early_plan) cp_async_wait<1>();   // the first weight half
    __syncwarp();
#pragma unroll 1
    for (int j = 0; j < nh; ++j) group(j);
    if (cb == 0 && !early_plan) cp_async_wait<0>();   // the second half
    __syncwarp();
#pragma unroll 1
    for (int j = nh; j < ng; ++j) group(j);
    // ---- 4-way reduction over the K quarters, fixed order
#pragma unroll
    for (int m = 0; m < 2; ++m)
      red[(warp * 2 + m) * 32 + lane] = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
    __syncthreads();
    {
      const int ln = tid >> 2, q = tid & 3;      // fragment (lane ln, element q)
      const float* rf = reinterpret_cast<const float*>(red);
      float v[2];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        float a = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) a = __fadd_rn(a, rf[((w * 2 + m) * 32 + ln) * 4 + q]);
        v[m] = a;
      }
      const int rr = (ln >> 2) + 8 * (q >> 1);   // row within an m16 tile
      const int c = cb + 2 * (ln & 3) + (q & 1);
      if (c < ncol_all) {
        const int orow = shared ? c : P.order[p0 + c];
        if (MODE == 0) {
          float* out = shared ? P.out_sh : P.out;
          out[(size_t)orow * (N / 2) + slab * 16 + rr] = silu_mul_f32(v[0], v[1]);
        } else if (MODE == 1) {
          float* out = shared ? P.out_sh : P.out;
          out[(size_t)orow * N + slab * kSlabRows + rr] = v[0];
          out[(size_t)orow * N + slab * kSlabRows + 16 + rr] = v[1];
        } else {
          P.outb[(size_t)orow * N + slab * kSlabRows + rr] = f2bf(v[0]);
          P.outb[(size_t)orow * N + slab * kSlabRows + 16 + rr] = f2bf(v[1]);
        }
      }
    }
  }

  if (MODE == 1) {
    // The last CTA to finish this output slab folds the partials: ordered
    // weighted sum over the k slots plus the gated shared expert.  Nobody
    // waits: every CTA counts itself in and only the last one does the sum.
    __shared__ int last;
    __syncthreads();
    if (tid == 0) {
      const int contributors = nuniq + (P.Wsh ? 1 : 0);
      last = (ticket_acq_rel(&P.counters[slab]) == contributors - 1);
    }
    __syncthreads();
    if (!last) return;
    const int D = P.N;
    for (int i = tid; i < P.T * kSlabRows; i += kThreads) {
      const int tt = i / kSlabRows, d = slab * kSlabRows + (i % kSlabRows);
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

int gemv_slab_rows() { return kSlabRows; }

cudaError_t launch_gemv_stream(int mode, const StreamParams& P, int max_cols, cudaStream_t s) {
  const int nb_x = P.umax + (P.Wsh ? 1 : 0);
  const int nmax = (P.Wsh && P.Nsh > P.N) ? P.Nsh : P.N;
  const int kmax = (P.Wsh && P.K_sh > P.K) ? P.K_sh : P.K;
  const int nb_y = (mode == 0) ? (nmax / 2 + 15) / 16 : (nmax + kSlabRows - 1) / kSlabRows;
  if (nb_x <= 0 || nb_y <= 0 || max_cols <= 0) return cudaSuccess;
  // columns staged per pass: two keep the plan at 3-6 CTAs per SM; an expert
  // with more columns makes more passes over the rows already in shared memory
  const int ncol = max_cols < kColsPerPass ? max_cols : kColsPerPass;
  const int smem = GemvPlan(kmax, ncol, mode == 1).total;
  dim3 grid(nb_x, nb_y);
  cudaError_t err = cudaSuccess;
  auto go = [&](auto kernel) {
    cudaError_t e = ensure_smem_attr((const void*)kernel, smem);
    return e != cudaSuccess ? e : launch_pdl(kernel, grid, dim3(kThreads), (size_t)smem, s, P, ncol);
  };
  if (mode == 0) err = go(gemv_stream_kernel<0>);
  else if (mode == 1) err = go(gemv_stream_kernel<1>);
  else err = go(gemv_stream_kernel<2>);
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
