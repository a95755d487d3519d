// Router: logits = bf16(x @ Wr^T) (canonical 8-partial order), softmax in
// fp32 -> bf16 probabilities, top-k with the lowest index winning ties, and
// bf16 renormalised scores.  Follows qwen3_5_moe/language.py:65-71 and the
// fused router of engine/patches/decode-fusion/fused_kernels.py:234-327.
//
// Two logits kernels compute bit-identical results:
//   * router_logits_gemv  — decode shapes: 4 experts per warp (8 lanes = the
//     8 canonical partials each), every weight row streamed once from HBM;
//   * router_logits_tiled — prefill shapes: a 64-token x 32-expert CTA tile,
//     x and W staged through a 4-stage cp.async ring in shared memory, 64
//     accumulators per thread (4 tokens x 8 experts, packed in expert pairs
//     for f32x2 FMAs) for one canonical partial, 512 threads.
// The optional shared-expert gate row wg is evaluated as expert row E; its
// fp32 logit goes to gate_logit[T].
#include "common.cuh"
#include "tmoe_internal.h"

namespace tmoe {

TMOE_DEV float tree8_sum(float v) {
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return v;
}

// One warp = 4 expert rows (8 lanes each, one per canonical partial) x one
// chunk of up to 8 tokens (blockIdx.y).  The warp first copies its 4 weight
// rows and its token rows into shared memory with cp.async (every byte in
// flight at once), then reduces.
constexpr int kGemvTok = 8;

__global__ void __launch_bounds__(32) router_logits_gemv(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr,
    const uint16_t* __restrict__ wg, int T, int H, int E, uint16_t* __restrict__ logits,
    float* __restrict__ gate_logit) {
  extern __shared__ __align__(16) uint8_t smem_r[];
  const int lane = threadIdx.x;
  const int p = lane & 7, sub = lane >> 3;
  const int e0 = blockIdx.x * 4;
  const int e = e0 + sub;
  const int nrows = E + (wg ? 1 : 0);
  const bool valid = e < nrows;
  const int nch = H >> 3;                     // 16-byte chunks per row
  uint4* ws = reinterpret_cast<uint4*>(smem_r);                 // [4][nch]
  uint4* xs = ws + 4 * nch;                                     // [8][nch]
  for (int i = lane; i < 4 * nch; i += 32) {
    const int r = i / nch, c = i % nch;
    const int er = e0 + r;
    const bool ok = er < nrows;
    const uint16_t* row = ok ? ((er < E) ? wr + (size_t)er * H : wg) : wr;
    cp_async16_zfill(&ws[i], row + (size_t)c * 8, ok);
  }
  // token chunks of kGemvTok are spread over blockIdx.y (and strided, should
  // the grid be smaller than T needs)
  for (int t0 = blockIdx.y * kGemvTok; t0 < T; t0 += gridDim.y * kGemvTok) {
    const int nt = min(kGemvTok, T - t0);
    __syncwarp();
    for (int i = lane; i < nt * nch; i += 32)
      cp_async16(&xs[i], x + (size_t)(t0 + i / nch) * H + (size_t)(i % nch) * 8);
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
    float acc[kGemvTok];
#pragma unroll
    for (int i = 0; i < kGemvTok; ++i) acc[i] = 0.0f;
    for (int c = p; c < nch; c += 8) {
      float wf[8];
      unpack8_bf16(ws[sub * nch + c], wf);
#pragma unroll
      for (int tt = 0; tt < kGemvTok; ++tt) {
        if (tt < nt) {
          float xf[8];
          unpack8_bf16(xs[tt * nch + c], xf);
#pragma unroll
          for (int u = 0; u < 8; ++u) acc[tt] = __fmaf_rn(xf[u], wf[u], acc[tt]);
        }
      }
    }
#pragma unroll
    for (int tt = 0; tt < kGemvTok; ++tt) {
      const float s = tree8_sum(acc[tt]);
      if (valid && p == tt && tt < nt) {
        if (e < E)
          logits[(size_t)(t0 + tt) * E + e] = f2bf(s);
        else
          gate_logit[t0 + tt] = s;
      }
    }
  }
}

// CTA tile: 64 tokens x 32 experts, K step 64 elements (8 chunks), 512
// threads.  Thread roles: p = lane & 7 is the canonical partial (chunk p of
// each step), gid = warp*4 + (lane>>3) in [0,64): gt = gid & 15 selects tokens
// tt*16 + gt (tt < 4), ge = gid >> 4 selects experts ee*4 + ge
// (conflict-free smem).
__global__ void __launch_bounds__(512) router_logits_tiled(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr,
    const uint16_t* __restrict__ wg, int T, int H, int E, uint16_t* __restrict__ logits,
    float* __restrict__ gate_logit) {
  constexpr int NS = 4;              // cp.async stages: 3 K steps of loads in flight
  __shared__ uint4 xs[NS][64][8];
  __shared__ uint4 ws[NS][32][8];
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int p = lane & 7;
  const int gid = warp * 4 + (lane >> 3);      // [0, 64)
  const int gt = gid & 15, ge = gid >> 4;       // tokens tt*16 + gt, experts ee*4 + ge
  const int tok0 = blockIdx.x * 64, exp0 = blockIdx.y * 32;
  const int nrows = E + (wg ? 1 : 0);
  const int nk = H / 64;

  auto load_stage = [&](int stage, int ks) {
    for (int i = tid; i < 768; i += 512) {
      if (i < 512) {
        int r = i >> 3, ch = i & 7;
        int t = tok0 + r;
        bool ok = t < T;
        const uint16_t* src = x + (size_t)(ok ? t : 0) * H + ks * 64 + ch * 8;
        cp_async16_zfill(&xs[stage][r][ch], src, ok);
      } else {
        int j = i - 512;
        int r = j >> 3, ch = j & 7;
        int e = exp0 + r;
        bool ok = e < nrows;
        const uint16_t* rowp = ok ? ((e < E) ? wr + (size_t)e * H : wg) : wr;
        cp_async16_zfill(&ws[stage][r][ch], rowp + ks * 64 + ch * 8, ok);
      }
    }
    cp_async_commit();
  };

  // accumulators of expert pairs (ee = 2q, 2q + 1) as float2: packed f32x2
  // FMAs, each component in the scalar order (u ascending within a K step)
  float2 acc2[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc2[a][b] = make_float2(0.0f, 0.0f);

  for (int s = 0; s < NS - 1; ++s) {   // one commit group per stage, empty ones too
    if (s < nk)
      load_stage(s, s);
    else
      cp_async_commit();
  }
  for (int ks = 0; ks < nk; ++ks) {
    cp_async_wait<NS - 2>();             // this thread's copies of step ks landed
    __syncthreads();                     // ... every thread's; step ks - 1 is consumed
    const int kn = ks + NS - 1;          // refill the stage step ks - 1 used
    if (kn < nk)
      load_stage(kn % NS, kn);
    else
      cp_async_commit();
    const int st = ks % NS;
    float2 w2[4][8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float wa[8], wb[8];
      unpack8_bf16(ws[st][(2 * q) * 4 + ge][p], wa);
      unpack8_bf16(ws[st][(2 * q + 1) * 4 + ge][p], wb);
#pragma unroll
      for (int u = 0; u < 8; ++u) w2[q][u] = make_float2(wa[u], wb[u]);
    }
#pragma unroll
    for (int tt = 0; tt < 4; ++tt) {
      float xf[8];
      unpack8_bf16(xs[st][tt * 16 + gt][p], xf);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float2 x2 = make_float2(xf[u], xf[u]);
#pragma unroll
        for (int q = 0; q < 4; ++q) acc2[tt][q] = __ffma2_rn(x2, w2[q][u], acc2[tt][q]);
      }
    }
  }
  float acc[4][8];
#pragma unroll
  for (int tt = 0; tt < 4; ++tt)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc[tt][2 * q] = acc2[tt][q].x;
      acc[tt][2 * q + 1] = acc2[tt][q].y;
    }
#pragma unroll
  for (int tt = 0; tt < 4; ++tt)
#pragma unroll
    for (int ee = 0; ee < 8; ++ee) acc[tt][ee] = tree8_sum(acc[tt][ee]);
  // lane p < 4 stores token tt = p of its group.
#pragma unroll
  for (int tt = 0; tt < 4; ++tt) {
    if (tt != p) continue;
    int t = tok0 + tt * 16 + gt;
    if (t >= T) continue;
#pragma unroll
    for (int ee = 0; ee < 8; ++ee) {
      int e = exp0 + ee * 4 + ge;
      if (e < E)
        logits[(size_t)t * E + e] = f2bf(acc[tt][ee]);
      else if (e == E && wg)
        gate_logit[t] = acc[tt][ee];
    }
  }
}

// One warp per token: lane l holds experts e = 32c + l.
template <int PER>
__global__ void __launch_bounds__(128) router_topk_kernel(
    const uint16_t* __restrict__ logits, int T, int E, int k, int32_t* __restrict__ idx,
    uint16_t* __restrict__ scores, uint16_t* __restrict__ probs_out) {
  const int lane = threadIdx.x & 31;
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  float lv[PER];
  float m = -__int_as_float(0x7f800000);
#pragma unroll
  for (int c = 0; c < PER; ++c) {
    int e = 32 * c + lane;
    lv[c] = (e < E) ? bf2f(logits[(size_t)t * E + e]) : -__int_as_float(0x7f800000);
    m = fmaxf(m, lv[c]);
  }
  m = warp_max(m);
  float ex[PER];
  float part = 0.0f;
#pragma unroll
  for (int c = 0; c < PER; ++c) {
    int e = 32 * c + lane;
    if (e < E) {
      ex[c] = cexp(__fsub_rn(lv[c], m));
      part = __fadd_rn(part, ex[c]);
    } else {
      ex[c] = 0.0f;
    }
  }
  const float sum = warp_butterfly_sum(part);
  const float inv = __fdiv_rn(1.0f, sum);
  uint32_t pb[PER];
#pragma unroll
  for (int c = 0; c < PER; ++c) {
    pb[c] = f2bf(__fmul_rn(ex[c], inv));
    int e = 32 * c + lane;
    if (probs_out && e < E) probs_out[(size_t)t * E + e] = (uint16_t)pb[c];
  }
  uint32_t taken = 0;
  float ssum = 0.0f;
  uint32_t my_p = 0;
  int my_e = 0;
  for (int j = 0; j < k; ++j) {
    uint32_t best = 0;
#pragma unroll
    for (int c = 0; c < PER; ++c) {
      int e = 32 * c + lane;
      if (e < E && !((taken >> c) & 1u)) {
        uint32_t key = (pb[c] << 16) | (uint32_t)(0xffff - e);
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
    scores[(size_t)t * k + lane] = f2bf(__fdiv_rn(bf2f((uint16_t)my_p), sb));
  }
}

cudaError_t launch_router_logits(const uint16_t* x, const uint16_t* wr, const uint16_t* wg, int T,
                                 int H, int E, uint16_t* logits, float* gate_logit,
                                 cudaStream_t s) {
  const int nrows = E + (wg ? 1 : 0);
  if (T <= 32) {
    const size_t smem = (size_t)(4 + kGemvTok) * H * 2;
    cudaError_t e = ensure_smem_attr((const void*)router_logits_gemv, (int)smem);
    if (e != cudaSuccess) return e;
    router_logits_gemv<<<dim3((nrows + 3) / 4, (T + kGemvTok - 1) / kGemvTok), 32, smem, s>>>(
        x, wr, wg, T, H, E, logits, gate_logit);
  } else {
    dim3 grid((T + 63) / 64, (nrows + 31) / 32);
    router_logits_tiled<<<grid, 512, 0, s>>>(x, wr, wg, T, H, E, logits, gate_logit);
  }
  return cudaGetLastError();
}

cudaError_t launch_router_topk(const uint16_t* logits, int T, int E, int k, int32_t* idx,
                               uint16_t* scores, uint16_t* probs_out, cudaStream_t s) {
  const int blocks = (T + 3) / 4;
  const int per = (E + 31) / 32;
  if (per <= 2)
    router_topk_kernel<2><<<blocks, 128, 0, s>>>(logits, T, E, k, idx, scores, probs_out);
  else if (per <= 4)
    router_topk_kernel<4><<<blocks, 128, 0, s>>>(logits, T, E, k, idx, scores, probs_out);
  else if (per <= 8)
    router_topk_kernel<8><<<blocks, 128, 0, s>>>(logits, T, E, k, idx, scores, probs_out);
  else if (per <= 16)
    router_topk_kernel<16><<<blocks, 128, 0, s>>>(logits, T, E, k, idx, scores, probs_out);
  else
    router_topk_kernel<32><<<blocks, 128, 0, s>>>(logits, T, E, k, idx, scores, probs_out);
  return cudaGetLastError();
}

}  // namespace tmoe
