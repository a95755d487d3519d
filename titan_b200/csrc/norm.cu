// The steps either side of the MoE block in a decoder layer:
//   the post-attention RMSNorm feeding the router and the experts
//   (titan/adapters/mlx/vendor/mlx_vlm/models/qwen3_5_moe/language.py:103-107,
//   137: out = h + mlp(post_attention_layernorm(h))), and
//   the write-back of the block's output: the plain residual add, or the
//   hyper-connection inject into an n-wide residual stream
//   (qwen4_exp/language.py:3198-3218: hyper + flatten(branch[..., None, :] *
//   weights[..., None])).
// Canonical arithmetic (restated by the CPU oracle):
//   RMSNorm: one warp per row; lane l sums x[e]^2 for e = l, l + 32, ... in
//   ascending order with fma, the xor butterfly 16..1 adds the lanes;
//   ms = sum / H; r = 1 / sqrt(ms + eps) (IEEE sqrt and divide);
//   out = bf16((x * r) * w).
//   Inject: y_j = bf16(bf16(branch * w_j) + hyper_j) per stream j; the plain
//   residual is one stream of weight 1: y = bf16(branch + residual).
#include "common.cuh"
#include "tmoe_internal.h"

namespace tmoe {

__global__ void __launch_bounds__(256) rmsnorm_kernel(const uint16_t* __restrict__ x,
                                                      const uint16_t* __restrict__ w, int T, int H,
                                                      float eps, uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= T) return;
  const uint16_t* xr = x + (size_t)row * H;
  float s = 0.0f;
  for (int e = lane; e < H; e += 32) {
    const float v = bf2f(xr[e]);
    s = __fmaf_rn(v, v, s);
  }
  s = warp_butterfly_sum(s);
  const float ms = __fdiv_rn(s, (float)H);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
  uint16_t* o = out + (size_t)row * H;
  for (int e = lane; e < H; e += 32)
    o[e] = f2bf(__fmul_rn(__fmul_rn(bf2f(xr[e]), r), bf2f(w[e])));
}

// out [T][n][H] (n = 0: the plain residual, out [T][H]).
__global__ void __launch_bounds__(256) inject_kernel(const uint16_t* __restrict__ branch,
                                                     const uint16_t* __restrict__ hyper,
                                                     const uint16_t* __restrict__ wts, int T, int H,
                                                     int n, uint16_t* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int ns = n > 0 ? n : 1;
  const long long total = (long long)T * ns * H;
  if (i >= total) return;
  const int c = (int)(i % H);
  const long long tj = i / H;
  const long long t = tj / ns;
  const int j = (int)(tj - t * ns);
  const float b = bf2f(branch[t * H + c]);
  const float p = n > 0 ? bfround(__fmul_rn(b, bf2f(wts[t * n + j]))) : b;
  out[i] = f2bf(__fadd_rn(p, bf2f(hyper[i])));
}

cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* w, int T, int H, float eps,
                           uint16_t* out, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  rmsnorm_kernel<<<(unsigned)(((long long)T * 32 + 255) / 256), 256, 0, s>>>(x, w, T, H, eps, out);
  return cudaGetLastError();
}

cudaError_t launch_inject(const uint16_t* branch, const uint16_t* hyper, const uint16_t* wts, int T,
                          int H, int n, uint16_t* out, cudaStream_t s) {
  const long long total = (long long)T * (n > 0 ? n : 1) * H;
  if (total <= 0) return cudaSuccess;
  inject_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(branch, hyper, wts, T, H, n, out);
  return cudaGetLastError();
}

}  // namespace tmoe
