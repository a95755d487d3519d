// Weight preparation.
//
//  * affine_quantize: MLX's mx.quantize(w, group_size=64, bits=4,
//    mode="affine") (third-party; call sites switch_layers.py:42,179) on the
//    GPU, one thread per group: zero is exactly representable (edge / q0
//    rescale), codes packed 8 per uint32, low nibble first, scales and biases
//    rounded to bf16.
//  * prepare_tables: the transposed [E, G, N] scale and bias tables the
//    grouped GEMM streams with its weight tiles (the layout argument of
//    moe_gather_int8.py:205-224: one contiguous run per group and column
//    tile).  The int8 kernel folds b + 8s itself, exactly as build_tables'
//    bf16 table holds it, so only the raw biases are stored.
//  * qsum: the reference's per (expert, group, row) nibble sums
//    (moe_gather_int8.py:189-202), provided for callers of the reference's
//    Int8Tables interface; the B200 kernels re-centre the nibbles in
//    registers and never read it.
#include "common.cuh"
#include "tmoe_internal.h"

namespace tmoe {

__global__ void __launch_bounds__(256) affine_quantize_kernel(const float* __restrict__ w,
                                                              long long ngroups,
                                                              uint32_t* __restrict__ wq,
                                                              uint16_t* __restrict__ scales,
                                                              uint16_t* __restrict__ biases) {
  const long long gi = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gi >= ngroups) return;
  const float4* v4 = reinterpret_cast<const float4*>(w + gi * 64);
  float v[64];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float4 f = v4[i];
    v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
  }
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int i = 1; i < 64; ++i) {
    mn = fminf(mn, v[i]);
    mx = fmaxf(mx, v[i]);
  }
  const bool mask = fabsf(mn) > fabsf(mx);
  float scale = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), 15.0f), 1e-7f);
  scale = mask ? scale : -scale;
  const float edge = mask ? mn : mx;
  const float q0 = rintf(__fdiv_rn(edge, scale));
  float bias = 0.0f;
  if (q0 != 0.0f) {
    scale = __fdiv_rn(edge, q0);
    bias = edge;
  }
  uint32_t* out = wq + gi * 8;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint32_t word = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      float q = rintf(__fdiv_rn(__fsub_rn(v[j * 8 + t], bias), scale));
      q = fminf(fmaxf(q, 0.0f), 15.0f);
      word |= ((uint32_t)q) << (4 * t);
    }
    out[j] = word;
  }
  scales[gi] = f2bf(scale);
  biases[gi] = f2bf(bias);
}

cudaError_t launch_affine_quantize(const float* w, long long rows, int K, uint32_t* wq,
                                   uint16_t* scales, uint16_t* biases, cudaStream_t s) {
  const long long ng = rows * (K / kGroup);
  if (ng > 0)
    affine_quantize_kernel<<<(unsigned)((ng + 255) / 256), 256, 0, s>>>(w, ng, wq, scales, biases);
  return cudaGetLastError();
}

// [E, N, G] -> [E, G, N] for two bf16 tables at once, 32x32 smem tiles.
__global__ void transpose_tables_kernel(const uint16_t* __restrict__ s, const uint16_t* __restrict__ b,
                                        int N, int G, uint16_t* __restrict__ st,
                                        uint16_t* __restrict__ bt) {
  __shared__ uint16_t ts[32][33], tb[32][33];
  const int e = blockIdx.z;
  const int n0 = blockIdx.x * 32, g0 = blockIdx.y * 32;
  const size_t base = (size_t)e * N * G;
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int n = n0 + r, g = g0 + threadIdx.x;
    if (n < N && g < G) {
      ts[r][threadIdx.x] = s[base + (size_t)n * G + g];
      tb[r][threadIdx.x] = b[base + (size_t)n * G + g];
    }
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int g = g0 + r, n = n0 + threadIdx.x;
    if (n < N && g < G) {
      st[base + (size_t)g * N + n] = ts[threadIdx.x][r];
      bt[base + (size_t)g * N + n] = tb[threadIdx.x][r];
    }
  }
}

cudaError_t launch_prepare_tables(const uint16_t* scales, const uint16_t* biases, int E, int N, int G,
                                  uint16_t* st, uint16_t* bt, cudaStream_t s) {
  dim3 grid((N + 31) / 32, (G + 31) / 32, E);
  if (E > 0 && N > 0 && G > 0) transpose_tables_kernel<<<grid, dim3(32, 8), 0, s>>>(scales, biases, N, G, st, bt);
  return cudaGetLastError();
}

__global__ void qsum_kernel(const uint32_t* __restrict__ w, int E, int N, int G,
                            uint16_t* __restrict__ qsum) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // (e*N + n)*G + g
  if (i >= (long long)E * N * G) return;
  const uint4* p = reinterpret_cast<const uint4*>(w + i * 8);
  const uint4 a = p[0], b = p[1];
  const uint32_t words[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t acc = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int t = 0; t < 8; ++t) acc += (words[j] >> (4 * t)) & 0xfu;
  const int g = (int)(i % G), n = (int)((i / G) % N), e = (int)(i / ((long long)G * N));
  qsum[((size_t)e * G + g) * N + n] = (uint16_t)acc;
}

cudaError_t launch_qsum(const uint32_t* w, int E, int N, int K, uint16_t* qsum, cudaStream_t s) {
  const long long n = (long long)E * N * (K / kGroup);
  if (n > 0) qsum_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(w, E, N, K / kGroup, qsum);
  return cudaGetLastError();
}

// Tile table for a dense (single-expert) GEMM over R rows: tiles of tile_m
// rows of expert 0.  Written on the device so the whole forward needs no
// host copy.
__global__ void dense_tiles_kernel(int R, int tile_m, int32_t* tile_row, int32_t* tile_exp,
                                   int32_t* ntiles, int32_t* offsets) {
  const int nt = (R + tile_m - 1) / tile_m;
  for (int i = threadIdx.x; i < nt; i += blockDim.x) {
    tile_row[i] = i * tile_m;
    tile_exp[i] = 0;
  }
  if (threadIdx.x == 0) {
    ntiles[0] = nt;
    offsets[0] = 0;
    offsets[1] = R;
  }
}

cudaError_t launch_dense_tiles(int R, int tile_m, int32_t* tile_row, int32_t* tile_exp,
                               int32_t* ntiles, int32_t* offsets, cudaStream_t s) {
  dense_tiles_kernel<<<1, 256, 0, s>>>(R, tile_m, tile_row, tile_exp, ntiles, offsets);
  return cudaGetLastError();
}

}  // namespace tmoe
