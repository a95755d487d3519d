// Shared device helpers for the titan_b200 MoE kernels (sm_100a).
//
// Canonical arithmetic: wherever the reference leaves an order or a rounding
// unspecified, these kernels evaluate one fixed sequence of IEEE binary32
// operations (explicit __fmaf_rn / __fadd_rn / __fmul_rn / __fdiv_rn, so the
// compiler cannot contract or reassociate them).  The sequences are:
//   * bf16 dot product (router Linear): 8 partials; the 8-element chunk c
//     (elements 8c..8c+7) feeds partial c mod 8 with fma in ascending order,
//     then the xor tree over offsets 4,2,1 (8 lanes of a warp, __shfl_xor);
//   * softmax denominator: 32 lane partials over e = 32c + l, xor butterfly
//     over offsets 16,8,4,2,1;
//   * exp: Cody-Waite reduction + degree-7 Taylor polynomial, 2^n applied in
//     two exact steps;
//   * group sum of the activation quantiser: pair sums, then the butterfly.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define TMOE_DEV __device__ __forceinline__
#define TMOE_HD __host__ __device__ __forceinline__

namespace tmoe {

constexpr int kGroup = 64;   // affine quantisation group (MLX group_size=64)

TMOE_DEV float bf2f(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

TMOE_DEV uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

TMOE_DEV float bfround(float f) { return bf2f(f2bf(f)); }

// A group of activations whose largest magnitude is gmax is exact as fp16
// values: below fp16's overflow and not wholly below its normal range.
TMOE_DEV bool fp16_group_ok(float gmax) {
  return gmax < 65504.0f && !(gmax > 0.0f && gmax < 6.103515625e-05f);
}

// e^x, the canonical sequence (see file header).
TMOE_DEV float cexp(float x) {
  if (x != x) return x;
  if (x > 88.7228393554688f) return __int_as_float(0x7f800000);
  if (x < -103.972084045410f) return 0.0f;
  float n = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(-n, 0.693145751953125f, x);
  r = __fmaf_rn(-n, 1.42860682030941723e-06f, r);
  float p = 1.98412698412698413e-4f;
  p = __fmaf_rn(p, r, 1.38888888888888889e-3f);
  p = __fmaf_rn(p, r, 8.33333333333333333e-3f);
  p = __fmaf_rn(p, r, 4.16666666666666667e-2f);
  p = __fmaf_rn(p, r, 1.66666666666666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int ni = (int)n;
  int n1 = ni / 2;
  int n2 = ni - n1;
  float s1 = __int_as_float((n1 + 127) << 23);
  float s2 = __int_as_float((n2 + 127) << 23);
  return __fmul_rn(__fmul_rn(p, s1), s2);
}

TMOE_DEV float csigmoid(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, cexp(-x)));
}

// SwiGLU with the reference's bf16 rounding after each op:
// sg = bf16(sigmoid(g)); a = bf16(g*sg); h = bf16(a*u).
TMOE_DEV float swiglu_bf16(float g, float u) {
  float sg = bfround(csigmoid(g));
  float a = bfround(__fmul_rn(g, sg));
  return bfround(__fmul_rn(a, u));
}

// Packed f32x2 arithmetic, checked on the B200 with nvcc 12.9: a
// __fmul2_rn whose result feeds a __fadd2_rn is contracted into one fused
// multiply-add (the scalar __fmul_rn never is).  Every packed product in this
// library therefore feeds a rounding (bfround2) or an FMA multiplicand; a
// product that must be rounded before an add is computed with __fmul_rn.
//
// Two lanes of cexp at once, bit-identical per component: rint(x * log2e)
// as (t + 1.5*2^23) - 1.5*2^23 (exact round-to-nearest-even for |t| < 2^22),
// the integer n read from the same sum's bits, the reduction and polynomial
// as packed f32x2 FMAs, the special cases selected afterwards.
TMOE_DEV float2 cexp2(float2 x) {
  // the product stays scalar: __fmul_rn is never fused into the add below,
  // so rint sees the rounded product exactly as cexp does
  const float2 t = make_float2(__fmul_rn(x.x, 1.44269504088896341f),
                               __fmul_rn(x.y, 1.44269504088896341f));
  const float2 big = __fadd2_rn(t, make_float2(12582912.0f, 12582912.0f));
  const float2 n = __fadd2_rn(big, make_float2(-12582912.0f, -12582912.0f));
  const float2 mn = make_float2(-n.x, -n.y);
  float2 r = __ffma2_rn(mn, make_float2(0.693145751953125f, 0.693145751953125f), x);
  r = __ffma2_rn(mn, make_float2(1.42860682030941723e-06f, 1.42860682030941723e-06f), r);
  auto k2 = [](float c) { return make_float2(c, c); };
  float2 p = k2(1.98412698412698413e-4f);
  p = __ffma2_rn(p, r, k2(1.38888888888888889e-3f));
  p = __ffma2_rn(p, r, k2(8.33333333333333333e-3f));
  p = __ffma2_rn(p, r, k2(4.16666666666666667e-2f));
  p = __ffma2_rn(p, r, k2(1.66666666666666667e-1f));
  p = __ffma2_rn(p, r, k2(0.5f));
  p = __ffma2_rn(p, r, k2(1.0f));
  p = __ffma2_rn(p, r, k2(1.0f));
  const int nx = (int)n.x, ny = (int)n.y;
  const int n1x = nx / 2, n1y = ny / 2;
  auto p2 = [](int k) { return __uint_as_float((uint32_t)(k + 127) << 23); };   // 2^k
  // the 2^n scaling stays scalar (two multiplies per lane)
  const float2 v = make_float2(__fmul_rn(__fmul_rn(p.x, p2(n1x)), p2(nx - n1x)),
                               __fmul_rn(__fmul_rn(p.y, p2(n1y)), p2(ny - n1y)));
  auto fix = [](float xi, float vi) {
    if (xi != xi) return xi;
    if (xi > 88.7228393554688f) return __int_as_float(0x7f800000);
    if (xi < -103.972084045410f) return 0.0f;
    return vi;
  };
  return make_float2(fix(x.x, v.x), fix(x.y, v.y));
}

// Two bf16 roundings in one conversion (round to nearest even, as f2bf).
TMOE_DEV float2 bfround2(float2 v) {
  const __nv_bfloat162 b = __float22bfloat162_rn(v);
  const uint32_t u = *reinterpret_cast<const uint32_t*>(&b);
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

// swiglu_bf16 on two lanes, bit-identical per component: the reciprocal is
// the correctly rounded 1 / y, as __fdiv_rn(1, y) is.
TMOE_DEV float2 swiglu_bf16x2(float2 g, float2 u) {
  const float2 e = cexp2(make_float2(-g.x, -g.y));
  const float2 y = __fadd2_rn(make_float2(1.0f, 1.0f), e);
  const float2 sg = bfround2(make_float2(__frcp_rn(y.x), __frcp_rn(y.y)));
  const float2 a = bfround2(__fmul2_rn(g, sg));
  return bfround2(__fmul2_rn(a, u));
}

// fp32 SiLU(g)*u of the decode path (decode-fusion semantics).
TMOE_DEV float silu_mul_f32(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, cexp(-g))), u);
}

TMOE_DEV float warp_butterfly_sum(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

TMOE_DEV float warp_max(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// The canonical 32-way butterfly evaluated by one thread over 32 values held
// in memory (lane l's value at p[l*stride]); same tree as warp_butterfly_sum.
TMOE_DEV float serial_butterfly32(const float* p, int stride) {
  float a[16];
#pragma unroll
  for (int l = 0; l < 16; ++l) a[l] = __fadd_rn(p[l * stride], p[(l + 16) * stride]);
#pragma unroll
  for (int l = 0; l < 8; ++l) a[l] = __fadd_rn(a[l], a[l + 8]);
#pragma unroll
  for (int l = 0; l < 4; ++l) a[l] = __fadd_rn(a[l], a[l + 4]);
#pragma unroll
  for (int l = 0; l < 2; ++l) a[l] = __fadd_rn(a[l], a[l + 2]);
  return __fadd_rn(a[0], a[1]);
}

// 8 packed bf16 (one 16-byte load) -> float.
TMOE_DEV void unpack8_bf16(uint4 v, float* f) {
  f[0] = __uint_as_float(v.x << 16); f[1] = __uint_as_float(v.x & 0xffff0000u);
  f[2] = __uint_as_float(v.y << 16); f[3] = __uint_as_float(v.y & 0xffff0000u);
  f[4] = __uint_as_float(v.z << 16); f[5] = __uint_as_float(v.z & 0xffff0000u);
  f[6] = __uint_as_float(v.w << 16); f[7] = __uint_as_float(v.w & 0xffff0000u);
}

TMOE_DEV uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

TMOE_DEV void cp_async16(void* smem, const void* gmem) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}
// Same copy, asking L2 to fetch the whole 256-byte span around the source:
// for rows read 16-32 bytes at a time in ascending order (packed weights one
// 64-group per step), the following steps then hit L2 instead of DRAM.
TMOE_DEV void cp_async16_l2pf(void* smem, const void* gmem) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}
TMOE_DEV void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  int src_bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
TMOE_DEV void cp_async8(void* smem, const void* gmem) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gmem));
}
TMOE_DEV void cp_async4(void* smem, const void* gmem) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem));
}
// Programmatic dependent launch.  pdl_trigger() lets the next kernel on the
// stream start launching; pdl_wait() blocks until the previous kernel has
// completed and its memory is visible.  A kernel launched with launch_pdl()
// must call pdl_wait() before it reads anything a predecessor wrote and
// before it writes anything a predecessor may still read.  Both are no-ops
// for a kernel launched without the attribute.
TMOE_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
TMOE_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
TMOE_DEV void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Ticket for "the last CTA to arrive does the rest": called by one thread
// after a CTA barrier, it publishes the CTA's prior writes (release, made
// cumulative by the barrier) and, for the last arrival, makes every other
// CTA's published writes visible (acquire).  Returns the previous count.
TMOE_DEV int ticket_acq_rel(int* counter) {
  int prev;
  asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(prev) : "l"(counter) : "memory");
  return prev;
}

TMOE_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
TMOE_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

}  // namespace tmoe
