// tcgen05 / mbarrier / TMA building blocks shared by the tensor-core kernels
// (sm_100a).  Inline PTX only; every wait is bounded by the caller's limit.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace tmoe {
namespace tc {

constexpr uint32_t kSpinLimit = 1u << 22;   // bound of every mbarrier wait (polls)
constexpr uint32_t kFastPolls = 1u << 12;   // polls before backing off

TMOE_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

TMOE_DEV void mbar_init(uint32_t a, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count));
}
TMOE_DEV void mbar_arrive(uint32_t a) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(a) : "memory");
}
TMOE_DEV void mbar_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes)
               : "memory");
}
TMOE_DEV bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; false on timeout (the abort flag raised, *err set) or abort.
TMOE_DEV bool mbar_wait(uint32_t a, uint32_t parity, volatile int* abort_flag, int* err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try(a, parity)) return true;
    if (*abort_flag) return false;
    if (i >= kFastPolls) __nanosleep(64);
  }
  *abort_flag = 1;
  atomicExch(err, 1);
  return false;
}

// SW128 K-major shared-memory matrix descriptor (rows of 128 B, 8-row atoms
// 1024 B apart), sm_100 descriptor version.
TMOE_DEV uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)64 << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: f16 x f16 -> f32, both K-major.
TMOE_HD uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

TMOE_DEV void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                      uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
TMOE_DEV void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
TMOE_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
TMOE_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

TMOE_DEV void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
TMOE_DEV void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
TMOE_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 8 nibbles (elements 0..7 of a chunk) -> 4 half2 in the pair order
// (0,4),(1,5),(2,6),(3,7): the fp16 operand layout of every A and B chunk.
// 0x6400|q is 1024 + q; pairs 1 and 3 are taken 4 bits up (1024 + 16q) and
// re-centred by one HFMA2 (x/16 - 72); every step is exact.  With `scale`
// each value is then multiplied by s2 (exact when (q-8)*s fits fp16).
TMOE_DEV uint4 widen8(uint32_t w, bool scale, __half2 s2) {
  const __half2 off = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
  const __half2 sixteenth = __halves2half2(__ushort_as_half(0x2c00), __ushort_as_half(0x2c00));
  const __half2 m72 = __halves2half2(__ushort_as_half(0xd480), __ushort_as_half(0xd480));
  const uint32_t w8 = w >> 8;
  uint32_t v[4] = {(w & 0x000f000fu) | 0x64006400u, (w & 0x00f000f0u) | 0x64006400u,
                   (w8 & 0x000f000fu) | 0x64006400u, (w8 & 0x00f000f0u) | 0x64006400u};
  __half2 h[4];
  h[0] = __hsub2(*reinterpret_cast<__half2*>(&v[0]), off);
  h[1] = __hfma2(*reinterpret_cast<__half2*>(&v[1]), sixteenth, m72);
  h[2] = __hsub2(*reinterpret_cast<__half2*>(&v[2]), off);
  h[3] = __hfma2(*reinterpret_cast<__half2*>(&v[3]), sixteenth, m72);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (scale) h[i] = __hmul2(h[i], s2);
    o[i] = *reinterpret_cast<uint32_t*>(&h[i]);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// position of element k within its 8-element chunk in the operand layout
TMOE_HD int p8(int k) { return (k & ~7) | (((k & 3) << 1) | ((k >> 2) & 1)); }

// 2D TMA tile load (no multicast) into this CTA's shared memory, completing
// `bytes` of transaction on the mbarrier.
TMOE_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
TMOE_DEV void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace tc
}  // namespace tmoe
