// Expert-parallel exchanges over NVLink peer memory (no reference
// counterpart: the reference runs one device).
//
// Each rank owns one device allocation (tmoe_ep_alloc) that the other ranks
// map through CUDA IPC.  Layout of rank d's allocation, for W ranks, a
// capacity of `cap` tokens per source rank, H hidden, k slots, T_max tokens
// of its own:
//   recv_x    [W][cap][H] bf16       rows sent to d by each source rank
//   recv_meta [W][cap][k + 1] int32  their k local expert ids (-1: not on d),
//                                    then the source's token index
//   ret       [T_max * k][H] bf16    expert output of d's (token, slot) pairs,
//                                    written by the owner of each slot
//   flags     [2][W] uint64          dispatch and return flags, one per peer:
//                                    epoch << 32 | count
// Dispatch: a source writes each of its token rows once to every rank that
// owns one of the token's experts (deduplicated), then posts (epoch, rows) in
// that rank's dispatch flag.  Return: an owner's down GEMM stores every served
// pair's output straight into the source's ret row (token, slot) from its
// epilogue, then ep_post posts the epoch in every source's return flag.
// Writes are plain stores to peer memory; the dispatch flag is posted after
// a system-scope fence by every writer and a ticket that picks the kernel's
// last CTA, the return flag by the launch after the GEMM, so a reader that
// sees a flag (an acquire load) sees the data.  Waits are bounded (4 s of device time): on timeout the kernel
// records an error that tmoe_device_status reports and returns.
//
// Reuse across layers needs no double buffer: a source dispatches layer L+1
// only after its weighted sum of layer L, which waited for every owner's
// return of layer L, and an owner returns only after its experts consumed
// the rows of layer L.
#include "common.cuh"
#include "tmoe_internal.h"

namespace tmoe {

__device__ int g_ep_error = 0;

namespace {

// A wait gives up after kEpLimitNs of device time (%globaltimer), or after
// kEpSpin polls should the timer not advance; polls past the first kEpFast
// back off by 256 ns.
constexpr unsigned long long kEpLimitNs = 4000000000ull;
constexpr uint32_t kEpSpin = 1u << 26;
constexpr uint32_t kEpFast = 1u << 10;

TMOE_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

TMOE_DEV void st_release_sys64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
TMOE_DEV unsigned long long ld_acquire_sys64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One CTA per token: its row (and metadata) to every owning rank, at a row
// taken from that rank's counter (rows land in any order: the owner serves
// each row on its own, so the order changes no bit of any output).  The last
// CTA posts the final counts and clears the counters for the next launch.
__global__ void __launch_bounds__(128) ep_dispatch_kernel(EpDispatchArgs a) {
  const int t = blockIdx.x, tid = threadIdx.x;
  const int W = a.world, k = a.k, H = a.H;
  __shared__ int s_last;
  __shared__ int s_row[32];
  if (t < a.T) {                                  // a CTA past the tokens only posts flags
    const int32_t* ids = a.idx + (size_t)t * k;
    if (tid < W) {
      bool mine = false;
      for (int j = 0; j < k; ++j) {
        const int e = ids[j];
        if (e < 0 || e >= W * a.epr) {          // no owner: the slot's return row would stay stale
          if (tid == 0) atomicExch(&g_ep_error, 2);
          continue;
        }
        mine |= e / a.epr == tid;
      }
      s_row[tid] = mine ? atomicAdd(a.counters + 1 + tid, 1) : -1;
    }
    __syncthreads();
    for (int d = 0; d < W; ++d) {
      const int pos = s_row[d];
      if (pos < 0) continue;
      uint8_t* base = static_cast<uint8_t*>(a.peer[d]);
      const size_t row = (size_t)a.rank * a.cap + pos;
      uint4* dst = reinterpret_cast<uint4*>(base + a.off_x + row * H * 2);
      const uint4* src = reinterpret_cast<const uint4*>(a.x + (size_t)t * H);
      for (int i = tid; i < H / 8; i += 128) dst[i] = src[i];
      int32_t* meta = reinterpret_cast<int32_t*>(base + a.off_meta) + row * (k + 1);
      if (tid < k) {
        const int e = ids[tid];
        meta[tid] = (e >= 0 && e / a.epr == d) ? e - d * a.epr : -1;
      } else if (tid == k) {
        meta[k] = t;
      }
    }
  }
  __threadfence_system();     // every writer's stores before the CTA's ticket
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    s_last = ticket_acq_rel(a.counters) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  if (tid < W) {
    const int n = atomicExch(a.counters + 1 + tid, 0);   // final: every CTA added before its ticket
    __threadfence_system();
    unsigned long long* flags = reinterpret_cast<unsigned long long*>(
        static_cast<uint8_t*>(a.peer[tid]) + a.off_flags);
    st_release_sys64(flags + a.rank, ((unsigned long long)(uint32_t)a.epoch << 32) | (uint32_t)n);
  }
  if (tid == 0) a.counters[0] = 0;
}

// The owner's slot list over its receive buffer, one thread per (row, slot)
// f = (s * cap + i) * k + j: the local expert of slot j of row i from source
// s when that row was written this layer (i < rows_in[s]) and the expert is
// here, else -1; and the address of the source's ret row token * k + j
// (0 for a slot not served).
__global__ void __launch_bounds__(256) ep_slots_kernel(EpSlotsArgs a) {
  const long long n = (long long)a.world * a.cap * a.k;
  const long long f = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= n) return;
  const int k = a.k;
  const long long row = f / k;
  const int j = (int)(f - row * k);
  const int s = (int)(row / a.cap), i = (int)(row - (long long)s * a.cap);
  const int32_t* m = a.meta + row * (k + 1);
  const int id = m[j];
  const bool ok = i < a.rows_in[s] && id >= 0 && id < a.epr;
  a.slot_exp[f] = ok ? id : -1;
  unsigned long long addr = 0;
  if (ok)
    addr = reinterpret_cast<unsigned long long>(a.peer[s]) + a.off_ret +
           ((unsigned long long)m[k] * k + j) * 2ull * a.H;
  a.y_rows[f] = addr;
}

// One thread per peer: wait for this epoch's flag; counts[s] = its count,
// or -1 when the wait gave up.
__global__ void ep_wait_kernel(const unsigned long long* flags, int W, int epoch, int32_t* counts) {
  const int s = threadIdx.x;
  if (s >= W) return;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 0; i < kEpSpin; ++i) {
    const unsigned long long v = ld_acquire_sys64(flags + s);
    if ((int)(v >> 32) == epoch) {
      counts[s] = (int)(v & 0xffffffffu);
      return;
    }
    if (i >= kEpFast) {
      __nanosleep(256);
      if (global_ns() - t0 > kEpLimitNs) break;
    }
  }
  counts[s] = -1;
  atomicExch(&g_ep_error, 1);
}

// One thread per rank d: (epoch, counts[d]) into this rank's slot of d's
// flag row `which`.  The return's rows were stored into the sources' ret rows
// by the down GEMM's epilogue (GemmParams::y_ptr / SwParams::y_ptr), an
// earlier launch on the stream, whose storing threads each end with a
// system-scope fence; the flag, stored after that launch completed and after
// this thread's own system-scope fence, cannot overtake them.
__global__ void ep_post_kernel(EpPostArgs a) {
  const int d = threadIdx.x;
  if (d >= a.world) return;
  __threadfence_system();
  unsigned long long* flags = reinterpret_cast<unsigned long long*>(
      static_cast<uint8_t*>(a.peer[d]) + a.off_flags);
  uint32_t n = a.counts ? (uint32_t)a.counts[d] : 0u;
  // a failed wait upstream (a dispatch count of -1) is passed on as count -1,
  // so the sources' guard sees that this layer's return is not valid
  for (int i = 0; a.poison && i < a.npoison; ++i)
    if (a.poison[i] < 0) n = 0xffffffffu;
  st_release_sys64(flags + (size_t)a.which * a.world + a.rank,
                   ((unsigned long long)(uint32_t)a.epoch << 32) | n);
}

// After the source's combine: when any return count is negative (an owner's
// wait gave up upstream, or this rank's own return wait did) the layer's
// output is not valid.  The guard then records the error for
// tmoe_device_status and overwrites the output with bf16 NaN, so no caller
// can take it for a result.  Grid-stride over n bf16 values.
__global__ void ep_guard_kernel(const int32_t* counts, int W, uint16_t* y, long long n) {
  bool bad = false;
  for (int s = 0; s < W; ++s) bad |= counts[s] < 0;
  if (!bad) return;
  if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(&g_ep_error, 1);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = 0x7fc0u;
}

}  // namespace

cudaError_t launch_ep_guard(const int32_t* counts, int W, uint16_t* y, long long n,
                            cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  long long blocks = (n + 255) / 256;
  if (blocks > 1184) blocks = 1184;
  ep_guard_kernel<<<(unsigned)blocks, 256, 0, s>>>(counts, W, y, n);
  return cudaGetLastError();
}

cudaError_t launch_ep_dispatch(const EpDispatchArgs& a, cudaStream_t s) {
  ep_dispatch_kernel<<<a.T > 0 ? a.T : 1, 128, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_ep_wait(const unsigned long long* flags, int W, int epoch, int32_t* counts,
                           cudaStream_t s) {
  ep_wait_kernel<<<1, 32, 0, s>>>(flags, W, epoch, counts);
  return cudaGetLastError();
}

cudaError_t launch_ep_slots(const EpSlotsArgs& a, cudaStream_t s) {
  const long long n = (long long)a.world * a.cap * a.k;
  if (n == 0) return cudaSuccess;
  ep_slots_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_ep_post(const EpPostArgs& a, cudaStream_t s) {
  ep_post_kernel<<<1, 32, 0, s>>>(a);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ C ABI

size_t ep_layout(int world, int cap, int H, int k, int T_max, size_t* off) {
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  size_t o = 0;
  off[0] = o; o = up(o + (size_t)world * cap * H * 2);              // recv_x
  off[1] = o; o = up(o + (size_t)world * cap * (k + 1) * 4);        // recv_meta
  off[2] = o; o = up(o + (size_t)T_max * k * H * 2);               // ret
  off[3] = o; o = up(o + (size_t)2 * world * 8);                    // flags
  return o;
}

int ep_error_flag() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_ep_error, sizeof(int));
  return v;
}

}  // namespace tmoe
