// tmoe_gather_qmm_int8_static: the int8 expert gather of tmoe_gather_qmm_int8
// for callers that cannot allocate device memory at the call site — a host
// binding that holds only the input and output pointers and has no device
// allocator of its own (a ctypes or cgo stub), or code that runs while a
// serving engine has reserved the whole device memory pool for itself.  Such a
// caller passes no workspace: the routing plan, the int8 activation codes and
// their scales live in one fixed scratch array compiled into this library's
// device image (kStaticScratchBytes per device), so no call allocates.
//
// Set-up: the first call on each device looks the array up with
// cudaGetSymbolAddress, with that device current (it is the calling thread's
// current device).  That lookup may load this library's device module, so
// make the first call on a device before any stream capture begins.  The
// address is cached with the CUDA context it belongs to; after a
// cudaDeviceReset (a new primary context, into which the module is loaded
// again) the next call sees a different context and looks the array up anew,
// so it is again a set-up call that must come before any capture.
//
// Sharing: every call on a device uses the same array.  Two calls in flight at
// once (on two streams, or from two host threads) overwrite each other's
// scratch; serialise them on one stream.  Nothing in the scratch has to start
// at zero: every piece is written in full by the routing-plan and quantiser
// kernels before the GEMM reads it.
#include <cstdio>
#include <mutex>

#include "../../include/titan_moe.h"
#include "tmoe_internal.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};
void* g_scratch_ctx[kMaxDevices] = {};   // the context g_scratch_ptr[dev] was looked up in

// The calling thread's current CUDA context (cuCtxGetCurrent through the
// runtime's driver entry point, so the library needs no libcuda link), or
// null when it cannot be read.
void* current_context() {
  typedef int (*CtxGetCurrent)(void**);
  static CtxGetCurrent fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<CtxGetCurrent>(f);
  }();
  void* ctx = nullptr;
  if (!fn || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Per-device set-up: the scratch array's device address, looked up once.
int scratch_for_current_device(void** out, char* msg, size_t msg_len) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    snprintf(msg, msg_len, "cudaGetDevice: %s", cudaGetErrorString(e));
    return TMOE_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    snprintf(msg, msg_len, "device ordinal %d outside 0..%d", dev, kMaxDevices - 1);
    return TMOE_ERR_UNSUPPORTED;
  }
  void* ctx = current_context();           // null until the runtime made a context current
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[dev] || !ctx || ctx != g_scratch_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p) {
      snprintf(msg, msg_len, "cudaGetSymbolAddress(static scratch) on device %d: %s", dev,
               cudaGetErrorString(e));
      return TMOE_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
    g_scratch_ctx[dev] = current_context();   // the lookup made the primary context current
  }
  *out = g_scratch_ptr[dev];
  return TMOE_OK;
}

thread_local char g_msg[256];

}  // namespace

extern "C" {

size_t tmoe_static_scratch_bytes(void) { return kStaticScratchBytes; }

int tmoe_gather_qmm_int8_static(const uint16_t* x, const uint32_t* w, const uint16_t* scales_t,
                                const uint16_t* biases_t, const int32_t* rhs, int R, int E, int N,
                                int K, uint16_t* y, void* stream) {
  const size_t need = tmoe_gather_qmm_int8_workspace_size(R, E, N, K);
  if (need > kStaticScratchBytes) {
    snprintf(g_msg, sizeof(g_msg),
             "tmoe_gather_qmm_int8_static: R=%d E=%d K=%d needs %zu bytes of scratch, more than the "
             "%zu-byte static scratch; use tmoe_gather_qmm_int8 with a workspace",
             R, E, K, need, kStaticScratchBytes);
    return tmoe::record_error(TMOE_ERR_WORKSPACE, g_msg);
  }
  void* ws = nullptr;
  if (int rc = scratch_for_current_device(&ws, g_msg, sizeof(g_msg)))
    return tmoe::record_error(rc, g_msg);
  return tmoe_gather_qmm_int8(x, w, scales_t, biases_t, rhs, R, E, N, K, ws, kStaticScratchBytes,
                              y, stream);
}

}  // extern "C"
