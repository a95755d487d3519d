// Host-side launch helpers shared by every kernel file: per-device caches
// guarded by one mutex, so a process that drives several GPUs from several
// host threads raises each kernel's shared-memory limit on every device it
// launches on, exactly once per (kernel, device).
#include <map>
#include <mutex>
#include <utility>

#include "tmoe_internal.h"

namespace tmoe {

namespace {
std::mutex g_attr_mu;
std::map<std::pair<const void*, int>, int> g_smem_set;   // (kernel, device) -> bytes raised to
std::map<int, int> g_sm_count;                           // device -> SMs
}  // namespace

cudaError_t ensure_smem_attr(const void* func, int bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  auto key = std::make_pair(func, dev);
  auto it = g_smem_set.find(key);
  if (it != g_smem_set.end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  g_smem_set[key] = bytes;
  return cudaSuccess;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 1;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  auto it = g_sm_count.find(dev);
  if (it != g_sm_count.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 1;
  g_sm_count[dev] = n;
  return n;
}

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}
}  // namespace

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base,
               unsigned long long cols, unsigned long long rows, unsigned box_cols,
               unsigned box_rows, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base || cols == 0 || rows == 0) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * (cuuint64_t)esize};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tmoe
