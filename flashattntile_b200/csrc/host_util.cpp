#include "host_util.h"

#include <atomic>
#include <mutex>
#include <set>
#include <utility>
#include <vector>

#include "../../include/flashattn_tile_b200.h"

namespace fat {

namespace {
thread_local std::string g_last_error;

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn resolve_encode() {
  static std::once_flag once;
  static EncodeFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeFn>(p);
    }
  });
  return fn;
}
}  // namespace

namespace {
std::atomic<uint64_t> g_wait_limit_ns{kDefaultWaitLimitNs};
std::atomic<int> g_expire_requests{0};
std::atomic<int> g_p_split{-1};
std::atomic<int> g_prefill_schedule{0};
}  // namespace

int set_prefill_schedule(int mode) { return g_prefill_schedule.exchange(mode, std::memory_order_relaxed); }
int prefill_schedule() { return g_prefill_schedule.load(std::memory_order_relaxed); }

int set_prefill_p_split(int mode) { return g_p_split.exchange(mode, std::memory_order_relaxed); }

int prefill_p_split(bool bf16) {
  const int mode = g_p_split.load(std::memory_order_relaxed);
  return mode >= 0 ? mode : (bf16 ? 3 : 0);
}

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

uint64_t set_wait_limit_ns(uint64_t ns) {
  return g_wait_limit_ns.exchange(ns == 0 ? kDefaultWaitLimitNs : ns, std::memory_order_relaxed);
}

bool take_expire_request() {
  int n = g_expire_requests.load(std::memory_order_relaxed);
  while (n > 0) {
    if (g_expire_requests.compare_exchange_weak(n, n - 1, std::memory_order_relaxed)) return true;
  }
  return false;
}

void request_expiry(int n) { g_expire_requests.store(n > 0 ? n : 0, std::memory_order_relaxed); }

void set_last_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

int invalid(const std::string& msg) {
  set_last_error(msg);
  return FAT_ERR_INVALID_ARGUMENT;
}

int unsupported(const std::string& msg) {
  set_last_error(msg);
  return FAT_ERR_UNSUPPORTED;
}

int cuda_failure(const char* what, cudaError_t err) {
  set_last_error(std::string(what) + ": " + cudaGetErrorString(err));
  return FAT_ERR_CUDA;
}

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

cudaError_t ensure_smem_limit(const void* func, int bytes, int device) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(func, device);
  if (done.count(key)) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert(key);
  return e;
}

int sm_count(int device) {
  static std::mutex mu;
  static std::vector<int> cache;
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0) device = 0;
  if (static_cast<size_t>(device) >= cache.size()) cache.resize(device + 1, 0);
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
    cache[device] = n;
  }
  return cache[device];
}

bool encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle,
                  std::string* why, CUtensorMapL2promotion promotion) {
  EncodeFn fn = resolve_encode();
  if (fn == nullptr) {
    *why = "cuTensorMapEncodeTiled is not available from the CUDA driver";
    return false;
  }
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i + 1 < rank) gstride[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), gdim, gstride, bdim, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promotion,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *why = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
}

}  // namespace fat
