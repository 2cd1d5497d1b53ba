// Host-side helpers shared by the C-ABI entry points: error reporting, device
// properties and TMA tensor-map encoding through the driver entry point (so
// the library does not link libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace fat {

// Thread-local message behind fat_last_error().
void set_last_error(const std::string& msg);
const char* last_error();

// Return FAT_ERR_INVALID_ARGUMENT with `msg` recorded.
int invalid(const std::string& msg);
int unsupported(const std::string& msg);
int cuda_failure(const char* what, cudaError_t err);

// Streaming-multiprocessor count of `device` (cached per device).
int sm_count(int device);
// Limit of every bounded in-kernel wait for launches made from now on
// (fat_set_wait_limit_ns; kDefaultWaitLimitNs until set).
constexpr uint64_t kDefaultWaitLimitNs = 2000000000ull;
uint64_t wait_limit_ns();
uint64_t set_wait_limit_ns(uint64_t ns);  // returns the previous limit; 0 restores the default
// Failure-path tests: true for each of the next `n` decode / prefill launches
// that asked (fat_expire_next_waits), false afterwards.
bool take_expire_request();
void request_expiry(int n);

// How prefill feeds P into P.V (fat_set_prefill_p_split): -1 automatic (bf16:
// mode 3, paged K/V mode 1; fp16: mode 0), 0 rounded once (the reference
// kernel's arithmetic), 1 a 16-bit remainder on key tiles holding a key that
// weighs more than 1/16 of its row so far, 2 remainder on every key tile, 3
// (bf16) P.V in fp16 against a scaled fp16 copy of V.
int set_prefill_p_split(int mode);  // returns the previous setting
int prefill_p_split(bool bf16);     // the mode a launch of that dtype uses

// Prefill grid (fat_set_prefill_schedule): 0 persistent when every CTA's item
// list fits (the default), 1 always one CTA per (head, sequence, query pair).
int set_prefill_schedule(int mode);  // returns the previous setting
int prefill_schedule();

// The calling thread's current CUDA device, or -1 when there is none (no
// device, or the runtime failed to report it).
int current_device();

// Raise `func`'s dynamic shared-memory limit to `bytes` once per (kernel, device).
cudaError_t ensure_smem_limit(const void* func, int bytes, int device);

// cuTensorMapEncodeTiled resolved through cudaGetDriverEntryPoint.
// dims/strides are innermost-first; strides[i] is the byte stride of dim i+1.
// `promotion` widens each L2 fill (use 128 B when a box row is only 128 B wide,
// so neighbouring rows of other heads are not fetched along).
bool encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle,
                  std::string* why, CUtensorMapL2promotion promotion = CU_TENSOR_MAP_L2_PROMOTION_L2_256B);

}  // namespace fat
