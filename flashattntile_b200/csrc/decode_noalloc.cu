// fat_paged_decode_noalloc: the paged decode for callers that cannot allocate
// device memory.
//
// Some callers of a decode kernel may not call cudaMalloc (or any allocating
// routine) on the path that runs it: engines that carve all device memory
// into a fixed arena at start-up and forbid later allocations, plugins whose
// host framework hands them no allocator and no scratch pointer, and
// latency-critical loops where an allocation could synchronise the device.
// This entry point serves them with the same kernel as fat_paged_decode, its
// split scratch taken from a fixed array in this library's device memory
// instead of a caller-provided buffer.
//
// The array is kNoAllocScratchBytes (4 MiB), a file-scope __device__ global,
// so every GPU that loads the library holds it until the process exits.  In
// host code its name is only a host-side stand-in; the device address is
// obtained once per device with cudaGetSymbolAddress (with that device
// current) and passed to the kernel.  All calls share the array: calls that
// overlap on the GPU (different streams, or different host threads, on one
// device) race on it and must be ordered by the caller.
#include <mutex>
#include <vector>

#include "../../include/flashattn_tile_b200.h"
#include "decode.h"
#include "host_util.h"

namespace fat {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on `device` (the current device), resolved once.
int scratch_address(int device, void** out) {
  static std::mutex mu;
  static std::vector<void*> addr;
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0) return invalid("paged_decode_noalloc: no current CUDA device");
  if (static_cast<size_t>(device) >= addr.size()) addr.resize(device + 1, nullptr);
  if (addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return cuda_failure("cudaGetSymbolAddress(noalloc scratch)", e);
    addr[device] = p;
  }
  *out = addr[device];
  return FAT_OK;
}

}  // namespace
}  // namespace fat

extern "C" int fat_paged_decode_noalloc(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache, const void* v_cache,
    int64_t kv_stride_page, int64_t kv_stride_slot, int64_t kv_stride_head, int64_t num_pages,
    const int32_t* page_table, int64_t page_table_stride, int64_t max_pages, const int32_t* seq_lens,
    const float* k_scale, const float* v_scale, int64_t scale_stride_page, void* out, int64_t out_stride_b,
    int64_t out_stride_h, int batch, int num_heads, int num_kv_heads, int head_dim, int page_size, int q_dtype,
    int kv_dtype, int out_dtype, float softmax_scale, int split_k_hint, int32_t* error_word, void* stream) {
  fat::set_last_error("");
  if (split_k_hint < 1 || split_k_hint > 64)
    return fat::invalid("paged_decode_noalloc: split_k must be in [1, 64], got " + std::to_string(split_k_hint));
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0 || batch < 0 || head_dim <= 0)
    return fat::invalid("paged_decode_noalloc: num_heads must be a positive multiple of num_kv_heads");
  if (batch == 0) return FAT_OK;
  const int device = fat::current_device();
  const size_t need = fat::decode_workspace_bytes(device, batch, num_heads, num_kv_heads, head_dim);
  if (need > fat::kNoAllocScratchBytes) {
    fat::set_last_error("paged_decode_noalloc: this problem needs " + std::to_string(need) +
                        " bytes of split scratch, more than the fixed " +
                        std::to_string(fat::kNoAllocScratchBytes) +
                        " bytes this entry point owns; call fat_paged_decode with a caller buffer");
    return FAT_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  int rc = fat::scratch_address(device, &scratch);
  if (rc != FAT_OK) return rc;

  fat::DecodeArgs a;
  a.q = q;
  a.q_sb = q_stride_b;
  a.q_sh = q_stride_h;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.kv_sp = kv_stride_page;
  a.kv_ss = kv_stride_slot;
  a.kv_sh = kv_stride_head;
  a.num_pages = num_pages;
  a.page_table = page_table;
  a.pt_sb = page_table_stride;
  a.max_pages = max_pages;
  a.seq_lens = seq_lens;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.scale_sp = scale_stride_page;
  a.out = out;
  a.o_sb = out_stride_b;
  a.o_sh = out_stride_h;
  a.batch = batch;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.page_size = page_size;
  a.q_dtype = q_dtype;
  a.kv_dtype = kv_dtype;
  a.out_dtype = out_dtype;
  a.softmax_scale = softmax_scale;
  a.workspace = scratch;
  a.workspace_bytes = fat::kNoAllocScratchBytes;
  a.error_word = error_word;
  a.stream = static_cast<cudaStream_t>(stream);
  // A refused call queues no GPU work: every argument is checked before the
  // ticket clear below.
  rc = fat::check_paged_decode(a);
  if (rc != FAT_OK) return rc;
  // The per-unit tickets must start at zero.  A completed call leaves them
  // zero, but one that stopped early (a device error) may not, and nothing on
  // the host knows without a synchronisation: clear them on this call's stream
  // (a memset node of 4 bytes per unit, ~2 us of GPU time, ahead of the kernel).
  size_t off = 0, bytes = 0;
  fat::decode_ticket_range(device, batch, num_heads, num_kv_heads, head_dim, &off, &bytes);
  const cudaError_t e =
      cudaMemsetAsync(static_cast<unsigned char*>(scratch) + off, 0, bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fat::cuda_failure("paged_decode_noalloc: clearing tickets", e);
  return fat::launch_paged_decode(a);
}
