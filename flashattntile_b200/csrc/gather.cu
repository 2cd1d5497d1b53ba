// Bit-exact page-table gather: padded contiguous [batch, max_len, kv_heads, dim]
// copies of a paged K/V cache, zero past each sequence's length.
//
// Same result as FlashAttnTile's gather_paged (flashattn_tile/paging.py:213-256),
// which loops over sequences in Python and calls index_select per sequence; here
// one launch copies every row with the widest vector width the pointers and
// strides allow.  Rows whose page id is outside [0, num_pages) are written as
// zeros and FAT_DEVERR_BAD_PAGE is raised in the error word.
#include "common.cuh"
#include "gather.h"
#include "host_util.h"

namespace fat {
namespace {

template <typename V>
__global__ void __launch_bounds__(256) gather_kernel(GatherArgs a, int vec_per_row) {
  const int b = blockIdx.y;
  const int len = max(__ldg(a.seq_lens + b), 0);
  const int rows_per_tok = a.num_kv_heads;
  const long long tok_base = (long long)blockIdx.x * 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int tt = warp; tt < 64; tt += 8) {
    const long long t = tok_base + tt;
    if (t >= a.max_len) break;
    int phys = -1;
    if (t < len) {
      const long long lp = t / a.page_size;
      phys = lp < a.max_pages ? __ldg(a.page_table + (long long)b * a.pt_sb + lp) : -1;
      if (phys < 0 || phys >= a.num_pages) {
        if (lane == 0) raise_error(a.error_word, FAT_DEVERR_BAD_PAGE);
        phys = -1;
      }
    }
    const int slot = int(t % a.page_size);
    for (int which = 0; which < 2; ++which) {
      const uint8_t* src = static_cast<const uint8_t*>(which ? a.v_cache : a.k_cache);
      uint8_t* dst = static_cast<uint8_t*>(which ? a.out_v : a.out_k);
      for (int h = 0; h < rows_per_tok; ++h) {
        V* d = reinterpret_cast<V*>(dst + (((long long)b * a.max_len + t) * rows_per_tok + h) * a.row_bytes);
        if (phys >= 0) {
          const V* s = reinterpret_cast<const V*>(src + (long long)phys * a.sp_bytes + (long long)slot * a.ss_bytes +
                                                  (long long)h * a.sh_bytes);
          for (int i = lane; i < vec_per_row; i += 32) d[i] = __ldg(s + i);
        } else {
          V z;
          memset(&z, 0, sizeof(V));
          for (int i = lane; i < vec_per_row; i += 32) d[i] = z;
        }
      }
    }
  }
}

template <typename V>
int launch(const GatherArgs& a) {
  const int vec = int(a.row_bytes / (long long)sizeof(V));
  dim3 grid(unsigned((a.max_len + 63) / 64), unsigned(a.batch));
  gather_kernel<V><<<grid, 256, 0, a.stream>>>(a, vec);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_failure("gather_paged launch", e);
  return FAT_OK;
}

}  // namespace

int launch_gather_paged(const GatherArgs& a) {
  if (a.batch < 0 || a.max_len < 0 || a.num_kv_heads <= 0 || a.row_bytes <= 0 || a.page_size <= 0)
    return invalid("gather_paged: sizes must be positive");
  if (a.batch == 0 || a.max_len == 0) return FAT_OK;
  if (a.k_cache == nullptr || a.v_cache == nullptr || a.page_table == nullptr || a.seq_lens == nullptr ||
      a.out_k == nullptr || a.out_v == nullptr)
    return invalid("gather_paged: null pointer argument");
  if (a.max_len > 65535LL * 64) return unsupported("gather_paged: max_len too large");
  uintptr_t bits = reinterpret_cast<uintptr_t>(a.k_cache) | reinterpret_cast<uintptr_t>(a.v_cache) |
                   reinterpret_cast<uintptr_t>(a.out_k) | reinterpret_cast<uintptr_t>(a.out_v) |
                   uintptr_t(a.sp_bytes) | uintptr_t(a.ss_bytes) | uintptr_t(a.sh_bytes) | uintptr_t(a.row_bytes);
  if ((bits & 15u) == 0) return launch<uint4>(a);
  if ((bits & 7u) == 0) return launch<uint2>(a);
  if ((bits & 3u) == 0) return launch<uint32_t>(a);
  if ((bits & 1u) == 0) return launch<uint16_t>(a);
  return launch<uint8_t>(a);
}

}  // namespace fat
