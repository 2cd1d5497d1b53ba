// Host-side interface of the page-table gather kernel (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fat {

struct GatherArgs {
  const void* k_cache{};
  const void* v_cache{};
  int64_t sp_bytes{}, ss_bytes{}, sh_bytes{};  // byte strides: page, slot, head
  int64_t num_pages{};
  const int32_t* page_table{};
  int64_t pt_sb{}, max_pages{};
  const int32_t* seq_lens{};
  void* out_k{};
  void* out_v{};
  int64_t max_len{};
  int batch{}, num_kv_heads{}, page_size{};
  int64_t row_bytes{};  // head_dim * element size
  int32_t* error_word{};
  cudaStream_t stream{};
};

int launch_gather_paged(const GatherArgs& a);

}  // namespace fat
