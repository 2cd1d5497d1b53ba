// Host-side interface of the KV append kernel (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fat {

struct AppendArgs {
  void* k_cache{};
  void* v_cache{};
  int64_t kv_sp{}, kv_ss{}, kv_sh{};  // element strides: page, slot, head
  int64_t num_pages{};
  const int32_t* page_table{};
  int64_t pt_sb{}, max_pages{};
  int32_t* seq_lens{};                 // read, then incremented by one per appended sequence
  const void* new_k{};
  const void* new_v{};
  int64_t new_sb{}, new_sh{};          // element strides of new_k / new_v: sequence, head
  float* k_scale{};                    // 8-bit caches: [num_pages][num_kv_heads] (stride scale_sp)
  float* v_scale{};
  int64_t scale_sp{};
  int batch{}, num_kv_heads{}, head_dim{}, page_size{};
  int kv_dtype{}, new_dtype{};
  int32_t* error_word{};
  cudaStream_t stream{};
};

int launch_append_tokens(const AppendArgs& a);

}  // namespace fat
