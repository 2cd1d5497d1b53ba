// Host-side interface of the decode kernels (internal to the library).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace fat {

struct DecodeArgs {
  const void* q{};
  int64_t q_sb{}, q_sh{};
  const void* k_cache{};
  const void* v_cache{};
  int64_t kv_sp{}, kv_ss{}, kv_sh{};  // element strides: page, slot, head
  int64_t num_pages{};
  const int32_t* page_table{};
  int64_t pt_sb{}, max_pages{};
  const int32_t* seq_lens{};
  const float* k_scale{};
  const float* v_scale{};
  int64_t scale_sp{};
  void* out{};
  int64_t o_sb{}, o_sh{};
  int batch{}, num_heads{}, num_kv_heads{}, head_dim{}, page_size{};
  int q_dtype{}, kv_dtype{}, out_dtype{};
  float softmax_scale{};
  void* workspace{};
  size_t workspace_bytes{};
  int32_t* error_word{};
  cudaStream_t stream{};
  float* lse = nullptr;  // optional [batch, num_heads] base-2 log-sum-exp of the scaled scores
  int64_t lse_sb = 0;
};

// Scratch bytes for one decode problem: per-CTA split partials + one ticket per unit.
size_t decode_workspace_bytes(int device, int batch, int num_heads, int num_kv_heads, int head_dim);

// Where, inside that scratch, the per-unit tickets live (they must be zero when a
// call starts; every successful call leaves them zero).
void decode_ticket_range(int device, int batch, int num_heads, int num_kv_heads, int head_dim, size_t* offset,
                         size_t* bytes);

// Every argument check of launch_paged_decode except the workspace size (no
// GPU work, no CUDA call). Returns a fat_status.
int check_paged_decode(const DecodeArgs& a);

// Validate, build the TMA descriptors and launch. Returns a fat_status.
int launch_paged_decode(const DecodeArgs& a);

}  // namespace fat
