// Host-side interface of the varlen prefill kernel (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fat {

struct PrefillArgs {
  const void* q{};
  int64_t q_st{}, q_sh{};  // element strides: token, head
  const void* k{};
  int64_t k_st{}, k_sh{};
  const void* v{};
  int64_t v_st{}, v_sh{};
  void* out{};
  int64_t o_st{}, o_sh{};
  const int32_t* cu_q{};
  const int32_t* cu_k{};
  int batch{};
  int64_t total_q{}, total_k{};
  int num_heads{}, num_kv_heads{}, head_dim{};
  int max_seqlen_q{}, max_seqlen_k{};
  int causal{};
  float softmax_scale{};
  int dtype{}, out_dtype{};
  int32_t* error_word{};
  cudaStream_t stream{};
  // Paged K/V (launch_prefill_paged): k / v are the caches [pages, page_size, kv heads, dim].
  const int32_t* page_table{};
  int64_t pt_sb{}, max_pages{}, num_pages{};
  int64_t kv_sp{}, kv_ss{}, kv_sh{};  // element strides: page, slot, head
  int page_size{};
  const int32_t* seq_lens_k{};         // [batch] cached tokens per sequence (the keys)
};

int launch_prefill_varlen(const PrefillArgs& a);
// Queries of sequence b are its last q_len cached positions (bottom-right
// causal alignment); keys are its seq_lens_k[b] tokens read through the page table.
int launch_prefill_paged(const PrefillArgs& a);

}  // namespace fat
