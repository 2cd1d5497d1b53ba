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
};

int launch_prefill_varlen(const PrefillArgs& a);

}  // namespace fat
