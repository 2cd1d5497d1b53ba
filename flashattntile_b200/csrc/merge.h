// Host-side interface of the log-sum-exp merge kernel (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fat {

struct MergeArgs {
  const float* o{};  // [parts][rows][head_dim] normalised partial outputs
  int64_t o_part_stride{};  // elements between parts
  const float* lse{};  // [parts][rows] base-2 log-sum-exp
  int64_t lse_part_stride{};
  int parts{};
  int64_t rows{};
  int head_dim{};
  void* out{};  // [rows][head_dim] of out_dtype
  int out_dtype{};
  float* lse_out{};  // optional [rows] merged log-sum-exp
  cudaStream_t stream{};
};

int launch_lse_merge(const MergeArgs& a);

}  // namespace fat
