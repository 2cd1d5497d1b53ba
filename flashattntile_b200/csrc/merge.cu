// Log-sum-exp merge of attention partials computed over disjoint key ranges.
//
// Part r holds, for every row (sequence, query head), the attention output
// normalised over its own keys, o_r, and the base-2 log-sum-exp of its scaled
// scores, lse_r = m_r + log2(l_r).  The attention over the union of the key
// ranges is
//     out = sum_r o_r 2^(lse_r - M) / sum_r 2^(lse_r - M),   M = max_r lse_r,
// the same merge as FlashAttnTile's split-K reduce (kernels/decode.py:341-352,
// there on unnormalised partials and natural logs).  Used to combine the
// sequence-parallel pieces that different GPUs compute for one long context.
#include <math_constants.h>

#include "common.cuh"
#include "host_util.h"
#include "merge.h"

namespace fat {
namespace {

template <typename T>
__global__ void __launch_bounds__(128) lse_merge_kernel(MergeArgs a) {
  const long long row = blockIdx.x;
  float M = -CUDART_INF_F;
  for (int r = 0; r < a.parts; ++r) M = fmaxf(M, __ldg(a.lse + r * a.lse_part_stride + row));
  float wsum = 0.f;
  for (int r = 0; r < a.parts; ++r) {
    const float l = __ldg(a.lse + r * a.lse_part_stride + row);
    wsum += (M == -CUDART_INF_F) ? 0.f : exp2f(l - M);
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  for (int d = threadIdx.x; d < a.head_dim; d += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < a.parts; ++r) {
      const float l = __ldg(a.lse + r * a.lse_part_stride + row);
      const float w = (M == -CUDART_INF_F) ? 0.f : exp2f(l - M);
      if (w != 0.f) acc += w * __ldg(a.o + r * a.o_part_stride + row * a.head_dim + d);
    }
    const float v = acc * inv;
    if (a.out_dtype == FAT_DTYPE_F32) {
      static_cast<float*>(a.out)[row * a.head_dim + d] = v;
    } else {
      static_cast<T*>(a.out)[row * a.head_dim + d] = from_float<T>(v);
    }
  }
  if (a.lse_out != nullptr && threadIdx.x == 0) a.lse_out[row] = (wsum > 0.f) ? M + log2f(wsum) : -CUDART_INF_F;
}

}  // namespace

int launch_lse_merge(const MergeArgs& a) {
  if (a.parts <= 0 || a.rows < 0 || a.head_dim <= 0) return invalid("lse_merge: sizes must be positive");
  if (a.rows == 0) return FAT_OK;
  if (a.o == nullptr || a.lse == nullptr || a.out == nullptr) return invalid("lse_merge: null pointer argument");
  if (a.rows > 2147483647LL) return unsupported("lse_merge: too many rows");
  const dim3 grid(unsigned(a.rows));
  switch (a.out_dtype) {
    case FAT_DTYPE_F16:
      lse_merge_kernel<__half><<<grid, 128, 0, a.stream>>>(a);
      break;
    case FAT_DTYPE_BF16:
      lse_merge_kernel<__nv_bfloat16><<<grid, 128, 0, a.stream>>>(a);
      break;
    case FAT_DTYPE_F32:
      lse_merge_kernel<float><<<grid, 128, 0, a.stream>>>(a);
      break;
    default:
      return unsupported("lse_merge: out dtype must be fp16, bf16 or fp32");
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_failure("lse_merge launch", e);
  return FAT_OK;
}

}  // namespace fat
