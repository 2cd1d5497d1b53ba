// Append one token per sequence to a paged KV cache, on the device.
//
// 16-bit caches: FlashAttnTile's append_tokens (flashattn_tile/paging.py:172-210)
// -- token b goes to page page_table[b, seq_lens[b] / page_size], slot
// seq_lens[b] % page_size, then seq_lens[b] += 1 -- without its host round
// trips (one CTA per sequence; a position or page id out of range is recorded
// as FAT_DEVERR_BAD_PAGE and that sequence is left unchanged).
//
// INT8 / FP8-e4m3 caches (quantise on write; the reference only quantises a
// whole cache offline, quant.py:84-142): the page receiving the token gets the
// scale quantize_kv_pages would give its valid tokens (slots 0..slot of this
// sequence, the old ones dequantised as code * scale, plus the new token):
//     scale = max(absmax / maxval, 1e-8),  maxval = 127 (int8) | 448 (e4m3),
// the old codes are requantised with it when it changed, and the new token is
// quantised with it (int8: round half to even, clamp to +-127; e4m3: clamp to
// +-448, round to nearest even).  Every step is one correctly rounded fp32
// operation, so the result is bit-identical to the same steps done on the CPU.
#include <cuda_fp8.h>

#include "append.h"
#include "common.cuh"
#include "host_util.h"

namespace fat {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;

template <typename TIn>
__device__ __forceinline__ float to_f32(TIn x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) {
  return x;
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) {
  return __half2float(x);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <int KVT>
struct Codec;

template <>
struct Codec<FAT_DTYPE_I8> {
  static constexpr float kMax = 127.f;
  __device__ static float decode(uint8_t c) { return float(int8_t(c)); }
  __device__ static uint8_t encode(float v) {
    const float r = fminf(fmaxf(rintf(v), -kMax), kMax);  // round half to even, then clamp
    return uint8_t(int8_t(r));
  }
};

template <>
struct Codec<FAT_DTYPE_E4M3> {
  static constexpr float kMax = 448.f;
  __device__ static float decode(uint8_t c) {
    return __half2float(__half(__nv_cvt_fp8_to_halfraw(__nv_fp8_storage_t(c), __NV_E4M3)));
  }
  __device__ static uint8_t encode(float v) {
    v = fminf(fmaxf(v, -kMax), kMax);
    return uint8_t(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
  }
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// KVT: cache element type; TIn: type of the new tokens.  One CTA per sequence,
// one warp per KV head at a time, lanes over head_dim (coalesced).
template <int KVT, typename TIn>
__global__ void __launch_bounds__(kThreads) append_kernel(const AppendArgs a) {
  constexpr bool kQuant = KVT == FAT_DTYPE_I8 || KVT == FAT_DTYPE_E4M3;
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = a.head_dim;
  const int pos = a.seq_lens[b];
  const long long cap = (long long)a.max_pages * a.page_size;
  int page = -1, slot = 0;
  if (pos >= 0 && pos < cap) {
    page = __ldg(a.page_table + (long long)b * a.pt_sb + pos / a.page_size);
    slot = pos % a.page_size;
  }
  if (page < 0 || page >= a.num_pages) {  // uniform for the CTA
    if (threadIdx.x == 0) raise_error(a.error_word, FAT_DEVERR_BAD_PAGE);
    return;
  }
  for (int h = warp; h < a.num_kv_heads; h += kWarps) {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const TIn* src = static_cast<const TIn*>(t ? a.new_v : a.new_k) + (long long)b * a.new_sb + (long long)h * a.new_sh;
      const long long head_off = (long long)page * a.kv_sp + (long long)h * a.kv_sh;
      if constexpr (!kQuant) {
        TIn* dst = static_cast<TIn*>(t ? a.v_cache : a.k_cache) + head_off + (long long)slot * a.kv_ss;
        for (int d = lane; d < hd; d += 32) dst[d] = src[d];  // bit-exact copy
      } else {
        using C = Codec<KVT>;
        uint8_t* codes = static_cast<uint8_t*>(t ? a.v_cache : a.k_cache) + head_off;
        float* scale = (t ? a.v_scale : a.k_scale) + (long long)page * a.scale_sp + h;
        float amax_new = 0.f;
        for (int d = lane; d < hd; d += 32) amax_new = fmaxf(amax_new, fabsf(to_f32<TIn>(src[d])));
        amax_new = warp_max(amax_new);
        const float s_old = *scale;
        float cmax = 0.f;  // largest |code| among this sequence's earlier tokens on the page
        for (int r = 0; r < slot; ++r)
          for (int d = lane; d < hd; d += 32) cmax = fmaxf(cmax, fabsf(C::decode(codes[(long long)r * a.kv_ss + d])));
        cmax = warp_max(cmax);
        const float amax_old = slot > 0 ? __fmul_rn(cmax, s_old) : 0.f;
        const float s_new = fmaxf(__fdiv_rn(fmaxf(amax_old, amax_new), C::kMax), 1e-8f);
        if (slot > 0 && s_new != s_old) {
          for (int r = 0; r < slot; ++r)
            for (int d = lane; d < hd; d += 32) {
              uint8_t* c = codes + (long long)r * a.kv_ss + d;
              *c = C::encode(__fdiv_rn(__fmul_rn(C::decode(*c), s_old), s_new));
            }
        }
        for (int d = lane; d < hd; d += 32)
          codes[(long long)slot * a.kv_ss + d] = C::encode(__fdiv_rn(to_f32<TIn>(src[d]), s_new));
        __syncwarp();
        if (lane == 0) *scale = s_new;
      }
    }
  }
  __syncthreads();  // every thread has read seq_lens[b]
  if (threadIdx.x == 0) a.seq_lens[b] = pos + 1;
}

template <int KVT, typename TIn>
int launch_dim(const AppendArgs& a) {
  append_kernel<KVT, TIn><<<dim3(unsigned(a.batch)), kThreads, 0, a.stream>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_failure("append_tokens launch", e);
  return FAT_OK;
}

template <int KVT>
int launch_quant(const AppendArgs& a) {
  switch (a.new_dtype) {
    case FAT_DTYPE_F16:
      return launch_dim<KVT, __half>(a);
    case FAT_DTYPE_BF16:
      return launch_dim<KVT, __nv_bfloat16>(a);
    case FAT_DTYPE_F32:
      return launch_dim<KVT, float>(a);
    default:
      return unsupported("append_tokens: new tokens must be fp16, bf16 or fp32 for an 8-bit cache");
  }
}

}  // namespace

int launch_append_tokens(const AppendArgs& a) {
  if (a.batch < 0 || a.num_kv_heads <= 0 || a.page_size <= 0 || a.head_dim <= 0)
    return invalid("append_tokens: batch must be non-negative; num_kv_heads, head_dim and page_size positive");
  if (a.batch == 0) return FAT_OK;
  if (a.k_cache == nullptr || a.v_cache == nullptr || a.page_table == nullptr || a.seq_lens == nullptr ||
      a.new_k == nullptr || a.new_v == nullptr)
    return invalid("append_tokens: null pointer argument");
  if (a.num_pages <= 0 || a.max_pages <= 0) return invalid("append_tokens: empty cache or page table");
  switch (a.kv_dtype) {
    case FAT_DTYPE_F16:
    case FAT_DTYPE_BF16:
      if (a.new_dtype != a.kv_dtype) return invalid("append_tokens: new_k/new_v dtype must match the cache dtype");
      return a.kv_dtype == FAT_DTYPE_F16 ? launch_dim<FAT_DTYPE_F16, __half>(a)
                                         : launch_dim<FAT_DTYPE_BF16, __nv_bfloat16>(a);
    case FAT_DTYPE_I8:
    case FAT_DTYPE_E4M3:
      if (a.k_scale == nullptr || a.v_scale == nullptr)
        return invalid("append_tokens: an int8/fp8 cache needs k_scale and v_scale");
      return a.kv_dtype == FAT_DTYPE_I8 ? launch_quant<FAT_DTYPE_I8>(a) : launch_quant<FAT_DTYPE_E4M3>(a);
    default:
      return unsupported("append_tokens: cache dtype must be fp16, bf16, int8 or float8_e4m3fn");
  }
}

}  // namespace fat
