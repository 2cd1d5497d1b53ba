// Value statistics of a paged cache's metadata in one launch and one 16-byte
// transfer: (min seq_len, max seq_len, min used page id, max used page id),
// where the used page-table entries are the first ceil(max seq_len / page_size)
// columns of every row.
//
// These are the numbers FlashAttnTile's validate_cache checks on the host
// (flashattn_tile/paging.py:84-130: non-negative lengths, lengths within the
// page table's capacity, page ids inside the pool); the reference reads the
// tensors back and reduces them with torch, a dozen small launches and a
// synchronisation per decode call.  One CTA reduces them here.
#include <limits.h>

#include "common.cuh"
#include "host_util.h"
#include "stats.h"

namespace fat {
namespace {

constexpr int kStatsThreads = 512;

__device__ __forceinline__ void block_minmax(int& lo, int& hi, int* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if (lane == 0) {
    sh[2 * warp] = lo;
    sh[2 * warp + 1] = hi;
  }
  __syncthreads();
  lo = INT_MAX;
  hi = INT_MIN;
  for (int w = 0; w < kStatsThreads / 32; ++w) {
    lo = min(lo, sh[2 * w]);
    hi = max(hi, sh[2 * w + 1]);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kStatsThreads) cache_stats_kernel(const int32_t* seq_lens, const int32_t* table,
                                                                    long long pt_sb, int batch, int max_pages,
                                                                    int page_size, int32_t* out) {
  __shared__ int sh[2 * kStatsThreads / 32];
  int lo = INT_MAX, hi = INT_MIN;
  for (int b = threadIdx.x; b < batch; b += kStatsThreads) {
    const int v = __ldg(seq_lens + b);
    lo = min(lo, v);
    hi = max(hi, v);
  }
  block_minmax(lo, hi, sh);
  // Columns a sequence of the maximum length reaches (none if that length is <= 0).
  const long long need64 = hi > 0 ? (static_cast<long long>(hi) + page_size - 1) / page_size : 0;
  const int need = static_cast<int>(min(need64, static_cast<long long>(max_pages)));
  // The used entries, flattened (row-major over [batch, need]), kUnroll
  // independent loads in flight per thread: one memory latency per
  // kUnroll * kStatsThreads entries instead of one per row segment.
  constexpr int kUnroll = 8;
  int pmin = INT_MAX, pmax = INT_MIN;
  const long long total = static_cast<long long>(batch) * need;
  for (long long base = 0; base < total; base += static_cast<long long>(kUnroll) * kStatsThreads) {
    int v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long i = base + static_cast<long long>(u) * kStatsThreads + threadIdx.x;
      v[u] = INT_MAX;
      if (i < total) {
        const long long b = i / need;
        v[u] = __ldg(table + b * pt_sb + (i - b * need));
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long i = base + static_cast<long long>(u) * kStatsThreads + threadIdx.x;
      if (i < total) {
        pmin = min(pmin, v[u]);
        pmax = max(pmax, v[u]);
      }
    }
  }
  block_minmax(pmin, pmax, sh);
  if (threadIdx.x == 0) {
    const int4 r = make_int4(lo, hi, need > 0 ? pmin : 0, need > 0 ? pmax : -1);  // no used entry: (0, -1)
    if ((reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
      *reinterpret_cast<int4*>(out) = r;  // one 16-byte store (out may be mapped host memory)
    } else {
      out[0] = r.x;
      out[1] = r.y;
      out[2] = r.z;
      out[3] = r.w;
    }
  }
}

}  // namespace

int cache_value_stats(const int32_t* seq_lens, const int32_t* page_table, int64_t page_table_stride, int batch,
                      int64_t max_pages, int page_size, int32_t* device_scratch, int32_t* host_out,
                      cudaStream_t stream) {
  if (batch <= 0 || max_pages < 0 || page_size <= 0) return invalid("cache_value_stats: sizes must be positive");
  if (max_pages > INT_MAX) return unsupported("cache_value_stats: page table too wide");
  if (seq_lens == nullptr || page_table == nullptr || device_scratch == nullptr || host_out == nullptr)
    return invalid("cache_value_stats: null pointer argument");
  // Pinned (page-locked, device-mapped) host memory is written by the kernel
  // itself, saving a transfer; any other host memory gets a copy.
  int32_t* direct = nullptr;
  cudaPointerAttributes attr{};
  if ((reinterpret_cast<uintptr_t>(host_out) & 15u) == 0 &&
      cudaPointerGetAttributes(&attr, host_out) == cudaSuccess && attr.type == cudaMemoryTypeHost &&
      attr.devicePointer != nullptr) {
    direct = static_cast<int32_t*>(attr.devicePointer);
  }
  (void)cudaGetLastError();  // a failed attribute query leaves no sticky error behind
  cache_stats_kernel<<<1, kStatsThreads, 0, stream>>>(seq_lens, page_table, page_table_stride, batch,
                                                       static_cast<int>(max_pages), page_size,
                                                       direct != nullptr ? direct : device_scratch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_failure("cache_stats_kernel launch", e);
  if (direct != nullptr) return FAT_OK;
  e = cudaMemcpyAsync(host_out, device_scratch, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return cuda_failure("cudaMemcpyAsync(cache stats)", e);
  return FAT_OK;
}

}  // namespace fat
