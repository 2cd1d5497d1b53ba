// Host-side interface of the cache-metadata statistics kernel (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fat {

// Queues the reduction and the copy of the four results to host_out on
// `stream` (the caller synchronises before reading host_out).
// device_scratch: 4 int32 on the device.
int cache_value_stats(const int32_t* seq_lens, const int32_t* page_table, int64_t page_table_stride, int batch,
                      int64_t max_pages, int page_size, int32_t* device_scratch, int32_t* host_out,
                      cudaStream_t stream);

}  // namespace fat
