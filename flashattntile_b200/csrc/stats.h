// Host-side interface of the cache-metadata statistics kernel (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fat {

// Queues the reduction on `stream`; it writes the four results straight into
// host_out when that is device-mapped pinned host memory, else into
// device_scratch (4 int32 on the device) followed by a copy to host_out.  The
// caller synchronises before reading host_out.
int cache_value_stats(const int32_t* seq_lens, const int32_t* page_table, int64_t page_table_stride, int batch,
                      int64_t max_pages, int page_size, int32_t* device_scratch, int32_t* host_out,
                      cudaStream_t stream);

}  // namespace fat
