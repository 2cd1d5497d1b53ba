// extern "C" entry points of libflashattn_sm100.so (declared in
// include/flashattn_tile_b200.h).  Each one packs its plain arguments and
// forwards to the internal launcher; no C++ types cross the boundary.
#include "../../include/flashattn_tile_b200.h"

#include "decode.h"
#include "gather.h"
#include "merge.h"
#include "append.h"
#include "prefill.h"
#include "stats.h"
#include "host_util.h"

extern "C" {

const char* fat_version(void) { return "flashattn_tile_b200 0.1.0 sm_100a"; }

const char* fat_last_error(void) { return fat::last_error(); }

uint64_t fat_set_wait_limit_ns(uint64_t limit_ns) { return fat::set_wait_limit_ns(limit_ns); }

void fat_expire_next_waits(int launches) { fat::request_expiry(launches); }

int fat_set_prefill_p_split(int mode) {
  if (mode < -1 || mode > 3) {
    fat::set_last_error("prefill p_split must be -1, 0, 1, 2 or 3, got " + std::to_string(mode));
    return -2;
  }
  fat::set_last_error("");
  return fat::set_prefill_p_split(mode);
}

int fat_set_prefill_schedule(int mode) {
  if (mode < 0 || mode > 1) {
    fat::set_last_error("prefill schedule must be 0 or 1, got " + std::to_string(mode));
    return -2;
  }
  fat::set_last_error("");
  return fat::set_prefill_schedule(mode);
}

size_t fat_paged_decode_workspace_size(int device, int batch, int num_heads, int num_kv_heads, int head_dim) {
  return fat::decode_workspace_bytes(device, batch, num_heads, num_kv_heads, head_dim);
}

namespace {
int decode_entry(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache, const void* v_cache,
                 int64_t kv_stride_page, int64_t kv_stride_slot, int64_t kv_stride_head, int64_t num_pages,
                 const int32_t* page_table, int64_t page_table_stride, int64_t max_pages, const int32_t* seq_lens,
                 const float* k_scale, const float* v_scale, int64_t scale_stride_page, void* out,
                 int64_t out_stride_b, int64_t out_stride_h, float* lse, int64_t lse_stride_b, int batch,
                 int num_heads, int num_kv_heads, int head_dim, int page_size, int q_dtype, int kv_dtype,
                 int out_dtype, float softmax_scale, int split_k_hint, void* workspace, size_t workspace_bytes,
                 int32_t* error_word, void* stream) {
  fat::set_last_error("");
  if (split_k_hint < 1 || split_k_hint > 64)
    return fat::invalid("paged_decode: split_k must be in [1, 64], got " + std::to_string(split_k_hint));
  fat::DecodeArgs a;
  a.q = q;
  a.q_sb = q_stride_b;
  a.q_sh = q_stride_h;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.kv_sp = kv_stride_page;
  a.kv_ss = kv_stride_slot;
  a.kv_sh = kv_stride_head;
  a.num_pages = num_pages;
  a.page_table = page_table;
  a.pt_sb = page_table_stride;
  a.max_pages = max_pages;
  a.seq_lens = seq_lens;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.scale_sp = scale_stride_page;
  a.out = out;
  a.o_sb = out_stride_b;
  a.o_sh = out_stride_h;
  a.batch = batch;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.page_size = page_size;
  a.q_dtype = q_dtype;
  a.kv_dtype = kv_dtype;
  a.out_dtype = out_dtype;
  a.softmax_scale = softmax_scale;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  a.error_word = error_word;
  a.stream = static_cast<cudaStream_t>(stream);
  a.lse = lse;
  a.lse_sb = lse_stride_b;
  return fat::launch_paged_decode(a);
}
}  // namespace

int fat_paged_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache,
                     const void* v_cache, int64_t kv_stride_page, int64_t kv_stride_slot, int64_t kv_stride_head,
                     int64_t num_pages, const int32_t* page_table, int64_t page_table_stride, int64_t max_pages,
                     const int32_t* seq_lens, const float* k_scale, const float* v_scale,
                     int64_t scale_stride_page, void* out, int64_t out_stride_b, int64_t out_stride_h, int batch,
                     int num_heads, int num_kv_heads, int head_dim, int page_size, int q_dtype, int kv_dtype,
                     int out_dtype, float softmax_scale, int split_k_hint, void* workspace, size_t workspace_bytes,
                     int32_t* error_word, void* stream) {
  return decode_entry(q, q_stride_b, q_stride_h, k_cache, v_cache, kv_stride_page, kv_stride_slot, kv_stride_head,
                      num_pages, page_table, page_table_stride, max_pages, seq_lens, k_scale, v_scale,
                      scale_stride_page, out, out_stride_b, out_stride_h, nullptr, 0, batch, num_heads,
                      num_kv_heads, head_dim, page_size, q_dtype, kv_dtype, out_dtype, softmax_scale, split_k_hint,
                      workspace, workspace_bytes, error_word, stream);
}

int fat_paged_decode_lse(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache,
                         const void* v_cache, int64_t kv_stride_page, int64_t kv_stride_slot, int64_t kv_stride_head,
                         int64_t num_pages, const int32_t* page_table, int64_t page_table_stride, int64_t max_pages,
                         const int32_t* seq_lens, const float* k_scale, const float* v_scale,
                         int64_t scale_stride_page, void* out, int64_t out_stride_b, int64_t out_stride_h,
                         float* lse, int64_t lse_stride_b, int batch, int num_heads, int num_kv_heads, int head_dim,
                         int page_size, int q_dtype, int kv_dtype, int out_dtype, float softmax_scale,
                         int split_k_hint, void* workspace, size_t workspace_bytes, int32_t* error_word,
                         void* stream) {
  if (lse == nullptr) {
    fat::set_last_error("paged_decode_lse: lse must not be null");
    return FAT_ERR_INVALID_ARGUMENT;
  }
  return decode_entry(q, q_stride_b, q_stride_h, k_cache, v_cache, kv_stride_page, kv_stride_slot, kv_stride_head,
                      num_pages, page_table, page_table_stride, max_pages, seq_lens, k_scale, v_scale,
                      scale_stride_page, out, out_stride_b, out_stride_h, lse, lse_stride_b, batch, num_heads,
                      num_kv_heads, head_dim, page_size, q_dtype, kv_dtype, out_dtype, softmax_scale, split_k_hint,
                      workspace, workspace_bytes, error_word, stream);
}

int fat_paged_decode_call(const fat_decode_call* c) {
  fat::set_last_error("");
  if (c == nullptr) return fat::invalid("paged_decode_call: null argument struct");
  if (c->stats_out != nullptr) {
    const int rc = fat::cache_value_stats(c->seq_lens, c->page_table, c->page_table_stride, c->batch, c->max_pages,
                                          c->page_size, c->stats_scratch, c->stats_out,
                                          static_cast<cudaStream_t>(c->stream));
    if (rc != FAT_OK) return rc;
    if (c->stats_event != nullptr) {
      const cudaError_t e =
          cudaEventRecord(static_cast<cudaEvent_t>(c->stats_event), static_cast<cudaStream_t>(c->stream));
      if (e != cudaSuccess) return fat::cuda_failure("paged_decode_call: recording stats_event", e);
    }
  }
  return decode_entry(c->q, c->q_stride_b, c->q_stride_h, c->k_cache, c->v_cache, c->kv_stride_page,
                      c->kv_stride_slot, c->kv_stride_head, c->num_pages, c->page_table, c->page_table_stride,
                      c->max_pages, c->seq_lens, c->k_scale, c->v_scale, c->scale_stride_page, c->out,
                      c->out_stride_b, c->out_stride_h, c->lse, c->lse_stride_b, c->batch, c->num_heads,
                      c->num_kv_heads, c->head_dim, c->page_size, c->q_dtype, c->kv_dtype, c->out_dtype,
                      c->softmax_scale, c->split_k_hint, c->workspace, c->workspace_bytes, c->error_word, c->stream);
}

int fat_lse_merge(const float* o, int64_t o_part_stride, const float* lse, int64_t lse_part_stride, int parts,
                  int64_t rows, int head_dim, void* out, int out_dtype, float* lse_out, void* stream) {
  fat::set_last_error("");
  fat::MergeArgs a;
  a.o = o;
  a.o_part_stride = o_part_stride;
  a.lse = lse;
  a.lse_part_stride = lse_part_stride;
  a.parts = parts;
  a.rows = rows;
  a.head_dim = head_dim;
  a.out = out;
  a.out_dtype = out_dtype;
  a.lse_out = lse_out;
  a.stream = static_cast<cudaStream_t>(stream);
  return fat::launch_lse_merge(a);
}

int fat_prefill_varlen(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k, int64_t k_stride_t,
                       int64_t k_stride_h, const void* v, int64_t v_stride_t, int64_t v_stride_h, void* out,
                       int64_t out_stride_t, int64_t out_stride_h, const int32_t* cu_seqlens_q,
                       const int32_t* cu_seqlens_k, int batch, int64_t total_q, int64_t total_k, int num_heads,
                       int num_kv_heads, int head_dim, int max_seqlen_q, int max_seqlen_k, int causal,
                       float softmax_scale, int dtype, int out_dtype, int32_t* error_word, void* stream) {
  fat::set_last_error("");
  fat::PrefillArgs a;
  a.q = q;
  a.q_st = q_stride_t;
  a.q_sh = q_stride_h;
  a.k = k;
  a.k_st = k_stride_t;
  a.k_sh = k_stride_h;
  a.v = v;
  a.v_st = v_stride_t;
  a.v_sh = v_stride_h;
  a.out = out;
  a.o_st = out_stride_t;
  a.o_sh = out_stride_h;
  a.cu_q = cu_seqlens_q;
  a.cu_k = cu_seqlens_k;
  a.batch = batch;
  a.total_q = total_q;
  a.total_k = total_k;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.max_seqlen_q = max_seqlen_q;
  a.max_seqlen_k = max_seqlen_k;
  a.causal = causal;
  a.softmax_scale = softmax_scale;
  a.dtype = dtype;
  a.out_dtype = out_dtype;
  a.error_word = error_word;
  a.stream = static_cast<cudaStream_t>(stream);
  return fat::launch_prefill_varlen(a);
}

int fat_gather_paged(const void* k_cache, const void* v_cache, int64_t stride_page_bytes, int64_t stride_slot_bytes,
                     int64_t stride_head_bytes, int64_t num_pages, const int32_t* page_table,
                     int64_t page_table_stride, int64_t max_pages, const int32_t* seq_lens, void* out_k, void* out_v,
                     int64_t max_len, int batch, int num_kv_heads, int page_size, int64_t row_bytes,
                     int32_t* error_word, void* stream) {
  fat::set_last_error("");
  fat::GatherArgs a;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.sp_bytes = stride_page_bytes;
  a.ss_bytes = stride_slot_bytes;
  a.sh_bytes = stride_head_bytes;
  a.num_pages = num_pages;
  a.page_table = page_table;
  a.pt_sb = page_table_stride;
  a.max_pages = max_pages;
  a.seq_lens = seq_lens;
  a.out_k = out_k;
  a.out_v = out_v;
  a.max_len = max_len;
  a.batch = batch;
  a.num_kv_heads = num_kv_heads;
  a.page_size = page_size;
  a.row_bytes = row_bytes;
  a.error_word = error_word;
  a.stream = static_cast<cudaStream_t>(stream);
  return fat::launch_gather_paged(a);
}

int fat_append_tokens(void* k_cache, void* v_cache, int64_t kv_stride_page, int64_t kv_stride_slot,
                      int64_t kv_stride_head, int64_t num_pages, const int32_t* page_table, int64_t page_table_stride,
                      int64_t max_pages, int32_t* seq_lens, const void* new_k, const void* new_v,
                      int64_t new_stride_b, int64_t new_stride_h, float* k_scale, float* v_scale,
                      int64_t scale_stride_page, int batch, int num_kv_heads, int head_dim, int page_size,
                      int kv_dtype, int new_dtype, int32_t* error_word, void* stream) {
  fat::set_last_error("");
  fat::AppendArgs a;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.kv_sp = kv_stride_page;
  a.kv_ss = kv_stride_slot;
  a.kv_sh = kv_stride_head;
  a.num_pages = num_pages;
  a.page_table = page_table;
  a.pt_sb = page_table_stride;
  a.max_pages = max_pages;
  a.seq_lens = seq_lens;
  a.new_k = new_k;
  a.new_v = new_v;
  a.new_sb = new_stride_b;
  a.new_sh = new_stride_h;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.scale_sp = scale_stride_page;
  a.batch = batch;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.page_size = page_size;
  a.kv_dtype = kv_dtype;
  a.new_dtype = new_dtype;
  a.error_word = error_word;
  a.stream = static_cast<cudaStream_t>(stream);
  return fat::launch_append_tokens(a);
}

int fat_prefill_paged(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k_cache,
                      const void* v_cache, int64_t kv_stride_page, int64_t kv_stride_slot, int64_t kv_stride_head,
                      int64_t num_pages, const int32_t* page_table, int64_t page_table_stride, int64_t max_pages,
                      const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, void* out, int64_t out_stride_t,
                      int64_t out_stride_h, int batch, int64_t total_q, int num_heads, int num_kv_heads,
                      int head_dim, int page_size, int max_seqlen_q, int causal, float softmax_scale, int dtype,
                      int out_dtype, int32_t* error_word, void* stream) {
  fat::set_last_error("");
  fat::PrefillArgs a;
  a.q = q;
  a.q_st = q_stride_t;
  a.q_sh = q_stride_h;
  a.k = k_cache;
  a.v = v_cache;
  a.kv_sp = kv_stride_page;
  a.kv_ss = kv_stride_slot;
  a.kv_sh = kv_stride_head;
  a.num_pages = num_pages;
  a.page_table = page_table;
  a.pt_sb = page_table_stride;
  a.max_pages = max_pages;
  a.cu_q = cu_seqlens_q;
  a.seq_lens_k = seq_lens_k;
  a.out = out;
  a.o_st = out_stride_t;
  a.o_sh = out_stride_h;
  a.batch = batch;
  a.total_q = total_q;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.page_size = page_size;
  a.max_seqlen_q = max_seqlen_q;
  a.causal = causal;
  a.softmax_scale = softmax_scale;
  a.dtype = dtype;
  a.out_dtype = out_dtype;
  a.error_word = error_word;
  a.stream = static_cast<cudaStream_t>(stream);
  return fat::launch_prefill_paged(a);
}


int fat_cache_value_stats(const int32_t* seq_lens, const int32_t* page_table, int64_t page_table_stride, int batch,
                          int64_t max_pages, int page_size, int32_t* device_scratch, int32_t* host_out, void* stream) {
  fat::set_last_error("");
  return fat::cache_value_stats(seq_lens, page_table, page_table_stride, batch, max_pages, page_size, device_scratch,
                                host_out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
