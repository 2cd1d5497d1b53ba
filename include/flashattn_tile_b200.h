/*
 * flashattn_tile_b200 -- C ABI of the B200 (sm_100a) paged-attention library.
 *
 * Every entry point takes raw device pointers, element strides (in elements,
 * the innermost dimension must be contiguous), plain integer sizes and a
 * cudaStream_t passed as void*.  Nothing here allocates device memory except
 * where a function says so; scratch space is passed in by the caller.
 *
 * Each function returns a fat_status.  On failure fat_last_error() holds a
 * message for the calling thread.  Kernels that can detect a problem only on
 * the device (a page id outside the pool, a pipeline wait that timed out)
 * OR a FAT_DEVERR_* bit into the caller's int32 device error word and
 * finish without faulting; the caller reads the word when it wants to know.
 *
 * Reference interface replaced (FlashAttnTile, path:line in that project):
 *   fat_paged_decode          flashattn_tile/ops.py:35-55 (flashattn_tile::paged_decode),
 *                             kernels/decode.py:533-642 (paged_decode_attention),
 *                             kernels/decode.py:645-704 (paged_decode_attention_fp8),
 *                             csrc/paged_decode.cu:297-344 (paged_decode_cuda)
 *   fat_prefill_varlen        flashattn_tile/ops.py:76-99 (flashattn_tile::prefill_varlen),
 *                             kernels/prefill.py:236-326 (prefill_attention)
 *   fat_gather_paged          flashattn_tile/paging.py:213-256 (gather_paged)
 *   fat_lse_merge             kernels/decode.py:316-356 (_decode_reduce_kernel)
 *   fat_prefill_paged         no counterpart: prefill (kernels/prefill.py:34-138 semantics) with
 *                             K/V read through the page table instead of packed tensors
 *                             (the reference's backend requires packed K/V, backend.py:158-162)
 *   fat_append_tokens         flashattn_tile/paging.py:172-210 (append_tokens); for 8-bit
 *                             caches also quant.py:84-142 (per-page scales, applied on write)
 */
#ifndef FLASHATTN_TILE_B200_H_
#define FLASHATTN_TILE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
enum {
  FAT_OK = 0,
  FAT_ERR_INVALID_ARGUMENT = 1, /* shapes, strides, pointers or values are inconsistent */
  FAT_ERR_UNSUPPORTED = 2,      /* a valid request this build has no kernel for       */
  FAT_ERR_CUDA = 3,             /* a CUDA runtime call or kernel launch failed         */
  FAT_ERR_WORKSPACE = 4         /* the scratch buffer passed in is too small           */
};

/* Bits OR-ed into the device error word. */
enum {
  FAT_DEVERR_TIMEOUT = 1,    /* a bounded pipeline wait gave up; the output is invalid  */
  FAT_DEVERR_BAD_PAGE = 2,   /* a page id used by a sequence is outside [0, num_pages) */
  FAT_DEVERR_BAD_LENGTH = 4  /* a sequence length exceeds the page table's capacity
                                (max_pages * page_size); it was cut to that capacity   */
};

/* Element types. */
enum {
  FAT_DTYPE_F16 = 0,
  FAT_DTYPE_BF16 = 1,
  FAT_DTYPE_F32 = 2,
  FAT_DTYPE_I8 = 3,  /* symmetric int8 with per-(page, kv head) fp32 scales */
  FAT_DTYPE_E4M3 = 4 /* float8_e4m3fn with per-(page, kv head) fp32 scales  */
};

/* Library version string, e.g. "flashattn_tile_b200 0.1.0 sm_100a". */
const char* fat_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* fat_last_error(void);

/* Time limit of every bounded wait inside the decode and prefill kernels,
 * for launches made after this call, from any thread (default 2 s; 0 restores
 * it).  A wait that runs out sets FAT_DEVERR_TIMEOUT; the kernel then drains
 * its own copies and tensor-core work and returns.  Returns the previous limit.
 * No reference counterpart: the reference's Triton and CUDA kernels have no
 * in-kernel waits. */
uint64_t fat_set_wait_limit_ns(uint64_t limit_ns);

/* Failure-path testing: each of the next `launches` decode or prefill kernel
 * launches (from any thread) first waits on a barrier phase that nothing
 * completes, so that this wait runs out after the wait limit and the launch
 * ends with FAT_DEVERR_TIMEOUT (no fault, no hang).  0 cancels requests not
 * yet taken.  No reference counterpart. */
void fat_expire_next_waits(int launches);

/* How the prefill kernels feed the probabilities P into the P.V product, for
 * launches made after this call, from any thread.  The reference kernel
 * rounds P to the input dtype once (kernels/prefill.py:128); with bf16's 8-bit
 * significand that alone moves outputs of rows with few keys by up to ~4e-3.
 *   -1  automatic (default): bf16 uses mode 3 (paged K/V: mode 1), fp16 mode 0
 *    0  P rounded to the input dtype once (the reference's arithmetic)
 *    1  a key tile's P enters as a 16-bit head plus a 16-bit remainder (a
 *       second P.V pass over that tile; ~2^-16 relative) when one of its keys
 *       holds more than 1/16 of its row's probability sum so far; every other
 *       key ends with weight <= 1/16, so its rounding moves an output by at
 *       most 2^-12 of |v|
 *    2  head plus remainder on every key tile (twice the P.V work)
 *    3  bf16 with packed K/V: P.V in fp16 -- P rounded to fp16 (~2^-12
 *       relative), V read from an fp16 copy made by a pre-pass (two small
 *       kernels on the call's stream) and scaled by 2^-e per (sequence, KV
 *       head) so that any finite bf16 V fits, the output scaled back by 2^e.
 *       The copy lives in a per-(device, stream) buffer of total_k * kv_heads *
 *       head_dim * 2 bytes, grown on demand and never freed; a stream whose
 *       buffer must grow while it is captured into a graph uses mode 1.  fp16
 *       inputs treat it as mode 0, paged K/V as mode 1
 * Returns the previous setting, or -2 (message in fat_last_error) for a mode
 * outside [-1, 3].  No reference counterpart. */
int fat_set_prefill_p_split(int mode);

/*
 * Grid of the prefill launches made from now on (process-wide; both prefill
 * entry points, all dtypes):
 *    0  persistent (default): one CTA per SM, each claiming (head, sequence,
 *       256-row query pair) items, heaviest first, from a per-stream counter
 *       until none is left, so an item's first loads and Q.K^T overlap the
 *       previous item's last softmax and output stores.  The counter (8 bytes
 *       of device memory per stream) is made on a stream's first prefill; a
 *       stream first used while it is being captured into a graph runs mode 1
 *    1  one CTA per item
 * Results are bitwise identical.  Returns the previous setting, or -2 (message
 * in fat_last_error) for another value.  No reference counterpart. */
int fat_set_prefill_schedule(int mode);

/*
 * Bytes of scratch fat_paged_decode needs for this problem on `device`.
 * The caller zero-fills the buffer once; every successful call leaves it
 * zero-filled again, so one buffer serves any number of calls that are
 * ordered on one stream.
 */
size_t fat_paged_decode_workspace_size(int device, int batch, int num_heads, int num_kv_heads, int head_dim);

/*
 * Single-query paged decode: out[b, h, :] = softmax(scale * q[b, h] . K^T) V over
 * the seq_lens[b] cached tokens of sequence b, K/V read through the page table
 * (token t in page page_table[b, t / page_size], slot t % page_size), query head
 * h reading KV head h / (num_heads / num_kv_heads).
 *
 *   q          [batch, num_heads, head_dim]          q_dtype (F16 | BF16)
 *   k/v_cache  [num_pages, page_size, num_kv_heads, head_dim]
 *              kv_dtype = q_dtype, or I8 / E4M3 with k/v_scale [num_pages, num_kv_heads] fp32
 *   page_table int32 [batch, >= ceil(max seq_len / page_size)]
 *   seq_lens   int32 [batch]; a sequence of length 0 produces zeros
 *   out        [batch, num_heads, head_dim]          out_dtype (= q_dtype, or F32)
 *
 * head_dim in {32, 64, 128, 256}; page_size 8 or a multiple of 16 up to 256; K/V
 * base addresses 16-byte aligned and their page/slot/head strides multiples of
 * 16 bytes.  split_k_hint (1..64) is accepted for interface compatibility: the
 * kernel chooses its own balanced split of the pages over all SMs, and the
 * result does not depend on it.
 */
int fat_paged_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache,
                     const void* v_cache, int64_t kv_stride_page, int64_t kv_stride_slot, int64_t kv_stride_head,
                     int64_t num_pages, const int32_t* page_table, int64_t page_table_stride, int64_t max_pages,
                     const int32_t* seq_lens, const float* k_scale, const float* v_scale,
                     int64_t scale_stride_page, void* out, int64_t out_stride_b, int64_t out_stride_h, int batch,
                     int num_heads, int num_kv_heads, int head_dim, int page_size, int q_dtype, int kv_dtype,
                     int out_dtype, float softmax_scale, int split_k_hint, void* workspace, size_t workspace_bytes,
                     int32_t* error_word, void* stream);

/*
 * fat_paged_decode_lse's arguments in one struct, for callers that keep them
 * between calls (an op whose tensors stay put from step to step pays the
 * argument conversion once and changes only `out`).  With `stats_out` set,
 * the call first queues fat_cache_value_stats(seq_lens, page_table, ...,
 * stats_scratch, stats_out) on the same stream (and records `stats_event`
 * after it), so value checks and decode cost one crossing; `lse` may be NULL.  Same status codes and device error
 * word as fat_paged_decode.  No reference counterpart (a calling convention).
 */
typedef struct fat_decode_call {
  const void* q;
  int64_t q_stride_b, q_stride_h;
  const void* k_cache;
  const void* v_cache;
  int64_t kv_stride_page, kv_stride_slot, kv_stride_head, num_pages;
  const int32_t* page_table;
  int64_t page_table_stride, max_pages;
  const int32_t* seq_lens;
  const float* k_scale;
  const float* v_scale;
  int64_t scale_stride_page;
  void* out;
  int64_t out_stride_b, out_stride_h;
  float* lse;
  int64_t lse_stride_b;
  int32_t batch, num_heads, num_kv_heads, head_dim, page_size;
  int32_t q_dtype, kv_dtype, out_dtype;
  float softmax_scale;
  int32_t split_k_hint;
  void* workspace;
  size_t workspace_bytes;
  int32_t* error_word;
  void* stream;
  int32_t* stats_out;      /* optional: 4 int32 (pinned host or device), see fat_cache_value_stats */
  int32_t* stats_scratch;  /* 4 int32 on the device, used with stats_out */
  void* stats_event;       /* optional cudaEvent_t, recorded on `stream` right after the statistics: a
                              host that waits on it to check the values does not wait for the decode */
} fat_decode_call;

int fat_paged_decode_call(const fat_decode_call* call);

/*
 * fat_paged_decode that also writes, per (sequence, query head), the base-2
 * log-sum-exp of the scaled scores, lse[b * lse_stride_b + h] = m + log2(l)
 * (-inf for a sequence with no cached tokens).  With out_dtype F32 the pair
 * (out, lse) is the partial a sequence-parallel decode exchanges: decode each
 * GPU's own key range (a page-table column slice with per-GPU lengths), gather
 * the partials, combine them with fat_lse_merge.  Replaces the split-K partial
 * outputs of FlashAttnTile's _decode_paged_split_kernel (kernels/decode.py:223-313).
 */
int fat_paged_decode_lse(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache,
                         const void* v_cache, int64_t kv_stride_page, int64_t kv_stride_slot, int64_t kv_stride_head,
                         int64_t num_pages, const int32_t* page_table, int64_t page_table_stride, int64_t max_pages,
                         const int32_t* seq_lens, const float* k_scale, const float* v_scale,
                         int64_t scale_stride_page, void* out, int64_t out_stride_b, int64_t out_stride_h,
                         float* lse, int64_t lse_stride_b, int batch, int num_heads, int num_kv_heads, int head_dim,
                         int page_size, int q_dtype, int kv_dtype, int out_dtype, float softmax_scale,
                         int split_k_hint, void* workspace, size_t workspace_bytes, int32_t* error_word,
                         void* stream);

/*
 * Merge `parts` attention partials over disjoint key ranges:
 *   out[row] = sum_r o[r][row] 2^(lse[r][row] - M) / sum_r 2^(lse[r][row] - M),  M = max_r lse[r][row]
 * o: fp32 [parts][rows][head_dim] (part r at o + r * o_part_stride), lse: fp32 [parts][rows]
 * (part r at lse + r * lse_part_stride), out: [rows][head_dim] of out_dtype (F16 | BF16 | F32),
 * lse_out: optional [rows] merged log-sum-exp.  Rows whose parts are all -inf give zeros.
 * Replaces FlashAttnTile's _decode_reduce_kernel (kernels/decode.py:316-356).
 */
int fat_lse_merge(const float* o, int64_t o_part_stride, const float* lse, int64_t lse_part_stride, int parts,
                  int64_t rows, int head_dim, void* out, int out_dtype, float* lse_out, void* stream);

/*
 * fat_paged_decode for callers that cannot allocate device memory.  No
 * counterpart exists in the reference: it is an addition for engines that
 * allocate every device buffer up front and forbid allocation afterwards,
 * plugins whose host framework gives them neither an allocator nor a scratch
 * pointer, and latency-critical loops where an allocation could synchronise
 * the device.  Same arguments and result as fat_paged_decode, minus the
 * workspace: the split scratch is a fixed 4 MiB array in this library's
 * device memory, held by every GPU that loads the library until the process
 * exits.  Problems whose scratch would exceed 4 MiB (about
 * fat_paged_decode_workspace_size) are refused with FAT_ERR_WORKSPACE.  The
 * first call on a device looks up the array's device address (once per
 * device; make that first call before any stream capture).  Each call clears
 * the tickets it uses on `stream`; all calls share the array, so calls that
 * overlap on the GPU race and must be ordered by the caller.  Allocates
 * nothing (no cudaMalloc / cudaFree).
 */
int fat_paged_decode_noalloc(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache,
                             const void* v_cache, int64_t kv_stride_page, int64_t kv_stride_slot,
                             int64_t kv_stride_head, int64_t num_pages, const int32_t* page_table,
                             int64_t page_table_stride, int64_t max_pages, const int32_t* seq_lens,
                             const float* k_scale, const float* v_scale, int64_t scale_stride_page, void* out,
                             int64_t out_stride_b, int64_t out_stride_h, int batch, int num_heads, int num_kv_heads,
                             int head_dim, int page_size, int q_dtype, int kv_dtype, int out_dtype,
                             float softmax_scale, int split_k_hint, int32_t* error_word, void* stream);

/*
 * Packed varlen prefill: for every sequence b (tokens cu_q[b]..cu_q[b+1] of q and
 * cu_k[b]..cu_k[b+1] of k/v) and query head h,
 *   out = softmax(scale * q k^T [+ bottom-right causal mask]) v,
 * with query i seeing key j when j <= i + kv_len - q_len (causal), query head h
 * reading KV head h / (num_heads / num_kv_heads), P rounded to the input dtype
 * before P.V and fp32 accumulation.
 *
 *   q   [total_q, num_heads, head_dim], k/v [total_k, num_kv_heads, head_dim]   dtype (F16 | BF16)
 *   out [total_q, num_heads, head_dim]   out_dtype (= dtype, or F32)
 *   cu_q, cu_k  int32 [batch + 1], non-decreasing from 0 (not checked on the device)
 *
 * head_dim in {64, 128, 256}; all bases 16-byte aligned, token/head strides multiples
 * of 16 bytes.  max_seqlen_q bounds the launch grid (queries past it are not
 * computed).  Allocates nothing.
 */
int fat_prefill_varlen(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k, int64_t k_stride_t,
                       int64_t k_stride_h, const void* v, int64_t v_stride_t, int64_t v_stride_h, void* out,
                       int64_t out_stride_t, int64_t out_stride_h, const int32_t* cu_seqlens_q,
                       const int32_t* cu_seqlens_k, int batch, int64_t total_q, int64_t total_k, int num_heads,
                       int num_kv_heads, int head_dim, int max_seqlen_q, int max_seqlen_k, int causal,
                       float softmax_scale, int dtype, int out_dtype, int32_t* error_word, void* stream);

/*
 * Prefill / chunked prefill over a paged cache: sequence b has q_len =
 * cu_seqlens_q[b+1] - cu_seqlens_q[b] queries (packed q, as fat_prefill_varlen)
 * that are the last q_len of its seq_lens_k[b] cached tokens; keys and values
 * are those tokens, read from k_cache/v_cache [num_pages, page_size, num_kv_heads,
 * head_dim] through page_table [batch, max_pages] (bottom-right causal alignment:
 * query i sees key j <= i + seq_lens_k[b] - q_len).  fp16/bf16; head_dim 64, 128 or 256 (256: page_size >= 16);
 * page_size a power of two in [8, 128] or a multiple of 128.  Rows past a
 * sequence's end never contribute; a page id outside [0, num_pages) is skipped
 * and ORs FAT_DEVERR_BAD_PAGE into *error_word.
 */
int fat_prefill_paged(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k_cache,
                      const void* v_cache, int64_t kv_stride_page, int64_t kv_stride_slot, int64_t kv_stride_head,
                      int64_t num_pages, const int32_t* page_table, int64_t page_table_stride, int64_t max_pages,
                      const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, void* out, int64_t out_stride_t,
                      int64_t out_stride_h, int batch, int64_t total_q, int num_heads, int num_kv_heads,
                      int head_dim, int page_size, int max_seqlen_q, int causal, float softmax_scale, int dtype,
                      int out_dtype, int32_t* error_word, void* stream);

/*
 * Append one token per sequence: new_k/new_v [batch, num_kv_heads, head_dim]
 * (element strides new_stride_b, new_stride_h; unit stride along head_dim) go to
 * page page_table[b, seq_lens[b] / page_size], slot seq_lens[b] % page_size, then
 * seq_lens[b] += 1 -- all on the device, no host synchronisation.  A position past
 * the page table or a page id outside [0, num_pages) leaves that sequence untouched
 * and ORs FAT_DEVERR_BAD_PAGE into *error_word.
 *   16-bit caches: new_dtype == kv_dtype, bit-exact copy; k_scale/v_scale unused.
 *   INT8 / FP8-e4m3 caches: new_dtype F16 | BF16 | F32; the page's fp32 scale
 *   (k_scale/v_scale [num_pages, num_kv_heads], stride scale_stride_page) becomes
 *   max(absmax / maxval, 1e-8) over this sequence's tokens on the page (earlier ones
 *   dequantised as code * scale) and the new token; earlier codes are requantised
 *   when the scale changed; the new token is quantised with it (int8: round half to
 *   even, clamp +-127; e4m3: clamp +-448, round to nearest even).
 */
int fat_append_tokens(void* k_cache, void* v_cache, int64_t kv_stride_page, int64_t kv_stride_slot,
                      int64_t kv_stride_head, int64_t num_pages, const int32_t* page_table, int64_t page_table_stride,
                      int64_t max_pages, int32_t* seq_lens, const void* new_k, const void* new_v,
                      int64_t new_stride_b, int64_t new_stride_h, float* k_scale, float* v_scale,
                      int64_t scale_stride_page, int batch, int num_kv_heads, int head_dim, int page_size,
                      int kv_dtype, int new_dtype, int32_t* error_word, void* stream);

/*
 * Page-table gather: out_k/out_v [batch, max_len, num_kv_heads, row_bytes] (contiguous)
 * receive, bit for bit, the rows of each sequence's first seq_lens[b] tokens, and
 * zeros past that.  The cache is addressed by byte strides (page, slot, head); the
 * element type does not matter (row_bytes = head_dim * element size).
 */
int fat_gather_paged(const void* k_cache, const void* v_cache, int64_t stride_page_bytes, int64_t stride_slot_bytes,
                     int64_t stride_head_bytes, int64_t num_pages, const int32_t* page_table,
                     int64_t page_table_stride, int64_t max_pages, const int32_t* seq_lens, void* out_k, void* out_v,
                     int64_t max_len, int batch, int num_kv_heads, int page_size, int64_t row_bytes,
                     int32_t* error_word, void* stream);

/*
 * Value statistics of a paged cache's metadata, for the host-side checks of
 * flashattn_tile/paging.py:84-130 (validate_cache): host_out[0..3] = min and max
 * of seq_lens[batch], then min and max of the page-table entries a sequence of
 * the maximum length reaches (the first ceil(max / page_size) columns of every
 * row, at most max_pages; (0, -1) when there are none).  Queues one kernel on
 * `stream`: when host_out is pinned host memory mapped into the device's
 * address space (cudaHostAlloc / cudaHostRegister memory, 16-byte aligned) the
 * kernel writes it directly, otherwise it writes device_scratch and a 16-byte
 * copy into host_out follows.  Synchronise the stream (or an event recorded
 * after this call) before reading host_out.  device_scratch: 4 int32 on the
 * device (unused when host_out is written directly).  Replaces
 * the reference's torch reductions + read-back of both tensors.
 */
int fat_cache_value_stats(const int32_t* seq_lens, const int32_t* page_table, int64_t page_table_stride, int batch,
                          int64_t max_pages, int page_size, int32_t* device_scratch, int32_t* host_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHATTN_TILE_B200_H_ */
