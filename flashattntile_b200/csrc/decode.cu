// Single-query paged decode for sm_100a.
//
// Replaces FlashAttnTile's decode family (flashattn_tile/kernels/decode.py:46-447:
// plain, GQA-grouped, split-K + LSE reduce, and INT8/FP8 kernels) with one
// persistent kernel:
//
// * Work is flattened into 64-token chunks of (sequence, KV head, head group)
//   units and split evenly over one CTA per SM.  Every CTA derives the same
//   split from seq_lens on the device (no host sync, no tuning): each CTA
//   owns a contiguous range of chunks, so the split adapts to ragged batches.
//   A unit split across CTAs is merged by a log-sum-exp combine done by the
//   last CTA that finishes a piece of it (an atomic ticket per unit); the
//   math is decode.py:12-14 / 341-352 in base 2.  A dedicated merge warp
//   does each piece's global epilogue (output rows, or the partial, ticket
//   and combine), so its L2 round trips overlap the next chunks' math.
// * Two producer warps take turns by chunk: each walks the CTA's chunks,
//   prefetches page ids (and 8-bit scales) through a cp.async ring, and issues
//   one 5-D TMA copy per (row box, K|V) -- whole token rows of one KV head,
//   128-byte swizzled -- into a ring of shared-memory stages guarded by
//   mbarriers.  Each K/V byte is read from HBM once per GQA group, not once per
//   query head.
// * Four consumer warps take 16 tokens each per stage.  Scores and P.V run on
//   the tensor cores (mma.sync m16n8k16, fp32 accumulate) with the group's
//   query heads as the M rows; P enters the P.V product as a 16-bit head plus
//   a 16-bit remainder in the otherwise unused rows 8-15, so the probabilities
//   keep ~fp32 precision, as in the reference's fp32 p.v (decode.py:120).
//   Online softmax state lives in registers; row maxima use quad shuffles.
// * INT8 / e4m3 caches are dequantised in registers: codes are widened to the
//   query's 16-bit type (exact) and the per-(page, KV head) scales are folded
//   into the score (K) and into p (V), as in decode.py:408-439.
//
// Every mbarrier wait is bounded; on a timeout the kernel records
// FAT_DEVERR_TIMEOUT, drains its own TMA copies and returns.
#include <math_constants.h>

#include <algorithm>

#include <type_traits>

#include "common.cuh"
#include "decode.h"
#include "host_util.h"

namespace fat {
namespace dec {

constexpr int kProducers = 2;              // producer warps (take turns by chunk)
constexpr int kMaxChunk = 256;             // largest chunk (tokens per pipeline stage) of any layout
constexpr int kMaxTokens = 1 << 30;        // longest sequence the kernel walks (positions stay far below 2^31)
constexpr int kMaxBoxes = 32;              // TMA row boxes per chunk at most (chunk / 8)
constexpr int kRows = 8;                   // query heads per unit (M rows 0-7; 8-15 carry P remainders)
constexpr size_t kSmemMax = 227 * 1024;    // shared memory per CTA (opt-in maximum)
constexpr float kDecodeRescaleLog2 = 8.f;  // running-max slack before O is rescaled (P <= 2^8)

enum : int { kFirst = 1, kLast = 2, kFull = 4, kDone = 8 };

// Producer lookahead: page ids are fetched kPF chunks ahead of the stage being
// filled and 8-bit scales kPF2 chunks ahead, through a ring of kRing slots.
constexpr int kPF = 6;
constexpr int kPF2 = 3;
constexpr int kRing = 8;
static_assert(kRing > kPF && kPF > kPF2 && kPF2 > 0, "prefetch ring too small");

struct RingInfo {
  int b, unit_local, chunk, len, chunks_b, nbox;
  long long S;
};
// Per-producer prefetch ring: unit info, page ids and (8-bit caches) the pages' K/V scales.
constexpr int ring_bytes(int eb) { return kRing * int(sizeof(RingInfo)) + kRing * kMaxBoxes * 4 * (eb == 1 ? 3 : 1); }

// Per-stage metadata; the per-8-token scales exist for 8-bit caches only.
template <int EB>
struct alignas(16) MetaT {
  int flags;
  int b;
  int unit_local;  // kv_head * head_groups + head_group
  int chunk;       // chunk index inside the unit
  int seq_len;
  int chunks_b;    // chunks per unit of this sequence
  long long unit_base;  // flattened index of the unit's first chunk
  float kscale[EB == 1 ? kMaxChunk / 8 : 1];
  float vscale[EB == 1 ? kMaxChunk / 8 : 1];
};

// A finished piece, handed from the consumer warps to the merge warp.
struct MergeEvent {
  int flags;
  int b;
  int unit_local;
  int chunks_b;
  long long unit_base;
  long long pad;
};

struct Params {
  const void* q;
  long long q_sb, q_sh;
  void* out;
  long long o_sb, o_sh;
  const int* page_table;
  long long pt_sb;
  const int* seq_lens;
  const float* k_scale;
  const float* v_scale;
  long long s_sp;  // scale stride per page (head stride 1)
  int batch, num_heads, num_kv_heads, group, head_groups, page_size, num_pages, box_rows, max_pages;
  int cap_tokens;  // min(max_pages * page_size, kMaxTokens): every length is cut to this
  float scale_log2;
  int out_f32;
  float* lse;    // optional [batch][num_heads] (stride lse_sb): m + log2(l), base-2 log-sum-exp
  long long lse_sb;
  float* ws_o;   // [grid][2][kRows][D]
  float* ws_ml;  // [grid][2][kRows][2]
  int* ws_count; // [units]
  int* err;
  unsigned long long wait_ns;  // limit of every bounded wait
  int expire;    // consumer warp 0 first waits on a barrier phase nothing completes (failure-path tests)
};

template <int D, int EB>
struct Layout {
  static constexpr int kRowBytes = D * EB;                         // one token row of one KV head
  static constexpr int kBoxBytes = kRowBytes >= 128 ? 128 : kRowBytes;  // TMA box row
  static constexpr int kCB = kRowBytes / kBoxBytes;                // column boxes per row
  // Consumer warps: 8-bit caches carry twice the tokens per byte and widen
  // every code before the MMA, so they get twice the math warps.
  static constexpr int kWarps = (EB == 1 && D <= 128) ? 8 : 4;
  static constexpr int kMergeWarp = kWarps + kProducers;           // warp index of the merge warp
  static constexpr int kThreads = (kWarps + kProducers + 1) * 32;
  // Tokens per consumer warp per stage: stages stay 32 KB (K + V) for narrow rows.
  static constexpr int kTW = (kRowBytes >= 256 ? 16 : (kRowBytes >= 128 ? 32 : 64)) * 4 / kWarps;
  static_assert(kTW % 16 == 0, "a consumer warp takes whole 16-token MMA slices");
  static constexpr int kChunk = kWarps * kTW;                      // tokens per pipeline stage
  static_assert(kChunk <= kMaxChunk, "chunk larger than the per-stage metadata");
  static constexpr int kTile = kChunk * kRowBytes;                 // K (or V) bytes per stage
  static constexpr int kStage = 2 * kTile;
  static constexpr int kQBytes = kRows * D * 2;
  static constexpr int kMergeFloats = kWarps * kRows * (D + 8) + 2 * kWarps * kRows;
  static constexpr int kRingBytes = ring_bytes(EB);
  using Meta = MetaT<EB>;
  // As many stages (up to 8) as shared memory holds: bytes in flight per SM
  // set the streaming rate (5 -> 4 stages of 32 KB cost 3.5% at cfg2).  The
  // prologue's scan buffer lives in the (then idle) first stage.
  static constexpr size_t kFixed = 1024 /*align slack*/ + size_t(kMergeFloats) * 4 + 2 * 8 /*merge barriers*/ +
                                   64 + sizeof(MergeEvent) + size_t(kProducers) * kRingBytes + 16;
  static constexpr size_t kPerStage = size_t(kStage) + kQBytes + sizeof(Meta) + 2 * 8 /*full, empty*/;
  static constexpr int kStages = (kSmemMax - kFixed) / kPerStage > 8 ? 8 : int((kSmemMax - kFixed) / kPerStage);
  static_assert(kStages >= 2, "decode stage ring needs two stages");
  static_assert(size_t(kThreads + kThreads / 32) * 8 <= size_t(kStage), "prologue scan must fit in one stage");
  static constexpr size_t kSmem = kFixed + size_t(kStages) * kPerStage;

  // Shared address of byte column `bc` (16-byte aligned part) of token row `row`
  // of a tile stored as [row][kCB column blocks][128 B]: with the 128-byte
  // swizzle, 16-byte chunk c of 128-byte segment g (g = row * kCB + block)
  // sits at chunk position c ^ (g & 7).
  static __device__ __forceinline__ uint32_t addr(uint32_t tile, int row, int bc) {
    if constexpr (kBoxBytes == 128) {
      const uint32_t seg = uint32_t(row * kCB + (bc >> 7));
      return tile + seg * 128u + ((uint32_t((bc & 127) >> 4) ^ (seg & 7u)) << 4) + uint32_t(bc & 15);
    } else {
      return tile + uint32_t(row * kBoxBytes + bc);
    }
  }
};

__device__ __forceinline__ long long range_start(long long c, long long total, int nc) { return c * total / nc; }

// The balanced split of `total` chunks over `nc` CTAs: CTA c owns
// [start(c), start(c + 1)) and chunk x belongs to owner(x).  32-bit
// arithmetic whenever the products fit (64-bit division is emulated).
struct Split {
  long long total;
  int nc;
  bool narrow;
  __device__ Split(long long t, int n) : total(t), nc(n), narrow((t + 1) * (n + 32) < (1ll << 32)) {}
  // c <= nc + 31
  __device__ __forceinline__ long long start(int c) const {
    return narrow ? (long long)(uint32_t(c) * uint32_t(total) / uint32_t(nc)) : (long long)c * total / nc;
  }
  // 0 <= x < total
  __device__ __forceinline__ int owner(long long x) const {
    return narrow ? int((uint32_t(x + 1) * uint32_t(nc) - 1u) / uint32_t(total)) : int(((x + 1) * nc - 1) / total);
  }
};

// Cached tokens of sequence b as the kernel walks them: a negative length
// counts as 0, a length past the page table (max_pages * page_size, at most
// kMaxTokens) is cut to it, so no token position, chunk count or page index
// derived from it can overflow 32 bits or leave the table.  The cut is
// reported (FAT_DEVERR_BAD_LENGTH) once per sequence by the zero-row pass.
__device__ __forceinline__ int seq_len_of(const Params& p, int b) {
  return min(max(__ldg(p.seq_lens + b), 0), p.cap_tokens);
}

// ---------------------------------------------------------------------------
// 8-bit KV codes -> 16-bit MMA operands, exactly (every int8 and every finite
// e4m3 value is representable in fp16 and in bf16).  widen4 turns the four
// bytes of a word into the pairs (byte0, byte1) and (byte2, byte3).
// ---------------------------------------------------------------------------
template <typename T, int KVT>
struct Widen;

// int8 -> fp16: with u = x + 128, the fp16 bit pattern 0x6400 | u is 1024 + u,
// so subtracting 1152 leaves x.
template <>
struct Widen<__half, FAT_DTYPE_I8> {
  static __device__ __forceinline__ void run(uint32_t w, uint32_t& p01, uint32_t& p23) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t a = __byte_perm(u, 0x64646464u, 0x4140);
    const uint32_t b = __byte_perm(u, 0x64646464u, 0x4342);
    const uint32_t magic = 0x64806480u;
    asm("sub.f16x2 %0, %1, %2;" : "=r"(p01) : "r"(a), "r"(magic));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(p23) : "r"(b), "r"(magic));
  }
};

// int8 -> bf16: with u = x + 128, the fp32 bit pattern 0x4B000000 | u is
// 2^23 + u; subtracting 2^23 + 128 leaves x, which bf16 holds exactly.
template <>
struct Widen<__nv_bfloat16, FAT_DTYPE_I8> {
  static __device__ __forceinline__ void run(uint32_t w, uint32_t& p01, uint32_t& p23) {
    const uint32_t u = w ^ 0x80808080u;
    const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.f;
    const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.f;
    const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.f;
    const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.f;
    p01 = pack2<__nv_bfloat16>(f0, f1);
    p23 = pack2<__nv_bfloat16>(f2, f3);
  }
};

// e4m3 -> fp16 with the hardware pair conversion.
template <>
struct Widen<__half, FAT_DTYPE_E4M3> {
  static __device__ __forceinline__ void run(uint32_t w, uint32_t& p01, uint32_t& p23) {
    const uint16_t lo = static_cast<uint16_t>(w & 0xffffu);
    const uint16_t hi = static_cast<uint16_t>(w >> 16);
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(p01) : "h"(lo));
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(p23) : "h"(hi));
  }
};

// e4m3 -> bf16: placing the code's exponent/mantissa bits (eeee mmm) at bf16
// bits 10..4 gives 2^(e-127) * 1.mmm (or the matching subnormal); one exact
// multiply by 2^120 rebiases it to 2^(e-7) * 1.mmm.
template <>
struct Widen<__nv_bfloat16, FAT_DTYPE_E4M3> {
  static __device__ __forceinline__ uint32_t pair(uint32_t two) {
    const uint32_t r = ((two & 0x00800080u) << 8) | ((two & 0x007F007Fu) << 4);
    uint32_t out;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(out) : "r"(r), "r"(0x7B807B80u));
    return out;
  }
  static __device__ __forceinline__ void run(uint32_t w, uint32_t& p01, uint32_t& p23) {
    p01 = pair(__byte_perm(w, 0u, 0x4140));
    p23 = pair(__byte_perm(w, 0u, 0x4342));
  }
};

// int8 codes -> fp16 with a +1152 bias, for fp16 queries: the fp16 bit
// pattern 0x6400 | (x + 128) is exactly 1152 + x, so dropping the subtraction
// of the exact widening leaves the byte placement only.  The bias comes back
// out per row: 1152 * sum(q) from every score and 1152 * sum(p) from every
// output column (both sums taken in fp32 as the MMAs see their operands).
constexpr float kI8Bias = 1152.f;

// Bytes 0-3 of w -> biased pairs (b0, b1) and (b2, b3).
__device__ __forceinline__ void widen_i8_biased(uint32_t w, uint32_t& p01, uint32_t& p23) {
  const uint32_t u = w ^ 0x80808080u;
  p01 = __byte_perm(u, 0x64646464u, 0x4140);
  p23 = __byte_perm(u, 0x64646464u, 0x4342);
}

// Bytes 0 and 2 of x -> the biased pair (b0, b2): (x & 0x00FF00FF) ^ 0x64806480
// in one LOP3 (bytes 1 and 3 of x are ignored).
__device__ __forceinline__ uint32_t biased_pair_i8(uint32_t x) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(x), "r"(0x00FF00FFu), "r"(0x64806480u));
  return r;
}

template <int KVT>
constexpr int elem_bytes() {
  return (KVT == FAT_DTYPE_I8 || KVT == FAT_DTYPE_E4M3) ? 1 : 2;
}

template <typename T, int D, int KVT>
__global__ void __launch_bounds__(Layout<D, elem_bytes<KVT>()>::kThreads, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const Params p) {
  constexpr int EB = elem_bytes<KVT>();
  using L = Layout<D, EB>;
  constexpr int kWarps = L::kWarps;
  constexpr int kThreads = L::kThreads;
  constexpr int kStages = L::kStages;
  constexpr int kChunk = L::kChunk;
  constexpr int kTW = L::kTW;
  constexpr int NT = D / 8;  // n-tiles of the output
  // 8-bit caches compute in fp16 whatever the query type: codes widen to fp16
  // exactly (int8 with a bias, e4m3 by conversion), and a bf16 query row is
  // brought into fp16 exactly by a power-of-two scale (kQConv, below).
  using Tc = typename std::conditional<EB == 1, __half, T>::type;
  constexpr bool kQConv = EB == 1 && !std::is_same<T, __half>::value;
  constexpr bool kBias = KVT == FAT_DTYPE_I8;  // biased int8 widening

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  T* qarea = reinterpret_cast<T*>(smem + size_t(kStages) * L::kStage);
  using Meta = typename L::Meta;
  Meta* meta = reinterpret_cast<Meta*>(reinterpret_cast<uint8_t*>(qarea) + size_t(kStages) * L::kQBytes);
  float* mO = reinterpret_cast<float*>(meta + kStages);
  float* mM = mO + kWarps * kRows * (D + 8);
  float* mL = mM + kWarps * kRows;
  uint64_t* bars = reinterpret_cast<uint64_t*>(mL + kWarps * kRows);
  volatile int* shi = reinterpret_cast<volatile int*>(bars + 2 * kStages + 2);  // [0] abort, [2..3] `never`
  long long* shl = reinterpret_cast<long long*>(const_cast<int*>(shi) + 4);   // [0] start_b [1] start_S [2] total
  volatile MergeEvent* evt = reinterpret_cast<volatile MergeEvent*>(shl + 4);
  long long* scan = reinterpret_cast<long long*>(stages);  // [kThreads + kThreads / 32], prologue only
  uint8_t* ring_base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(const_cast<MergeEvent*>(evt) + 1) + 15) & ~uintptr_t(15));  // producer prefetch ring

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8u * kStages;
  const uint32_t mfull = full0 + 16u * kStages;  // consumer warps -> merge warp: a piece is in the merge area
  const uint32_t mfree = mfull + 8u;             // merge warp -> consumer warps: the merge area is free
  const uint32_t never = smem_u32(const_cast<int*>(shi) + 2);  // initialised, never arrived on
  const int nkg = p.num_kv_heads * p.head_groups;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, kWarps);
    }
    mbar_init(mfull, kWarps * 32);
    mbar_init(mfree, 1);
    mbar_init(never, 1);
    shi[0] = 0;
    shl[0] = -1;
    fence_barrier_init();
  }

  // ---- every CTA derives the same balanced split of all chunks -------------
  {
    const int per = (p.batch + kThreads - 1) / kThreads;
    const int b0 = tid * per;
    const int b1 = min(p.batch, b0 + per);
    long long mine = 0;
    for (int b = b0; b < b1; ++b) mine += (seq_len_of(p, b) + kChunk - 1) / kChunk;
    // Exclusive prefix sum of `mine` over the block: warp scans, then a scan
    // of the warp totals by warp 0 (a serial loop here cost microseconds).
    long long* wsum = scan + kThreads;  // [kThreads / 32]
    long long v = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    if (lane == 31) wsum[warp] = v;
    __syncthreads();
    if (warp == 0) {
      long long w = lane < kThreads / 32 ? wsum[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += n;
      }
      if (lane < kThreads / 32) wsum[lane] = w;  // inclusive totals
      if (lane == kThreads / 32 - 1) shl[2] = w;
    }
    __syncthreads();
    scan[tid] = v - mine + (warp > 0 ? wsum[warp - 1] : 0);
    __syncthreads();
    const long long total = shl[2] * nkg;
    const long long x0 = range_start(blockIdx.x, total, gridDim.x);
    const long long pre = scan[tid] * nkg;
    if (x0 < total && pre <= x0 && x0 < pre + mine * nkg) {
      long long s = scan[tid];
      for (int b = b0; b < b1; ++b) {
        const long long cb = (seq_len_of(p, b) + kChunk - 1) / kChunk;
        if (x0 < (s + cb) * nkg) {
          shl[0] = b;
          shl[1] = s;
          break;
        }
        s += cb;
      }
    }
    __syncthreads();
  }
  const long long total = shl[2] * nkg;
  const long long x0 = range_start(blockIdx.x, total, gridDim.x);
  const long long x1 = range_start(blockIdx.x + 1, total, gridDim.x);
  volatile int* abort_flag = shi;

  // Sequences without cached tokens own no chunks: their output rows are zero.
  for (int b = blockIdx.x; b < p.batch; b += gridDim.x) {
    const int raw_len = __ldg(p.seq_lens + b);
    if (raw_len > p.cap_tokens && tid == 0) raise_error(p.err, FAT_DEVERR_BAD_LENGTH);
    if (raw_len > 0) continue;
    for (int idx = tid; idx < p.num_heads * D; idx += kThreads) {
      const int h = idx / D, d = idx - h * D;
      const long long off = (long long)b * p.o_sb + (long long)h * p.o_sh + d;
      if (p.out_f32) {
        reinterpret_cast<float*>(p.out)[off] = 0.f;
      } else {
        reinterpret_cast<T*>(p.out)[off] = from_float<T>(0.f);
      }
      if (p.lse != nullptr && d == 0) p.lse[(long long)b * p.lse_sb + h] = -CUDART_INF_F;
    }
  }

  if (warp >= kWarps && warp < L::kMergeWarp) {
    // ======================= producer warps =======================
    // kProducers warps take turns: producer `pid` fills the stages of chunks
    // pid, pid + kProducers, ... of this CTA's range, so the per-chunk
    // bookkeeping of one warp overlaps with the others' TMA traffic.
    const int pid = warp - kWarps;
    // K/V bytes are read once: evict-first keeps the 0.5-4 GB stream from
    // churning L2 (+3% at cfg2 over the default policy).
    const uint64_t kv_policy = policy_evict_first();
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
    }
    // The walk over this CTA's chunks runs kPF own chunks ahead of the stage
    // being filled: for each future chunk it records the unit info in a small
    // shared ring and starts cp.async copies of its page ids (and, for 8-bit
    // caches, kPF2 chunks ahead, of the pages' scales), so the TMA issue for
    // a stage never waits on a dependent global load.
    const int n = int(x1 - x0);  // chunks of this CTA (fits in 32 bits)
    const int n_own = n > pid ? (n - pid + kProducers - 1) / kProducers : 0;
    int own_issued = 0;
    RingInfo* rinfo = reinterpret_cast<RingInfo*>(ring_base + pid * L::kRingBytes);
    int* rids = reinterpret_cast<int*>(rinfo + kRing);
    float* rks = reinterpret_cast<float*>(rids + kRing * kMaxBoxes);
    float* rvs = rks + kRing * kMaxBoxes;
    if (n_own > 0) {
      // The walk keeps (sequence, unit, chunk) incrementally, so the loop does
      // no 64-bit division (emulated and slow on the GPU).
      int wb = int(shl[0]);
      long long wS = shl[1];
      int wlen = seq_len_of(p, wb);
      int wchunks = (wlen + kChunk - 1) / kChunk;
      int wunit, wchunk;
      {
        const long long pos = x0 - wS * nkg;
        wunit = int(pos / wchunks);
        wchunk = int(pos - (long long)wunit * wchunks);
      }
      int wi = 0;  // chunk (relative to x0) the walk points at
      auto advance = [&]() {
        ++wi;
        if (++wchunk == wchunks) {
          wchunk = 0;
          if (++wunit == nkg && wi < n) {
            wunit = 0;
            wS += wchunks;
            do {
              ++wb;
              wlen = seq_len_of(p, wb);
              wchunks = (wlen + kChunk - 1) / kChunk;
            } while (wchunks == 0 && wb + 1 < p.batch);
          }
        }
      };
      for (int k = 0; k < pid && wi < n; ++k) advance();
      int jl = 0;  // next own chunk whose ids are fetched
      auto prefetch_ids = [&]() {
        if (jl < n_own) {
          const int r = jl & (kRing - 1);
          const int unit_local = wunit;
          const int chunk = wchunk;
          const int tok0 = chunk * kChunk;
          const int nbox = (min(kChunk, wlen - tok0) + p.box_rows - 1) / p.box_rows;
          if (lane == 0) {
            rinfo[r].b = wb;
            rinfo[r].unit_local = unit_local;
            rinfo[r].chunk = chunk;
            rinfo[r].len = wlen;
            rinfo[r].chunks_b = wchunks;
            rinfo[r].nbox = nbox;
            rinfo[r].S = wS;
          }
          if (lane < nbox) {
            const int lp = (tok0 + lane * p.box_rows) / p.page_size;
            int* dst = rids + r * kMaxBoxes + lane;
            if (lp >= 0 && lp < p.max_pages) {
              cp_async_4(smem_u32(dst), p.page_table + (long long)wb * p.pt_sb + lp);
            } else {
              *dst = -1;
            }
          }
          ++jl;
          for (int k = 0; k < kProducers && wi < n; ++k) advance();
        }
        cp_async_commit();
      };
      // Scales of own chunk j (its page ids must have landed): 8-bit caches only.
      auto prefetch_scales = [&](int j) {
        if constexpr (EB == 1) {
          if (j >= 0 && j < n_own) {
            const int r = j & (kRing - 1);
            const int nbox = rinfo[r].nbox;
            const int kvh = rinfo[r].unit_local / p.head_groups;
            if (lane < nbox) {
              const int ph = rids[r * kMaxBoxes + lane];
              if (ph >= 0 && ph < p.num_pages) {
                cp_async_4(smem_u32(rks + r * kMaxBoxes + lane), p.k_scale + (long long)ph * p.s_sp + kvh);
                cp_async_4(smem_u32(rvs + r * kMaxBoxes + lane), p.v_scale + (long long)ph * p.s_sp + kvh);
              }
            }
          }
        }
        cp_async_commit();
      };
      // Step k commits two groups: page ids of own chunk k, then scales of own
      // chunk k-(kPF-kPF2) (empty for 16-bit caches).  Before issuing the
      // scales of chunk y we need y's ids: 2*(kPF-kPF2) groups were committed
      // after them.  Before filling the stage of own chunk j (step j+kPF) we
      // need j's scales: 2*kPF2 groups were committed after them.
      auto step = [&](int k) {
        prefetch_ids();
        cp_async_wait<2 * (kPF - kPF2)>();
        __syncwarp();
        prefetch_scales(k - (kPF - kPF2));
      };
      for (int k = 0; k < kPF; ++k) step(k);
      for (int j = 0; j < n_own; ++j) {
        const int i = pid + j * kProducers;  // chunk index within the CTA's range
        step(j + kPF);
        cp_async_wait<2 * kPF2>();
        __syncwarp();
        const int r = j & (kRing - 1);
        const int b = rinfo[r].b, unit_local = rinfo[r].unit_local, chunk = rinfo[r].chunk;
        const int len = rinfo[r].len, chunks_b = rinfo[r].chunks_b, nbox = rinfo[r].nbox;
        const long long S = rinfo[r].S;
        const bool first = (i == 0) || chunk == 0;
        const bool last = (i == n - 1) || chunk == chunks_b - 1;
        // The CTA covers the whole unit iff its first and last chunks are in range.
        const bool full_seg = (i - chunk >= 0) && (i - chunk + chunks_b <= n);
        const int s = i % kStages;
        const uint32_t parity = uint32_t(((i / kStages) & 1) ^ 1);
        if (!mbar_wait_bounded(empty0 + 8u * s, parity, p.err, abort_flag, p.wait_ns)) break;

        const int kvh = unit_local / p.head_groups;
        const int hg = unit_local - kvh * p.head_groups;
        const int tok0 = chunk * kChunk;
        int phys = -1;
        if (lane < nbox) {
          phys = rids[r * kMaxBoxes + lane];
          if (phys < 0 || phys >= p.num_pages) {
            raise_error(p.err, FAT_DEVERR_BAD_PAGE);
            phys = -1;
          }
        }
        const unsigned okmask = __ballot_sync(0xffffffffu, phys >= 0);
        Meta& mt = meta[s];
        if constexpr (EB == 1) {
          // One scale pair per 8-token group of the chunk; groups past the
          // sequence end (or on a rejected page) get 0 so that masked tokens
          // never meet stale shared memory.
          const float ksc = phys >= 0 ? rks[r * kMaxBoxes + lane] : 0.f;
          const float vsc = phys >= 0 ? rvs[r * kMaxBoxes + lane] : 0.f;
          const int per8 = p.box_rows / 8;  // 8-token groups per box
          const int src = lane / per8;
          const float kg = __shfl_sync(0xffffffffu, ksc, src);
          const float vg = __shfl_sync(0xffffffffu, vsc, src);
          if (lane < kChunk / 8) {
            mt.kscale[lane] = kg;
            mt.vscale[lane] = vg;
          }
        }
        // The copies go out first (their bytes are expected before any can
        // land); the query rows and the stage metadata are written meanwhile,
        // and the producer's arrival after them publishes the stage.
        const uint32_t bytes = uint32_t(__popc(okmask)) * uint32_t(p.box_rows) * uint32_t(L::kRowBytes) * 2u;
        const uint32_t fb = full0 + 8u * s;
        if (lane == 0) mbar_expect_tx(fb, bytes);
        __syncwarp();
        // One TMA copy per (row box, K|V): the box spans every 128-byte column
        // block of its rows (5-D map), landing as [rows][row bytes] in the stage.
        const uint32_t st = smem_u32(stages) + uint32_t(s) * L::kStage;
        for (int j0 = 0; j0 < 2 * nbox; j0 += 32) {
          const int j = j0 + lane;
          const int box = j >> 1, tensor = j & 1;
          const int ph = __shfl_sync(0xffffffffu, phys, box & 31);
          if (j < 2 * nbox && ph >= 0) {
            const int t = tok0 + box * p.box_rows;
            const uint32_t dst = st + uint32_t(tensor) * L::kTile + uint32_t(box * p.box_rows * L::kRowBytes);
            tma_load_5d_hint(dst, tensor ? &tm_v : &tm_k, fb, 0, 0, kvh, t % p.page_size, ph, kv_policy);
          }
        }
        if (first) {
          // Query rows of this head group -> qarea[s] (zero rows past the group).
          const int rows = min(kRows, p.group - hg * kRows);
          const int h0 = kvh * p.group + hg * kRows;
          constexpr int kVec = D * 2 / 16;  // 16-byte vectors per row
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(qarea) + size_t(s) * L::kQBytes);
          for (int i = lane; i < kRows * kVec; i += 32) {
            const int r = i / kVec, v = i - r * kVec;
            uint4 val = make_uint4(0, 0, 0, 0);
            if (r < rows) {
              const T* src = reinterpret_cast<const T*>(p.q) + (long long)b * p.q_sb + (long long)(h0 + r) * p.q_sh;
              val = __ldg(reinterpret_cast<const uint4*>(src) + v);
            }
            dst[i] = val;
          }
        }
        if (lane == 0) {
          mt.flags = (first ? kFirst : 0) | (last ? kLast : 0) | (full_seg ? kFull : 0);
          mt.b = b;
          mt.unit_local = unit_local;
          mt.chunk = chunk;
          mt.seq_len = len;
          mt.chunks_b = chunks_b;
          mt.unit_base = S * nkg + (long long)unit_local * chunks_b;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(fb);
        ++own_issued;
      }
    }
    cp_async_wait<0>();
    // Termination marker, written by the producer that owns slot n (or, after
    // an abort, drain this producer's own copies).
    if (!*abort_flag && n % kProducers == pid) {
      const int s = n % kStages;
      const uint32_t parity = uint32_t(((n / kStages) & 1) ^ 1);
      if (mbar_wait_bounded(empty0 + 8u * s, parity, p.err, abort_flag, p.wait_ns)) {
        if (lane == 0) {
          meta[s].flags = kDone;
          mbar_arrive(full0 + 8u * s);
        }
      }
    }
    if (*abort_flag && lane == 0) {
      for (int j = max(0, own_issued - kStages); j < own_issued; ++j) {
        const int i = pid + j * kProducers;
        mbar_wait_bounded(full0 + 8u * (i % kStages), uint32_t((i / kStages) & 1), nullptr, nullptr, p.wait_ns);
      }
    }
    return;
  }

  if (warp == L::kMergeWarp) {
    // ======================= merge warp =======================
    // For each finished piece: fold the consumer warps' partials (merge area)
    // into registers, free the area, then write the output rows of a unit
    // this CTA covered whole -- or, for a unit split across CTAs, write the
    // piece's partial (o, m, l) to its workspace slot and, if it is the last
    // piece to arrive, combine all pieces of the unit in CTA order (the same
    // arithmetic whichever CTA arrives last, so results are deterministic).
    constexpr int VE = D / 32;                 // output columns per lane: d = j * 32 + lane
    constexpr int kPair = (D <= 128 && EB == 2) ? 2 : 1;  // workspace pieces loaded per round trip
    const auto store_rows = [&](int b, int h0, int rows, const float (&M)[kRows], const float (&Ls)[kRows],
                                const float (&O)[kRows][VE]) {
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        if (r >= rows) break;
        const long long off = (long long)b * p.o_sb + (long long)(h0 + r) * p.o_sh + lane;
        const float inv = __frcp_rn(Ls[r]);
#pragma unroll
        for (int j = 0; j < VE; ++j) {
          const float val = O[r][j] * inv;
          if (p.out_f32) {
            reinterpret_cast<float*>(p.out)[off + j * 32] = val;
          } else {
            reinterpret_cast<T*>(p.out)[off + j * 32] = from_float<T>(val);
          }
        }
        if (p.lse != nullptr && lane == 0) p.lse[(long long)b * p.lse_sb + h0 + r] = M[r] + __log2f(Ls[r]);
      }
    };
    // Fold one piece (m, l, o) into the running (M, Ls, O); the first piece is taken as it is.
    const auto fold = [&](float (&M)[kRows], float (&Ls)[kRows], float (&O)[kRows][VE], int rows,
                          const float (&qm)[kRows], const float (&ql)[kRows], const float (&qo)[kRows][VE]) {
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        if (r >= rows) break;
        if (M[r] == -CUDART_INF_F) {
          M[r] = qm[r];
          Ls[r] = ql[r];
#pragma unroll
          for (int j = 0; j < VE; ++j) O[r][j] = qo[r][j];
        } else {
          const float mn = fmaxf(M[r], qm[r]);
          const float a = fast_exp2(M[r] - mn);
          const float w = fast_exp2(qm[r] - mn);
          Ls[r] = Ls[r] * a + ql[r] * w;
#pragma unroll
          for (int j = 0; j < VE; ++j) O[r][j] = O[r][j] * a + qo[r][j] * w;
          M[r] = mn;
        }
      }
    };
    // Load one piece from its workspace slot and zero the o entries this lane read.
    const auto load = [&](long long base, int rows, float (&qm)[kRows], float (&ql)[kRows], float (&qo)[kRows][VE]) {
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        if (r >= rows) break;
        qm[r] = __ldcg(p.ws_ml + (base + r) * 2);
        ql[r] = __ldcg(p.ws_ml + (base + r) * 2 + 1);
#pragma unroll
        for (int j = 0; j < VE; ++j) {
          qo[r][j] = __ldcg(p.ws_o + (base + r) * D + j * 32 + lane);
          __stcg(p.ws_o + (base + r) * D + j * 32 + lane, 0.f);
        }
      }
    };
    const Split split(total, gridDim.x);
    int ev = 0;
    while (true) {
      if (!mbar_wait_bounded(mfull, uint32_t(ev & 1), p.err, abort_flag, p.wait_ns)) break;
      const int flags = evt->flags;
      if (flags & kDone) break;
      const int b = evt->b, unit_local = evt->unit_local, chunks_b = evt->chunks_b;
      const long long unit_base = evt->unit_base;
      const bool whole = (flags & kFull) != 0;
      const long long unit = (long long)b * nkg + unit_local;
      // A split unit's ticket, read now so that its latency overlaps the fold
      // below.  An acquire load: if it shows every other piece's ticket, their
      // workspace writes are visible to this lane (a fence here costs ~1 us).
      const int ticket0 = whole ? 0 : ld_acquire_gpu(p.ws_count + unit);
      const int kvh = unit_local / p.head_groups;
      const int hg = unit_local - kvh * p.head_groups;
      const int rows = min(kRows, p.group - hg * kRows);
      const int h0 = kvh * p.group + hg * kRows;

      // This piece: the consumer warps' partials folded together.
      float M[kRows], Ls[kRows], O[kRows][VE];
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        M[r] = -CUDART_INF_F;
        Ls[r] = 0.f;
#pragma unroll
        for (int j = 0; j < VE; ++j) O[r][j] = 0.f;
        if (r < rows) {
#pragma unroll
          for (int w = 0; w < kWarps; ++w) M[r] = fmaxf(M[r], mM[w * kRows + r]);
#pragma unroll
          for (int w = 0; w < kWarps; ++w) {
            const float wt = fast_exp2(mM[w * kRows + r] - M[r]);
            Ls[r] += mL[w * kRows + r] * wt;
#pragma unroll
            for (int j = 0; j < VE; ++j) O[r][j] += mO[(w * kRows + r) * (D + 8) + j * 32 + lane] * wt;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(mfree);
      ++ev;

      if (whole) {
        store_rows(b, h0, rows, M, Ls, O);
        continue;
      }

      // ---- a unit split across CTAs ----
      // Its pieces belong to the CTAs whose (non-empty) chunk ranges overlap
      // it: owner(first chunk) .. owner(last chunk), skipping CTAs with empty
      // ranges (more CTAs than chunks when the problem is small).  A piece's
      // workspace slot is 1 if it ends its CTA's range, else 0.
      const int ca = split.owner(unit_base);
      const int cb = split.owner(unit_base + chunks_b - 1);
      const auto piece = [&](int cc, long long& base) -> bool {
        const long long rs = split.start(cc);
        base = ((long long)cc * 2 + ((rs < unit_base) ? 1 : 0)) * kRows;
        return cc <= cb && split.start(cc + 1) > rs;
      };
      int parts = 0;
      for (int c0 = ca; c0 <= cb; c0 += 32) {
        long long unused;
        parts += __popc(__ballot_sync(0xffffffffu, piece(c0 + lane, unused)));
      }
      // Last piece?  Either every other piece had taken its ticket when this
      // one looked (then it takes none), or its own ticket is the last one.
      // The first piece of a unit that arrives last keeps its partial in
      // registers: it is the first term of the combine either way.
      bool last = ticket0 == parts - 1;
      const bool keep = last && ca == int(blockIdx.x);
      if (!keep) {
        const long long base = ((long long)blockIdx.x * 2 + ((x0 < unit_base) ? 1 : 0)) * kRows;
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          if (r >= rows) break;
#pragma unroll
          for (int j = 0; j < VE; ++j) __stcg(p.ws_o + (base + r) * D + j * 32 + lane, O[r][j]);
          if (lane == 0) {
            __stcg(p.ws_ml + (base + r) * 2, M[r]);
            __stcg(p.ws_ml + (base + r) * 2 + 1, Ls[r]);
          }
        }
        __syncwarp();
      }
      if (!last) {
        int t = 0;
        if (lane == 0) {
          __threadfence();
          t = atomicAdd(p.ws_count + unit, 1);
        }
        last = __shfl_sync(0xffffffffu, t, 0) == parts - 1;
        if (!last) continue;
        ld_acquire_gpu(p.ws_count + unit);  // every lane acquires the other pieces' writes
      }

      // Combine the pieces in CTA order (the same arithmetic whoever merges).
      if (!keep) {
#pragma unroll
        for (int r = 0; r < kRows; ++r) M[r] = -CUDART_INF_F;
      }
      for (int c0 = ca; c0 <= cb; c0 += 32) {
        long long my_base;
        unsigned mask = __ballot_sync(0xffffffffu, piece(c0 + lane, my_base));
        if (keep && c0 == ca) mask &= ~1u;  // this CTA's piece, already the first term
        while (mask != 0u) {
          const int i0 = __ffs(mask) - 1;
          mask &= mask - 1u;
          const long long b0 = __shfl_sync(0xffffffffu, my_base, i0);
          float am[kRows], al[kRows], ao[kRows][VE];
          if constexpr (kPair == 2) {
            if (mask != 0u) {
              const int i1 = __ffs(mask) - 1;
              mask &= mask - 1u;
              const long long b1 = __shfl_sync(0xffffffffu, my_base, i1);
              float bm[kRows], bl[kRows], bo[kRows][VE];
              load(b0, rows, am, al, ao);
              load(b1, rows, bm, bl, bo);
              fold(M, Ls, O, rows, am, al, ao);
              fold(M, Ls, O, rows, bm, bl, bo);
              continue;
            }
          }
          load(b0, rows, am, al, ao);
          fold(M, Ls, O, rows, am, al, ao);
        }
      }
      store_rows(b, h0, rows, M, Ls, O);
      // Leave the workspace zero-filled for the next call: the (m, l) pairs
      // once every lane has read them, then the ticket.
      __syncwarp();
      for (int c0 = ca; c0 <= cb; c0 += 32) {
        long long base;
        const int cc = c0 + lane;
        if (!piece(cc, base) || (keep && cc == int(blockIdx.x))) continue;
        for (int r = 0; r < rows; ++r) {
          __stcg(p.ws_ml + (base + r) * 2, 0.f);
          __stcg(p.ws_ml + (base + r) * 2 + 1, 0.f);
        }
      }
      if (lane == 0) p.ws_count[unit] = 0;
    }
    return;
  }

  // ======================= consumer warps =======================
  const int g = lane >> 2;
  const int c = lane & 3;
  const int ctid = tid;  // 0..127
  float o[NT][4];
  float m_run = -CUDART_INF_F, l_run = 0.f;
  float cs_run = 0.f;  // biased int8: running sum of the p fed to P.V (rescaled like l_run)
  float qbias = 0.f;   // biased int8: 1152 * sum(q) of row g
  float qmul = 1.f;    // bf16 queries with 8-bit caches: the power of two the row was scaled by
  uint32_t qa[D / 16][2];
  int it = 0;
  int ev = 0;  // pieces handed to the merge warp
  // Failure-path test: a wait that nothing ends runs out after p.wait_ns,
  // records FAT_DEVERR_TIMEOUT and raises the abort flag; every other warp
  // then stops at its next wait and drains its copies.
  if (p.expire && warp == 0) mbar_wait_bounded(never, 0, p.err, abort_flag, p.wait_ns);

  while (true) {
    const int s = it % kStages;
    if (!mbar_wait_bounded(full0 + 8u * s, uint32_t((it / kStages) & 1), p.err, abort_flag, p.wait_ns)) break;
    const Meta& mt = meta[s];
    const int flags = mt.flags;
    if (flags & kDone) break;
    const int b = mt.b, unit_local = mt.unit_local, chunk = mt.chunk, seq_len = mt.seq_len, chunks_b = mt.chunks_b;
    const long long unit_base = mt.unit_base;

    if (flags & kFirst) {
      m_run = -CUDART_INF_F;
      l_run = 0.f;
      cs_run = 0.f;
#pragma unroll
      for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      const T* qs = reinterpret_cast<const T*>(reinterpret_cast<const uint8_t*>(qarea) + size_t(s) * L::kQBytes);
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        // 8-bit caches use a permuted reduction order (see the K fragments below).
        const int d0 = (EB == 2) ? ks * 16 + 2 * c : c * (D / 4) + 4 * ks;
        const int d1 = (EB == 2) ? ks * 16 + 8 + 2 * c : c * (D / 4) + 4 * ks + 2;
        qa[ks][0] = *reinterpret_cast<const uint32_t*>(qs + g * D + d0);
        qa[ks][1] = *reinterpret_cast<const uint32_t*>(qs + g * D + d1);
      }
      if constexpr (kQConv) {
        // Scale the row by the power of two that puts its largest magnitude in
        // [2^14, 2^15): multiplying by it is exact, and so is the bf16 -> fp16
        // conversion of every element that stays above fp16's normal minimum
        // (those below are 2^-28 of the largest and vanish in the dot product).
        // The power of two goes back into the score multiplier; |e| <= 126 keeps
        // both 2^e and 2^-e normal floats, and covers every finite bf16 row.
        float mx = 0.f;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          float x0, x1, x2, x3;
          unpack2<T>(qa[ks][0], x0, x1);
          unpack2<T>(qa[ks][1], x2, x3);
          mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x0), fabsf(x1)), fmaxf(fabsf(x2), fabsf(x3))));
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        int e = 0;
        if (mx > 0.f && mx < CUDART_INF_F) e = max(-126, min(126, ((__float_as_int(mx) >> 23) & 0xFF) - 127 - 14));
        const float down = __int_as_float((127 - e) << 23);
        qmul = __int_as_float((127 + e) << 23);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float x0, x1;
            unpack2<T>(qa[ks][h], x0, x1);
            qa[ks][h] = pack2<__half>(x0 * down, x1 * down);
          }
        }
      }
      if constexpr (kBias) {
        float sq = 0.f;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          float x0, x1, x2, x3;
          unpack2<Tc>(qa[ks][0], x0, x1);
          unpack2<Tc>(qa[ks][1], x2, x3);
          sq += (x0 + x1) + (x2 + x3);
        }
        sq += __shfl_xor_sync(0xffffffffu, sq, 1);
        sq += __shfl_xor_sync(0xffffffffu, sq, 2);
        qbias = kI8Bias * sq;
      }
    }

    const uint32_t kt = smem_u32(stages) + uint32_t(s) * L::kStage;
    const uint32_t vt = kt + L::kTile;
    // Each warp owns kTW consecutive tokens of the chunk, done 16 at a time.
#pragma unroll 1
    for (int sub = 0; sub < kTW / 16; ++sub) {
    const int wrow = warp * kTW + sub * 16;  // first row of this slice in the stage
    const int tok0 = chunk * kChunk + wrow;
    const int nvalid = seq_len - tok0;
    if (nvalid > 0) {
      if (nvalid < 16) {
        // Rows past the sequence may hold anything (even NaN): zero their V so
        // that p = 0 contributes exactly nothing.
        constexpr int kVecPerRow = L::kRowBytes / 16;
        for (int i = lane; i < (16 - nvalid) * kVecPerRow; i += 32) {
          const int r = nvalid + i / kVecPerRow;
          const int bc = (i % kVecPerRow) * 16;
          const uint32_t a = L::addr(vt, wrow + r, bc);
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0) : "memory");
        }
        __syncwarp();
      }

      // ---- S = Q K^T for 16 tokens (two n-tiles) ----
      float sacc[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
      if constexpr (EB == 2) {
        const int row = wrow + ((lane >> 4) << 3) + (lane & 7);
        const int khalf = ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(L::addr(kt, row, (ks * 16 + khalf) * 2), b0, b1, b2, b3);
          const uint32_t a[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
          MmaOp<Tc>::run(sacc[0], a, b0, b1);
          MmaOp<Tc>::run(sacc[1], a, b2, b3);
        }
      } else {
        // 8-bit codes.  Lane (g, c) owns the reduction slice d in
        // [c*D/4, (c+1)*D/4) of token rows g and g+8: k-step ks maps its k-slots
        // (2c, 2c+1) to dims c*D/4 + 4ks + {0,1} and (2c+8, 2c+9) to + {2,3}.
        // The same permutation was applied to the query fragments, so the dot
        // products are unchanged; each lane reads contiguous bytes.
        constexpr int kSlice = D / 4;  // bytes per lane per row
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int row = wrow + j * 8 + g;
#pragma unroll
          for (int v = 0; v < kSlice / 16 + (kSlice % 16 ? 1 : 0); ++v) {
            uint32_t wv[4];
            const uint32_t a = L::addr(kt, row, c * kSlice + v * 16);
            if constexpr (kSlice >= 16) {
              asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(wv[0]), "=r"(wv[1]), "=r"(wv[2]), "=r"(wv[3])
                           : "r"(a));
            } else {
              asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(wv[0]), "=r"(wv[1]) : "r"(a));
              wv[2] = wv[3] = 0u;
            }
#pragma unroll
            for (int i = 0; i < (kSlice >= 16 ? 4 : 2); ++i) {
              const int ks = v * 4 + i;
              uint32_t b0, b1;
              if constexpr (kBias) {
                widen_i8_biased(wv[i], b0, b1);
              } else {
                Widen<Tc, KVT>::run(wv[i], b0, b1);
              }
              const uint32_t av[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
              MmaOp<Tc>::run(sacc[j], av, b0, b1);
            }
          }
        }
      }

      // ---- online softmax on the fragment (rows g: heads, cols: tokens) ----
      const int toks[4] = {2 * c, 2 * c + 1, 8 + 2 * c, 9 + 2 * c};
      const float sv_raw[4] = {sacc[0][0], sacc[0][1], sacc[1][0], sacc[1][1]};
      float sv[4];
      float ksc[2] = {1.f, 1.f}, vsc[2] = {1.f, 1.f};
      if constexpr (EB == 1) {
        const int grp = (wrow) / 8;
        ksc[0] = mt.kscale[grp];
        ksc[1] = mt.kscale[grp + 1];
        vsc[0] = mt.vscale[grp];
        vsc[1] = mt.vscale[grp + 1];
      }
      // Scores in log2 units: (s - qbias) * scale * k_scale as one FMA per score.
      const float kf[2] = {p.scale_log2 * qmul * ksc[0], p.scale_log2 * qmul * ksc[1]};
      const float kb[2] = {-qbias * kf[0], -qbias * kf[1]};
      if (nvalid >= 16) {
        // 8-bit layouts: two-lane FMAs (their consumer warps are issue-bound);
        // 16-bit layouts keep the scalar form, which measured no slower.
        if constexpr (EB == 1) {
          fma2(sv[0], sv[1], sv_raw[0], sv_raw[1], kf[0], kb[0]);
          fma2(sv[2], sv[3], sv_raw[2], sv_raw[3], kf[1], kb[1]);
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) sv[i] = fmaf(sv_raw[i], kf[i >> 1], kb[i >> 1]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          sv[i] = (toks[i] < nvalid) ? fmaf(sv_raw[i], kf[i >> 1], kb[i >> 1]) : -CUDART_INF_F;
      }
      float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      // The running max moves only when a score exceeds it by more than 2^8
      // (log2 units), so P stays <= 256 and O is rescaled rarely; o, l and m
      // stay consistent, so the fold and the log-sum-exp merge are unchanged.
      const float m_new = (mx > m_run + kDecodeRescaleLog2) ? mx : m_run;
      const float alpha = fast_exp2(m_run - m_new);
      float pr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pr[i] = fast_exp2(sv[i] - m_new);
      l_run = l_run * alpha + ((pr[0] + pr[1]) + (pr[2] + pr[3]));
      m_run = m_new;
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          if constexpr (EB == 1) {
            mul2(o[n][0], o[n][1], o[n][0], o[n][1], alpha);
            mul2(o[n][2], o[n][3], o[n][2], o[n][3], alpha);
          } else {
            o[n][0] *= alpha;
            o[n][1] *= alpha;
            o[n][2] *= alpha;
            o[n][3] *= alpha;
          }
        }
      }

      // ---- O += P V : rows 0-7 carry P rounded to 16 bits, rows 8-15 the remainder ----
      uint32_t pa[4];
      float pv[4] = {pr[0], pr[1], pr[2], pr[3]};
      if constexpr (EB == 1) {
        mul2(pv[0], pv[1], pr[0], pr[1], vsc[0]);
        mul2(pv[2], pv[3], pr[2], pr[3], vsc[1]);
      }
      split_hi_lo<Tc>(pv[0], pv[1], pa[0], pa[1]);
      split_hi_lo<Tc>(pv[2], pv[3], pa[2], pa[3]);
      if constexpr (kBias) cs_run = cs_run * alpha + ((pv[0] + pv[1]) + (pv[2] + pv[3]));
      if constexpr (EB == 2) {
        const int row = wrow + ((lane >> 3) & 1) * 8 + (lane & 7);
        const int dsel = (lane >> 4) << 3;
#pragma unroll
        for (int np = 0; np < D / 16; ++np) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(L::addr(vt, row, (np * 16 + dsel) * 2), b0, b1, b2, b3);
          MmaOp<Tc>::run(o[2 * np], pa, b0, b1);
          MmaOp<Tc>::run(o[2 * np + 1], pa, b2, b3);
        }
      } else {
        // 8-bit V: lane (g, c) owns output dims [g*D/8, (g+1)*D/8) (B column g
        // of n-tile nt is dim g*D/8 + nt) and reads token rows 2c, 2c+1, 2c+8,
        // 2c+9; byte nt of two rows forms the pair of one B register.
        constexpr int kSlice = D / 8;  // bytes per lane per row
        const int rbase = wrow + 2 * c;
        uint32_t rw[4][kSlice / 4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int row = rbase + (r & 1) + (r >> 1) * 8;
#pragma unroll
          for (int v = 0; v < kSlice / 4; v += 4) {
            const uint32_t a = L::addr(vt, row, g * kSlice + v * 4);
            if constexpr (kSlice >= 16) {
              asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(rw[r][v]), "=r"(rw[r][v + 1]), "=r"(rw[r][v + 2]), "=r"(rw[r][v + 3])
                           : "r"(a));
            } else if constexpr (kSlice >= 8) {
              asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(rw[r][v]), "=r"(rw[r][v + 1]) : "r"(a));
            } else {
              asm volatile("ld.shared.u32 %0, [%1];" : "=r"(rw[r][v]) : "r"(a));
            }
          }
        }
        if constexpr (kBias) {
          // Pair (row 2c, row 2c+1) and (row 2c+8, row 2c+9) of byte i: one
          // PRMT gathers the two codes, one LOP3 makes the biased fp16 pair.
#pragma unroll
          for (int w = 0; w < kSlice / 4; ++w) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t sel = uint32_t(i) * 0x11u + uint32_t(4 + i) * 0x1100u;
              const uint32_t b0 = biased_pair_i8(__byte_perm(rw[0][w], rw[1][w], sel));
              const uint32_t b1 = biased_pair_i8(__byte_perm(rw[2][w], rw[3][w], sel));
              MmaOp<Tc>::run(o[4 * w + i], pa, b0, b1);
            }
          }
        } else {
#pragma unroll
        for (int w = 0; w < kSlice / 4; ++w) {
          uint32_t b0a, b0b, b0c, b0d, b1a, b1b, b1c, b1d;
          Widen<Tc, KVT>::run(__byte_perm(rw[0][w], rw[1][w], 0x5140), b0a, b0b);
          Widen<Tc, KVT>::run(__byte_perm(rw[0][w], rw[1][w], 0x7362), b0c, b0d);
          Widen<Tc, KVT>::run(__byte_perm(rw[2][w], rw[3][w], 0x5140), b1a, b1b);
          Widen<Tc, KVT>::run(__byte_perm(rw[2][w], rw[3][w], 0x7362), b1c, b1d);
          MmaOp<Tc>::run(o[4 * w + 0], pa, b0a, b1a);
          MmaOp<Tc>::run(o[4 * w + 1], pa, b0b, b1b);
          MmaOp<Tc>::run(o[4 * w + 2], pa, b0c, b1c);
          MmaOp<Tc>::run(o[4 * w + 3], pa, b0d, b1d);
        }
        }
      }
      if (nvalid < 16) fence_proxy_async_smem();
    }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8u * s);
    ++it;

    if (flags & kLast) {
      // ---- end of this CTA's piece of a unit: hand the warps' partials to
      // the merge warp (once it has taken the previous piece) and go on ----
      if (ev > 0 && !mbar_wait_bounded(mfree, uint32_t((ev - 1) & 1), p.err, abort_flag, p.wait_ns)) break;
      const float l_row = l_run + __shfl_xor_sync(0xffffffffu, l_run, 1);
      const float l_tot = l_row + __shfl_xor_sync(0xffffffffu, l_row, 2);
      float corr = 0.f;  // biased int8: 1152 * sum(p) of row g over the piece
      if constexpr (kBias) {
        const float c_row = cs_run + __shfl_xor_sync(0xffffffffu, cs_run, 1);
        corr = kI8Bias * (c_row + __shfl_xor_sync(0xffffffffu, c_row, 2));
      }
      float* myO = mO + (warp * kRows + g) * (D + 8);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        if constexpr (EB == 2) {
          *reinterpret_cast<float2*>(myO + n * 8 + 2 * c) = make_float2(o[n][0] + o[n][2], o[n][1] + o[n][3]);
        } else {
          myO[(2 * c) * (D / 8) + n] = (o[n][0] + o[n][2]) - corr;
          myO[(2 * c + 1) * (D / 8) + n] = (o[n][1] + o[n][3]) - corr;
        }
      }
      if (c == 0) {
        mM[warp * kRows + g] = m_run;
        mL[warp * kRows + g] = l_tot;
      }
      if (ctid == 0) {
        evt->flags = flags;
        evt->b = b;
        evt->unit_local = unit_local;
        evt->chunks_b = chunks_b;
        evt->unit_base = unit_base;
      }
      mbar_arrive(mfull);
      ++ev;
    }
  }
  // No more pieces: tell the merge warp (after it has taken the last one).
  // After an abort it stops on the shared abort flag instead.
  if (!*abort_flag && (ev == 0 || mbar_wait_bounded(mfree, uint32_t((ev - 1) & 1), p.err, abort_flag, p.wait_ns))) {
    if (ctid == 0) evt->flags = kDone;
    mbar_arrive(mfull);
  }
}

}  // namespace dec
}  // namespace fat

// =============================================================================
// Host side
// =============================================================================
namespace fat {
namespace {

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct WsLayout {
  size_t o_off, ml_off, count_off, total;
};

WsLayout ws_layout(int grid, long long units, int head_dim) {
  WsLayout w;
  w.o_off = 0;
  w.ml_off = align_up(size_t(grid) * 2 * dec::kRows * head_dim * sizeof(float), 256);
  w.count_off = align_up(w.ml_off + size_t(grid) * 2 * dec::kRows * 2 * sizeof(float), 256);
  w.total = align_up(w.count_off + size_t(units) * sizeof(int), 256);
  return w;
}

template <typename T, int D, int KVT>
int launch_t(const DecodeArgs& a, int device, int grid, const WsLayout& ws) {
  constexpr int EB = (KVT == FAT_DTYPE_I8 || KVT == FAT_DTYPE_E4M3) ? 1 : 2;
  using L = dec::Layout<D, EB>;
  auto kern = dec::paged_decode_kernel<T, D, KVT>;
  static_assert(L::kSmem <= 227 * 1024, "decode stage ring exceeds shared memory");
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), int(L::kSmem), current_device());
  if (e != cudaSuccess) return cuda_failure("cudaFuncSetAttribute(decode)", e);

  // One TMA box covers gcd(page_size, chunk) token rows -- as tall as possible
  // (whole pages up to the 64-token chunk) while never crossing a page or a
  // chunk boundary, so large pages need fewer, taller copies.
  int box_rows = L::kChunk;
  while (a.page_size % box_rows) box_rows >>= 1;
  // 5-D view of the cache: {elements of a 128-byte column block, column block,
  // kv head, slot, page}; one box = box_rows slots x every column block of one
  // head, i.e. whole token rows.
  const uint64_t dims[5] = {uint64_t(L::kBoxBytes / EB), uint64_t(L::kCB), uint64_t(a.num_kv_heads),
                            uint64_t(a.page_size), uint64_t(a.num_pages)};
  const uint64_t strides[4] = {uint64_t(L::kBoxBytes), uint64_t(a.kv_sh) * EB, uint64_t(a.kv_ss) * EB,
                               uint64_t(a.kv_sp) * EB};
  const uint32_t box[5] = {uint32_t(L::kBoxBytes / EB), uint32_t(L::kCB), 1u, uint32_t(box_rows), 1u};
  const CUtensorMapDataType dt = EB == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUtensorMapSwizzle sw = L::kBoxBytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
  // A token row narrower than 256 B sits next to another head's row: widen L2
  // fills only to the row itself so that neighbour is not read along with it.
  const CUtensorMapL2promotion promo =
      L::kRowBytes >= 256 ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B : CU_TENSOR_MAP_L2_PROMOTION_L2_128B;
  CUtensorMap tmk, tmv;
  std::string why;
  if (!encode_tiled(&tmk, dt, 5, a.k_cache, dims, strides, box, sw, &why, promo)) return invalid("k_cache: " + why);
  if (!encode_tiled(&tmv, dt, 5, a.v_cache, dims, strides, box, sw, &why, promo)) return invalid("v_cache: " + why);

  dec::Params p;
  p.q = a.q;
  p.q_sb = a.q_sb;
  p.q_sh = a.q_sh;
  p.out = a.out;
  p.o_sb = a.o_sb;
  p.o_sh = a.o_sh;
  p.page_table = a.page_table;
  p.pt_sb = a.pt_sb;
  p.max_pages = int(a.max_pages);
  p.cap_tokens = int(std::min<long long>((long long)a.max_pages * a.page_size, dec::kMaxTokens));
  p.seq_lens = a.seq_lens;
  p.k_scale = a.k_scale;
  p.v_scale = a.v_scale;
  p.s_sp = a.scale_sp;
  p.batch = a.batch;
  p.num_heads = a.num_heads;
  p.num_kv_heads = a.num_kv_heads;
  p.group = a.num_heads / a.num_kv_heads;
  p.head_groups = (p.group + dec::kRows - 1) / dec::kRows;
  p.page_size = a.page_size;
  p.num_pages = int(a.num_pages);
  p.box_rows = box_rows;
  p.scale_log2 = float(double(a.softmax_scale) * 1.4426950408889634);
  p.out_f32 = a.out_dtype == FAT_DTYPE_F32;
  uint8_t* wsb = static_cast<uint8_t*>(a.workspace);
  p.ws_o = reinterpret_cast<float*>(wsb + ws.o_off);
  p.ws_ml = reinterpret_cast<float*>(wsb + ws.ml_off);
  p.ws_count = reinterpret_cast<int*>(wsb + ws.count_off);
  p.err = a.error_word;
  p.lse = a.lse;
  p.lse_sb = a.lse_sb;
  p.wait_ns = wait_limit_ns();
  p.expire = take_expire_request() ? 1 : 0;
  (void)device;
  kern<<<grid, L::kThreads, L::kSmem, a.stream>>>(tmk, tmv, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_failure("paged_decode launch", e);
  return FAT_OK;
}

template <typename T, int KVT>
int dispatch_dim(const DecodeArgs& a, int device, int grid, const WsLayout& ws) {
  switch (a.head_dim) {
    case 32:
      return launch_t<T, 32, KVT>(a, device, grid, ws);
    case 64:
      return launch_t<T, 64, KVT>(a, device, grid, ws);
    case 128:
      return launch_t<T, 128, KVT>(a, device, grid, ws);
    case 256:
      return launch_t<T, 256, KVT>(a, device, grid, ws);
    default:
      return unsupported("paged_decode: head_dim must be 32, 64, 128 or 256, got " + std::to_string(a.head_dim));
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

size_t decode_workspace_bytes(int device, int batch, int num_heads, int num_kv_heads, int head_dim) {
  if (num_kv_heads <= 0 || num_heads <= 0 || batch < 0 || head_dim <= 0) return 0;
  const int group = num_heads / num_kv_heads;
  const long long units = (long long)batch * num_kv_heads * ((group + dec::kRows - 1) / dec::kRows);
  return ws_layout(sm_count(device), units, head_dim).total;
}

void decode_ticket_range(int device, int batch, int num_heads, int num_kv_heads, int head_dim, size_t* offset,
                         size_t* bytes) {
  *offset = 0;
  *bytes = 0;
  if (num_kv_heads <= 0 || num_heads <= 0 || batch < 0 || head_dim <= 0) return;
  const int group = num_heads / num_kv_heads;
  const long long units = (long long)batch * num_kv_heads * ((group + dec::kRows - 1) / dec::kRows);
  *offset = ws_layout(sm_count(device), units, head_dim).count_off;
  *bytes = size_t(units) * sizeof(int);
}

int check_paged_decode(const DecodeArgs& a) {
  if (a.batch < 0) return invalid("paged_decode: batch must be non-negative");
  if (a.num_heads <= 0 || a.num_kv_heads <= 0) return invalid("paged_decode: head counts must be positive");
  if (a.num_heads % a.num_kv_heads != 0)
    return invalid("paged_decode: num_heads " + std::to_string(a.num_heads) + " must be divisible by num_kv_heads " +
                   std::to_string(a.num_kv_heads));
  // Pages are moved in boxes of min(page_size, 16) token rows that must not
  // straddle two pages: 8, or a multiple of 16 up to the TMA box limit.
  if (!(a.page_size == 8 || (a.page_size % 16 == 0 && a.page_size <= 256)))
    return unsupported("paged_decode: page_size must be 8 or a multiple of 16 up to 256, got " +
                       std::to_string(a.page_size));
  if (a.q_dtype != FAT_DTYPE_F16 && a.q_dtype != FAT_DTYPE_BF16)
    return unsupported("paged_decode: q must be fp16 or bf16");
  const bool quant = a.kv_dtype == FAT_DTYPE_I8 || a.kv_dtype == FAT_DTYPE_E4M3;
  if (!quant && a.kv_dtype != a.q_dtype) return invalid("paged_decode: q dtype must match the cache dtype");
  if (quant && (a.k_scale == nullptr || a.v_scale == nullptr))
    return invalid("paged_decode: an int8/fp8 cache needs k_scale and v_scale");
  if (a.out_dtype != a.q_dtype && a.out_dtype != FAT_DTYPE_F32)
    return invalid("paged_decode: out dtype must be q's dtype or fp32");
  if (a.batch == 0) return FAT_OK;
  if (a.q == nullptr || a.k_cache == nullptr || a.v_cache == nullptr || a.page_table == nullptr ||
      a.seq_lens == nullptr || a.out == nullptr || a.workspace == nullptr)
    return invalid("paged_decode: null pointer argument");
  if (a.num_pages <= 0 || a.max_pages <= 0) return invalid("paged_decode: empty cache or page table");
  const int eb = quant ? 1 : 2;
  if (!aligned16(a.k_cache) || !aligned16(a.v_cache) || (a.kv_sp * eb) % 16 || (a.kv_ss * eb) % 16 ||
      (a.kv_sh * eb) % 16)
    return unsupported("paged_decode: K/V base addresses and page/slot/head strides must be 16-byte aligned");
  if (!aligned16(a.q) || (a.q_sb * 2) % 16 || (a.q_sh * 2) % 16)
    return unsupported("paged_decode: q must be 16-byte aligned with 16-byte-multiple strides");
  if (a.head_dim != 32 && a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256)
    return unsupported("paged_decode: head_dim must be 32, 64, 128 or 256, got " + std::to_string(a.head_dim));
  return FAT_OK;
}

int launch_paged_decode(const DecodeArgs& a) {
  const int rc = check_paged_decode(a);
  if (rc != FAT_OK || a.batch == 0) return rc;
  const int device = current_device();
  const int grid = sm_count(device);
  const int group = a.num_heads / a.num_kv_heads;
  const long long units = (long long)a.batch * a.num_kv_heads * ((group + dec::kRows - 1) / dec::kRows);
  const WsLayout ws = ws_layout(grid, units, a.head_dim);
  if (a.workspace_bytes < ws.total)
  {
    set_last_error("paged_decode: workspace holds " + std::to_string(a.workspace_bytes) + " bytes, needs " +
                   std::to_string(ws.total));
    return FAT_ERR_WORKSPACE;
  }
  if (device < 0) return invalid("paged_decode: no current CUDA device");

  if (a.q_dtype == FAT_DTYPE_F16) {
    switch (a.kv_dtype) {
      case FAT_DTYPE_F16:
        return dispatch_dim<__half, FAT_DTYPE_F16>(a, device, grid, ws);
      case FAT_DTYPE_I8:
        return dispatch_dim<__half, FAT_DTYPE_I8>(a, device, grid, ws);
      case FAT_DTYPE_E4M3:
        return dispatch_dim<__half, FAT_DTYPE_E4M3>(a, device, grid, ws);
    }
  } else {
    switch (a.kv_dtype) {
      case FAT_DTYPE_BF16:
        return dispatch_dim<__nv_bfloat16, FAT_DTYPE_BF16>(a, device, grid, ws);
      case FAT_DTYPE_I8:
        return dispatch_dim<__nv_bfloat16, FAT_DTYPE_I8>(a, device, grid, ws);
      case FAT_DTYPE_E4M3:
        return dispatch_dim<__nv_bfloat16, FAT_DTYPE_E4M3>(a, device, grid, ws);
    }
  }
  return unsupported("paged_decode: unsupported dtype combination");
}

}  // namespace fat
