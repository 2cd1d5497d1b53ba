// Packed varlen prefill attention (causal or not, GQA/MQA) for sm_100a.
//
// Replaces FlashAttnTile's _fwd_varlen_kernel (flashattn_tile/kernels/prefill.py:34-138):
// per (query tile, query head, sequence) an online-softmax pass over 128-row
// K/V tiles with bottom-right causal alignment (query i sees keys
// j <= i + kv_len - q_len), GQA head h reading KV head h / G, P rounded to the
// input dtype before P.V (prefill.py:128) and fp32 accumulation.  Optionally
// (p_split) a key tile's P enters P.V as a 16-bit head plus a 16-bit remainder,
// keeping the probabilities to ~2^-16: for bf16 by default on every key tile
// that holds a key weighing more than 1/16 of its row's sum so far.
//
// One CTA per pair of 128-row query tiles (256 rows), warp-specialised:
//   warps 0-3   softmax of query tile 0, warps 4-7 softmax of query tile 1:
//               thread r owns row r of its tile (tensor-memory lane r), reads
//               its S row, keeps the running max and sum in registers, writes P
//               (16-bit) over its S row, and rescales its O row in tensor
//               memory only when the row max grew by more than 2^8 (P <= 256);
//   warp 8      TMA producer: both Q tiles once, then K and V tiles into two
//               independent 128-byte-swizzled rings;
//   warp 9      tcgen05 issuer (one thread), per K/V tile j:
//                 O0 += P0 V_{j-1};  S0 = Q0 K_j^T;  O1 += P1 V_{j-1};  S1 = Q1 K_j^T
//               so the tensor core works on one tile while the other tile's
//               softmax runs (ping-pong between the two warpgroups);
//   warps 10-11 idle (they complete the third warpgroup for setmaxnreg).
// Tensor memory (512 columns): S0 [0,128), S1 [128,256), O0 [256,256+D),
// O1 [384,384+D).  P_t is written over S_t; S_t(j) is issued after O_t += P_t(j-1)
// V_{j-1} by the same thread, and tcgen05.mma operations of one thread execute
// in issue order, so the completion of S_t(j) also means O_t holds every
// earlier P.V (the softmax may rescale O_t as soon as it sees S_t(j)).
// head_dim 256 uses one query tile per CTA (warps 0-3 softmax, 4 producer,
// 5 MMA issuer; S in columns [0,128), O in [128,384); single K and V buffers of
// 64 KB), the same code with the second tile absent.
// Every wait is bounded; on a timeout the CTA records FAT_DEVERR_TIMEOUT,
// drains its copies and MMAs, frees tensor memory and exits.
#include <math_constants.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>
#include <type_traits>

#include "common.cuh"
#include "host_util.h"
#include "prefill.h"
#include "tcgen05.cuh"

namespace fat {
namespace pre {

constexpr int BM = 128;    // query rows per tile (the MMA's M)
constexpr int BN = 128;    // keys per K/V tile
constexpr int kSoftmaxThreads = 128;  // per tile
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P <= 2^8 without rescaling
// Persistent grid: items in flight between the producer warp (which claims
// and describes them) and the MMA issuer and softmax warps.
constexpr int kItemSlots = 4;

struct Params {
  const int* cu_q;
  const int* cu_k;       // packed K/V: [batch + 1] token offsets
  void* out;
  long long o_st, o_sh;
  int num_heads, group;
  float scale_log2;
  int causal;
  int out_f32;
  int o_tma;             // tm_o describes out (16-bit output): full 32-row groups leave by TMA stores
  int* err;
  // Paged K/V (kPaged): sequence b's keys are its seq_lens_k[b] cached tokens.
  const int* page_table;
  long long pt_sb;
  int max_pages, num_pages, page_size;
  int rows_per_box;      // min(page_size, BN): token rows one TMA box brings from one page
  int cap_tokens;        // min(max_pages * page_size, 2^30): cached lengths are cut to this
  const int* seq_lens_k;
  unsigned long long wait_ns;  // limit of every bounded wait
  int expire;            // the MMA issuer first waits on a barrier phase nothing completes (failure-path tests)
  int p_split;           // P into P.V as head + remainder: 0 never, 1 where a key weighs (vote), 2 always
  int batch, num_pairs;  // sequences; 2-tile query pairs of the longest sequence
  int* sched;            // kPersist: {next rank, CTAs done}, zero at launch and zeroed again by the last CTA
  const unsigned* pv_emax;  // kHalfPV: largest finite |v| (bf16 bits) per (sequence, KV head), b * Hkv + kv head
  int num_kv_heads;
};

// p_split == 1: a key tile of a query tile enters P.V as a 16-bit head plus a
// 16-bit remainder (a second P.V pass; P kept to ~2^-16 relative) when any of
// its rows has a key whose probability exceeds kSplitTheta of the row's sum so
// far.  That sum only grows, so every key of an unsplit tile ends with weight
// <= kSplitTheta, and the 16-bit rounding of its P moves the output by at most
// 2^-8 * kSplitTheta * |v|; rows with few keys, or a few dominant keys, are
// always split.
constexpr float kSplitTheta = 1.0f / 16.0f;

// head_dim <= 128: two 128-row query tiles per CTA in ping-pong (S0, S1, O0,
// O1 fill the 512 tensor-memory columns).  head_dim 256: one tile per CTA (S in
// 128 columns, O in 256) with single K and V buffers (64 KB tiles).
template <int D>
struct Layout {
  static constexpr int kTiles = D <= 128 ? 2 : 1;  // query tiles per CTA
  static constexpr int kRowsPerCta = BM * kTiles;
  static constexpr int kProducerWarp = 4 * kTiles;
  static constexpr int kMmaWarp = kProducerWarp + 1;
  static constexpr int kThreads = (4 * kTiles + 4) * 32;  // softmax warpgroup(s) + {producer, MMA, 2 idle}
  // Two tiles: launched at 168 registers (65536 / 384, rounded to 8); the last
  // warpgroup (producer, MMA, 2 idle warps) drops to 88 and the two softmax
  // warpgroups rise to 208: 2*128*208 + 128*88 = 64512 = 384 * 168.  One tile
  // (256 threads) needs no split.
  static constexpr bool kSplitRegs = kTiles == 2;
  static constexpr int kRegsSoftmax = 208;
  static constexpr int kRegsOther = 88;
  static_assert(!kSplitRegs || 2 * 128 * kRegsSoftmax + 128 * kRegsOther <= kThreads * 168,
                "register split exceeds the launch");
  static constexpr int kCB = D / 64;        // 128-byte column blocks (16-bit elements)
  static constexpr int kTile = BM * D * 2;  // one Q, K or V tile
  static constexpr int kStagesK = D <= 64 ? 4 : (D <= 128 ? 3 : 1);
  static constexpr int kStagesV = D <= 64 ? 4 : (D <= 128 ? 2 : 1);
  // q_full, K and V full/empty rings, s_full and p_full per tile, drain, vtail,
  // never, q_empty, item_full and item_empty per item slot; then the
  // tensor-memory slot, the abort flag, the split votes ([tile][warp][parity]
  // ints) and the item slots (8 ints each).
  static constexpr int kBarBytes =
      8 * (1 + 2 * kStagesK + 2 * kStagesV + 2 * kTiles + 4 + 2 * kItemSlots) + 8 + 4 * 8 * kTiles + 32 * kItemSlots;
  static constexpr size_t kSmem = 1024 + size_t(kTile) * (kTiles + kStagesK + kStagesV) + kBarBytes;
  static_assert(kSmem <= 227 * 1024, "prefill tiles exceed shared memory");
  static constexpr uint32_t kColS = 0;               // S_t at column kColS + 128 t
  static constexpr uint32_t kColO = 128 * kTiles;    // O_t at columns [kColO + 128 t, kColO + 128 t + D)
  static_assert(kColO + 128 * (kTiles - 1) + D <= kTmemCols, "tensor memory overflow");
};

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <int Regs>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(Regs));
}
template <int Regs>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Regs));
}

// Number of K/V tiles query tile `t` of the CTA needs (0 if the tile is empty).
__device__ __forceinline__ int tiles_needed(int m0, int q_len, int kv_len, int causal) {
  if (m0 >= q_len || kv_len <= 0) return 0;
  const int n_kv = (kv_len + BN - 1) / BN;
  if (!causal) return n_kv;
  const int lim = min(m0 + BM, q_len) - 1 + (kv_len - q_len);  // last key any row of the tile sees
  return lim < 0 ? 0 : min(n_kv, lim / BN + 1);
}

// One work item: query pair `pair` (rows [256 pair, 256 pair + 256) with two
// tiles) of head h of sequence b, and the K/V tiles each of its tiles needs.
struct Work {
  int b, h, kvh, q0, q_len, k0, kv_len, m0, offset, n0, n1, n_max, q_tiles;
};

// kHalfPV: V of (sequence, KV head) was stored as fp16 times 2^-e, e = E - 14
// for E the binary exponent of its largest finite |v|: every finite scaled
// value is below 2^15 (inside fp16's range) and the largest at least 2^14 (small V keeps
// fp16's full precision); the output is scaled back by 2^e.  e is kept in
// [-100, 114] so that 2^e and 2^-e are normal floats (an all-zero V gets -100).
__host__ __device__ __forceinline__ int pv_exponent(unsigned absmax_bits) {
  const int biased = int((absmax_bits >> 7) & 0xffu);  // bf16: 8 exponent bits above 7 mantissa bits
  return min(114, max(-100, biased - 127 - 14));
}

// The tile counts of an item whose sequence fields are set.
template <int kTiles>
__device__ __forceinline__ void finish_work(const Params& p, int pair, Work& w) {
  w.kvh = w.h / p.group;
  w.m0 = pair * BM * kTiles;
  w.offset = w.kv_len - w.q_len;  // bottom-right causal alignment
  w.n0 = tiles_needed(w.m0, w.q_len, w.kv_len, p.causal);
  w.n1 = kTiles > 1 ? tiles_needed(w.m0 + BM, w.q_len, w.kv_len, p.causal) : 0;
  w.n_max = max(w.n0, w.n1);
  w.q_tiles = (kTiles > 1 && w.m0 + BM < w.q_len) ? 2 : 1;
}

template <int kTiles, bool kPaged>
__device__ __forceinline__ Work describe_work(const Params& p, int b, int h, int pair) {
  Work w;
  w.b = b;
  w.h = h;
  w.q0 = __ldg(p.cu_q + b);
  w.q_len = __ldg(p.cu_q + b + 1) - w.q0;
  w.k0 = kPaged ? 0 : __ldg(p.cu_k + b);
  // Paged: a length past the page table is cut to its capacity (and reported),
  // so tile positions stay in 32 bits and inside the table.
  w.kv_len = kPaged ? min(__ldg(p.seq_lens_k + b), p.cap_tokens) : __ldg(p.cu_k + b + 1) - w.k0;
  finish_work<kTiles>(p, pair, w);
  return w;
}

// An item as the producer warp publishes it: {b (-1: no more items), h, pair,
// q0, q_len, k0, kv_len}.
template <int kTiles>
__device__ __forceinline__ Work work_from_slot(const Params& p, const volatile int* e) {
  Work w;
  w.b = e[0];
  w.h = e[1];
  w.q0 = e[3];
  w.q_len = e[4];
  w.k0 = e[5];
  w.kv_len = e[6];
  finish_work<kTiles>(p, e[2], w);
  return w;
}

__device__ __forceinline__ void write_slot(volatile int* d, const Work& w, int pair, bool have) {
  d[0] = have ? w.b : -1;
  d[1] = w.h;
  d[2] = pair;
  d[3] = w.q0;
  d[4] = w.q_len;
  d[5] = w.k0;
  d[6] = w.kv_len;
}

template <bool kHalfPV>
__device__ __forceinline__ float pv_unscale(const Params& p, const Work& w) {
  if constexpr (!kHalfPV) {
    return 1.f;
  } else {
    const int e = pv_exponent(__ldg(p.pv_emax + (long long)w.b * p.num_kv_heads + w.kvh));
    return __int_as_float((127 + e) << 23);  // 2^e, -100 <= e <= 114
  }
}

// Persistent grid: the live items in one global order -- query pair index
// descending (for causal attention the heaviest items first), then sequence,
// then head -- are claimed one at a time from a counter, so CTAs that finish
// early take more.  A CTA's claimed ranks only grow, so it maps them to items
// with a cursor that only moves forward: the pair holding the rank, and within
// it the scan position over the sequences long enough for that pair.
struct ItemCursor {
  int pr;               // pair of the ranks [base, end)
  long long base, end;
  int bscan, seen;      // next 32-sequence chunk of pair pr to scan; live sequences before it
};

template <int kTiles>
__device__ __forceinline__ bool seq_reaches(const Params& p, int b, int m0) {
  return b < p.batch && __ldg(p.cu_q + b + 1) - __ldg(p.cu_q + b) > m0;
}

// Map rank r (no smaller than any rank this cursor mapped before) to its item;
// false once r lies past the last live item.  Run by one whole warp.
template <int kTiles>
__device__ bool cursor_map(const Params& p, ItemCursor& c, long long r, int lane, int& b, int& h, int& pair) {
  constexpr int kRows = BM * kTiles;
  while (r >= c.end) {
    if (--c.pr < 0) return false;
    const int m0 = c.pr * kRows;
    int n = 0;
    for (int b0 = 0; b0 < p.batch; b0 += 32)
      n += __popc(__ballot_sync(0xffffffffu, seq_reaches<kTiles>(p, b0 + lane, m0)));
    c.base = c.end;
    c.end = c.base + (long long)n * p.num_heads;
    c.bscan = 0;
    c.seen = 0;
  }
  const long long i = r - c.base;
  const int want = int(i / p.num_heads);
  h = int(i - (long long)want * p.num_heads);
  pair = c.pr;
  const int m0 = c.pr * kRows;
  for (; c.bscan < p.batch; c.bscan += 32) {
    const bool lv = seq_reaches<kTiles>(p, c.bscan + lane, m0);
    const unsigned m = __ballot_sync(0xffffffffu, lv);
    if (c.seen + __popc(m) > want) {
      const unsigned hit = __ballot_sync(0xffffffffu, lv && c.seen + __popc(m & ((1u << lane) - 1u)) == want);
      b = c.bscan + __ffs(hit) - 1;
      return true;
    }
    c.seen += __popc(m);
  }
  return false;  // not reached: want < the pair's live count
}

// kPaged: K/V come from a paged cache through the page table (4-D maps
// {head_dim, kv head, slot, page}); otherwise from packed [tokens, heads, dim].
// kSplit: this instantiation can feed P as head + remainder (p_split 1 and 2).
// kHalfPV (bf16 inputs, packed K/V): P.V in fp16 -- P rounded to fp16, V read
// from an fp16 copy scaled by 2^-e per (sequence, KV head) (pv_emax), and the
// output multiplied by 2^e.
// kPersist: one CTA per SM claiming items (rounded P only: the split kernel's
// softmax and issuer need every register they have, and its per-item build runs
// faster); otherwise one CTA per item.
// The other one is the plain kernel, without the split code in its softmax loop
// (compiled apart: the branch alone cost 13% in the common path).
template <typename T, int D, bool kPaged, bool kSplit, bool kPersist, bool kHalfPV>
__global__ void __launch_bounds__(Layout<D>::kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                   const Params p) {
  using L = Layout<D>;
  constexpr int SK = L::kStagesK, SV = L::kStagesV;
  constexpr int kTiles = L::kTiles, kRowsPerCta = L::kRowsPerCta;
  constexpr int kProducerWarp = L::kProducerWarp, kMmaWarp = L::kMmaWarp;
  constexpr int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t kIdescQK = tc::idesc_f16(BM, BN, fmt, 0, 0);
  constexpr uint32_t kIdescPV = tc::idesc_f16(BM, D, kHalfPV ? 0 : fmt, 0, 1);
  using PT = std::conditional_t<kHalfPV, __half, T>;  // P's 16-bit type

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);  // [kTiles] tiles
  const uint32_t sK = sQ + kTiles * L::kTile;
  const uint32_t sV = sK + SK * L::kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + size_t(L::kTile) * (kTiles + SK + SV));
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t q_full = bar0;
  const uint32_t k_full = bar0 + 8;          // [SK]
  const uint32_t k_empty = k_full + 8 * SK;  // [SK]
  const uint32_t v_full = k_empty + 8 * SK;  // [SV]
  const uint32_t v_empty = v_full + 8 * SV;  // [SV]
  const uint32_t s_full = v_empty + 8 * SV;  // [kTiles]: S_t(j) complete (and every earlier MMA)
  const uint32_t p_full = s_full + 8 * kTiles;  // [kTiles]: P_t(j) written, O_t rescaled; or O_t seen final
  const uint32_t drain = p_full + 8 * kTiles;   // every MMA of the CTA complete
  const uint32_t vtail = drain + 8;             // paged: a partly valid V tile landed (before zeroing its tail)
  const uint32_t never = vtail + 8;             // initialised, never arrived on (failure-path tests)
  const uint32_t q_empty = never + 8;           // an item's last Q.K^T completed: its Q buffers are free
  const uint32_t item_full = q_empty + 8;                 // [kItemSlots]: the producer published an item
  const uint32_t item_empty = item_full + 8 * kItemSlots;  // [kItemSlots]: every consumer is done with it
  volatile uint32_t* tmem_slot =
      reinterpret_cast<volatile uint32_t*>(bars + 1 + 2 * SK + 2 * SV + 2 * kTiles + 4 + 2 * kItemSlots);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Split votes of the softmax warps, read by the MMA issuer after p_full:
  // [tile][warp of the warpgroup][key tile parity].
  volatile int* votes = reinterpret_cast<volatile int*>(tmem_slot + 2);
  // Published items (persistent grid): [slot][8] ints, see work_from_slot.
  volatile int* slots = votes + 8 * kTiles;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // One CTA per item: this CTA's (sequence, head, pair).
  const int own_b = blockIdx.x / p.num_heads, own_h = blockIdx.x % p.num_heads;
  const int own_pair = gridDim.y - 1 - blockIdx.y;  // heaviest (latest) query tiles start first
  if (!kPersist) {
    // Paged: a length past the page table is cut to its capacity (and reported),
    // so tile positions stay in 32 bits and inside the table.
    if (kPaged && tid == 0 && __ldg(p.seq_lens_k + own_b) > p.cap_tokens) raise_error(p.err, FAT_DEVERR_BAD_LENGTH);
    if (own_pair * kRowsPerCta >= __ldg(p.cu_q + own_b + 1) - __ldg(p.cu_q + own_b)) return;  // before any barrier
    // The item goes to slot 0 now, so no role waits on these loads after the barrier setup.
    if (tid == 0) write_slot(slots, describe_work<kTiles, kPaged>(p, own_b, own_h, own_pair), own_pair, true);
  }

  if (warp == kMmaWarp) {
    tc::tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_slot)), kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < SK; ++s) {
      mbar_init(k_full + 8 * s, 1);
      mbar_init(k_empty + 8 * s, 1);
    }
    for (int s = 0; s < SV; ++s) {
      mbar_init(v_full + 8 * s, 1);
      mbar_init(v_empty + 8 * s, 1);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(s_full + 8 * t, 1);
      mbar_init(p_full + 8 * t, kSoftmaxThreads);
    }
    mbar_init(drain, 1);
    mbar_init(vtail, 1);
    mbar_init(never, 1);
    mbar_init(q_empty, 1);
    for (int e = 0; e < kItemSlots; ++e) {
      mbar_init(item_full + 8 * e, 1);
      mbar_init(item_empty + 8 * e, 1 + 4 * kTiles);  // the MMA issuer and every softmax warp
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // Item k as the consumers (MMA issuer, softmax warps) see it: the CTA's own
  // item (one CTA per item, k == 0 only), or ring slot k % kItemSlots once the
  // producer has published it.  False when there is no item k (or a wait failed).
  auto consumer_item = [&](int k, Work& w, bool& ok) -> bool {
    if (!kPersist) {
      if (k > 0) return false;
      w = work_from_slot<kTiles>(p, slots);
      return true;
    }
    const int e = k % kItemSlots;
    if (!mbar_wait_bounded(item_full + 8 * e, (k / kItemSlots) & 1, p.err, abort_flag, p.wait_ns)) {
      ok = false;
      return false;
    }
    if (slots[8 * e] < 0) return false;
    w = work_from_slot<kTiles>(p, slots + 8 * e);
    return true;
  };
  // The same item again, once consumer_item(k) returned it and before release_item(k).
  auto peek_item = [&](int k) { return work_from_slot<kTiles>(p, slots + 8 * (k % kItemSlots)); };
  auto release_item = [&](int k) {
    if (kPersist) mbar_arrive(item_empty + 8 * (k % kItemSlots));
  };

  if (warp >= kProducerWarp) {
    if constexpr (L::kSplitRegs) regs_dec<L::kRegsOther>();
    if (warp == kProducerWarp) {
      // ============================ TMA producer ============================
      // The whole warp: it claims and describes the items (persistent grid) and
      // publishes them to the consumers.  Ring positions and phases run on
      // across items; an item's Q waits until the previous item's last Q.K^T
      // has read the Q buffers (q_empty).  Packed K/V: lane 0 issues the copies.
      // Paged K/V: lane l brings token rows [l' * rows_per_box, ...) of column
      // block cb (l = l' * kCB + cb) of one K or V tile from its page.
      [[maybe_unused]] const int rpb = p.rows_per_box;
      [[maybe_unused]] const int pages_per_tile = kPaged ? BN / rpb : 0;
      [[maybe_unused]] const int i_page = lane / L::kCB, cb = lane - i_page * L::kCB;
      int issued_k = 0, issued_v = 0, tails = 0, loads_q = 0;
      if (lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
      }
      ItemCursor cur{p.num_pairs, 0, 0, 0, 0};
      int claimed = 0;  // lane 0: the rank claimed for the next item
      if (kPersist) {
        if (kPaged && blockIdx.x == 0)
          for (int b = lane; b < p.batch; b += 32)
            if (__ldg(p.seq_lens_k + b) > p.cap_tokens) raise_error(p.err, FAT_DEVERR_BAD_LENGTH);
        if (lane == 0) claimed = atomicAdd(p.sched, 1);
      }
      bool ok = true;
      for (int k = 0; ok && (kPersist || k < 1); ++k) {
        Work w{};
        bool have;
        if (!kPersist) {
          have = k == 0;
          if (have) w = work_from_slot<kTiles>(p, slots);
        } else {
          const long long r = __shfl_sync(0xffffffffu, claimed, 0);
          int b = 0, h = 0, pair = 0;
          have = cursor_map<kTiles>(p, cur, r, lane, b, h, pair);
          // Claim the next rank now: its round trip overlaps this item's copies.
          if (have && lane == 0) claimed = atomicAdd(p.sched, 1);
          if (have) w = describe_work<kTiles, kPaged>(p, b, h, pair);
          if (lane == 0) {
            const int e = k % kItemSlots;
            ok = mbar_wait_bounded(item_empty + 8 * e, ((k / kItemSlots) & 1) ^ 1, p.err, abort_flag, p.wait_ns);
            if (ok) {
              write_slot(slots + 8 * e, w, pair, have);
              mbar_arrive(item_full + 8 * e);
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
        }
        if (!have || !ok) break;
        if (w.n_max == 0) continue;
        if (lane == 0) {
          if (loads_q > 0) ok = mbar_wait_bounded(q_empty, (loads_q - 1) & 1, p.err, abort_flag, p.wait_ns);
          if (ok) {
            mbar_arrive_expect_tx(q_full, w.q_tiles * L::kTile);
            for (int t = 0; t < w.q_tiles; ++t)
#pragma unroll
              for (int c2 = 0; c2 < L::kCB; ++c2)
                tma_load_3d(sQ + t * L::kTile + c2 * BM * 128, &tm_q, q_full, c2 * 64, w.h, w.q0 + w.m0 + t * BM);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        ++loads_q;
        if constexpr (!kPaged) {
          if (lane == 0) {
            for (int j = 0; j < w.n_max; ++j) {
              const int sk = issued_k % SK, sv = issued_v % SV;
              if (!mbar_wait_bounded(k_empty + 8 * sk, ((issued_k / SK) & 1) ^ 1, p.err, abort_flag, p.wait_ns)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(k_full + 8 * sk, L::kTile);
#pragma unroll
              for (int c2 = 0; c2 < L::kCB; ++c2)
                tma_load_3d(sK + sk * L::kTile + c2 * BN * 128, &tm_k, k_full + 8 * sk, c2 * 64, w.kvh, w.k0 + j * BN);
              ++issued_k;
              if (!mbar_wait_bounded(v_empty + 8 * sv, ((issued_v / SV) & 1) ^ 1, p.err, abort_flag, p.wait_ns)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(v_full + 8 * sv, L::kTile);
#pragma unroll
              for (int c2 = 0; c2 < L::kCB; ++c2)
                tma_load_3d(sV + sv * L::kTile + c2 * BN * 128, &tm_v, v_full + 8 * sv, c2 * 64, w.kvh, w.k0 + j * BN);
              ++issued_v;
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
        } else {
          const int kv_len = w.kv_len;
          for (int j = 0; j < w.n_max; ++j) {
            const int sk = issued_k % SK, sv = issued_v % SV;
            const int tok0 = j * BN;
            const int valid_rows = min(BN, kv_len - tok0);
            // This lane's page: rows [tok0 + i_page * rpb, + rpb) of the sequence.
            const int row0 = i_page * rpb;
            int page = -1, slot0 = 0;
            if (i_page < pages_per_tile && row0 < valid_rows) {
              const int tok = tok0 + row0;
              const int lp = tok / p.page_size;
              slot0 = tok - lp * p.page_size;
              if (lp < p.max_pages) page = __ldg(p.page_table + (long long)w.b * p.pt_sb + lp);
              if (page < 0 || page >= p.num_pages) {
                raise_error(p.err, FAT_DEVERR_BAD_PAGE);
                page = -1;
              }
            }
            const unsigned loaded = __ballot_sync(0xffffffffu, page >= 0 && cb == 0);
            const uint32_t bytes = uint32_t(__popc(loaded)) * uint32_t(rpb) * 128u * L::kCB;
            // Rows no copy fills (past the sequence, or on a rejected page) are
            // zeroed in V so that p = 0 there contributes exactly nothing.
            const bool tail = valid_rows < BN || __popc(loaded) * rpb < BN;
            // K tile j.
            if (lane == 0)
              ok = mbar_wait_bounded(k_empty + 8 * sk, ((issued_k / SK) & 1) ^ 1, p.err, abort_flag, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            if (lane == 0) mbar_arrive_expect_tx(k_full + 8 * sk, bytes);
            __syncwarp();
            if (page >= 0)
              tma_load_4d(sK + sk * L::kTile + cb * BN * 128 + row0 * 128, &tm_k, k_full + 8 * sk, cb * 64, w.kvh,
                          slot0, page);
            ++issued_k;
            // V tile j.
            if (lane == 0)
              ok = mbar_wait_bounded(v_empty + 8 * sv, ((issued_v / SV) & 1) ^ 1, p.err, abort_flag, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            const uint32_t vbar = tail ? vtail : v_full + 8 * sv;
            if (lane == 0) mbar_arrive_expect_tx(vbar, bytes);
            __syncwarp();
            if (page >= 0)
              tma_load_4d(sV + sv * L::kTile + cb * BN * 128 + row0 * 128, &tm_v, vbar, cb * 64, w.kvh, slot0, page);
            ++issued_v;
            if (tail) {
              ++tails;
              if (lane == 0) ok = mbar_wait_bounded(vtail, (tails - 1) & 1, p.err, abort_flag, p.wait_ns);
              ok = __shfl_sync(0xffffffffu, ok, 0);
              if (!ok) break;
              // Zero every row no copy filled or that lies past the sequence end
              // (16-byte stores; the swizzle does not matter for zeros), then
              // publish the tile to the async proxy.
              const uint32_t vt = sV + sv * L::kTile;
              for (int i = lane; i < L::kCB * BN * 8; i += 32) {
                const int c2 = i / (BN * 8), r = (i / 8) % BN;
                const bool filled = ((loaded >> ((r / rpb) * L::kCB)) & 1u) != 0;
                if (!filled || r >= valid_rows) {
                  const uint32_t a = vt + uint32_t(c2 * BN * 128 + r * 128 + (i % 8) * 16);
                  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0) : "memory");
                }
              }
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) mbar_arrive(v_full + 8 * sv);
            }
          }
        }
      }
      if (*abort_flag && lane == 0) {
        // Drain this CTA's own copies before the shared memory goes away.
        if (loads_q > 0) mbar_wait_bounded(q_full, (loads_q - 1) & 1, nullptr, nullptr, p.wait_ns);
        for (int j = max(0, issued_k - SK); j < issued_k; ++j)
          mbar_wait_bounded(k_full + 8 * (j % SK), (j / SK) & 1, nullptr, nullptr, p.wait_ns);
        for (int j = max(0, issued_v - SV); j < issued_v; ++j)
          mbar_wait_bounded(v_full + 8 * (j % SV), (j / SV) & 1, nullptr, nullptr, p.wait_ns);
        if (tails > 0) mbar_wait_bounded(vtail, (tails - 1) & 1, nullptr, nullptr, p.wait_ns);
      }
    } else if (warp == kMmaWarp && lane == 0) {
      // ============================ MMA issuer ============================
      // The issue loop is kept lean (the tensor core retires an M128 N128 K16
      // MMA every 64 cycles, so per-MMA address arithmetic shows up directly
      // as idle tensor time): descriptor words are built once, and operands
      // move by adding (byte offset >> 4) to the 14-bit start-address field in
      // the low word (no carry: the shared window is below 2^18 bytes).
      const uint64_t dK = tc::sdesc_sw128(sK, 16, 1024);  // Q uses the same layout words
      const uint64_t dV = tc::sdesc_sw128(sV, BN * 128, 1024);
      const uint32_t hiK = uint32_t(dK >> 32), loK0 = uint32_t(dK);
      const uint32_t hiV = uint32_t(dV >> 32), loV0 = uint32_t(dV);
      const uint32_t loQ0 = uint32_t(tc::sdesc_sw128(sQ, 16, 1024));
      constexpr uint32_t kTileDesc = uint32_t(L::kTile) >> 4;
      auto desc = [](uint32_t lo, uint32_t hi) { return (uint64_t(hi) << 32) | lo; };
      auto issue_s = [&](uint32_t d_tmem, uint32_t loQ, uint32_t loK) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = uint32_t(((kk >> 2) * (BM * 128) + (kk & 3) * 32) >> 4);
          tc::mma_ss(d_tmem, desc(loQ + off, hiK), desc(loK + off, hiK), kIdescQK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](uint32_t d_tmem, uint32_t a_tmem, uint32_t loV, uint32_t acc0) {
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          tc::mma_ts(d_tmem, a_tmem + kk * 8, desc(loV + uint32_t((kk * 16 * 128) >> 4), hiV), kIdescPV,
                     kk > 0 ? 1u : acc0);
      };
      // P.V of key tile jj of query tile t: the head in columns [0, 64) of the
      // tile's S area, and for a split tile the remainder in columns [64, 128)
      // accumulated on top (votes are visible: p_full's arrivals release them).
      auto issue_p = [&](uint32_t d_tmem, uint32_t a_tmem, uint32_t loV, int jj, int t) {
        issue_pv(d_tmem, a_tmem, loV, jj > 0 ? 1u : 0u);
        if constexpr (kSplit) {
          bool split = p.p_split == 2;
          if (p.p_split == 1) {
            const volatile int* v = votes + t * 8 + (jj & 1);
            split = (v[0] | v[2] | v[4] | v[6]) != 0;
          }
          if (split) issue_pv(d_tmem, a_tmem + BN / 2, loV, 1u);
        }
      };
      int sk = 0, kph = 0, sv = 0, vph = 0, pph0 = 0, pph1 = 0, items_q = 0;
      // ack_t: tile t's softmax has yet to confirm it saw its previous item's
      // final phase (its p_full arrival); S_t of the next item waits for it, so
      // no s_full phase of tile t completes unobserved.
      bool ack0 = false, ack1 = false;
      // Failure-path test: a wait that nothing ends runs out after p.wait_ns and
      // raises the abort flag; the other roles stop at their next wait.
      if (p.expire) mbar_wait_bounded(never, 0, p.err, abort_flag, p.wait_ns);
      bool ok = true;
      for (int it = 0; ok && (kPersist || it < 1); ++it) {
        Work w;
        if (!consumer_item(it, w, ok)) break;
        release_item(it);  // read: the slot is free again as far as the issuer goes
        const int n0 = w.n0, n1 = w.n1, n_max = w.n_max;
        if (n_max == 0) continue;
        if (!mbar_wait_bounded(q_full, items_q & 1, p.err, abort_flag, p.wait_ns)) break;
        ++items_q;
        for (int j = 0; j <= n_max; ++j) {
          if (j < n_max && !mbar_wait_bounded(k_full + 8 * sk, kph, p.err, abort_flag, p.wait_ns)) {
            ok = false;
            break;
          }
          const uint32_t loK = loK0 + uint32_t(sk) * kTileDesc;
          const uint32_t loV = loV0 + uint32_t(sv) * kTileDesc;
          bool v_ready = false;
          // ---- tile 0: O0 += P0 V_{j-1}, then S0 = Q0 K_j^T ----
          if (j >= 1 && j <= n0) {
            if (!mbar_wait_bounded(p_full, pph0, p.err, abort_flag, p.wait_ns) ||
                !mbar_wait_bounded(v_full + 8 * sv, vph, p.err, abort_flag, p.wait_ns)) {
              ok = false;
              break;
            }
            pph0 ^= 1;
            v_ready = true;
            tc::fence_after_sync();
            issue_p(tmem + L::kColO, tmem + L::kColS, loV, j - 1, 0);
          }
          if (j < n0) {
            if (j == 0 && ack0) {
              if (!mbar_wait_bounded(p_full, pph0, p.err, abort_flag, p.wait_ns)) {
                ok = false;
                break;
              }
              pph0 ^= 1;
              ack0 = false;
            }
            tc::fence_after_sync();
            issue_s(tmem + L::kColS, loQ0, loK);
          }
          // One s_full phase per S0 and one more after the last P.V: the softmax
          // warps then know O0 is final.
          if (j <= n0 && (j < n0 || j > 0)) tc::commit(s_full);
          // ---- tile 1 ----
          if (j >= 1 && j <= n1) {
            if (!mbar_wait_bounded(p_full + 8, pph1, p.err, abort_flag, p.wait_ns) ||
                (!v_ready && !mbar_wait_bounded(v_full + 8 * sv, vph, p.err, abort_flag, p.wait_ns))) {
              ok = false;
              break;
            }
            pph1 ^= 1;
            tc::fence_after_sync();
            issue_p(tmem + L::kColO + 128, tmem + L::kColS + 128, loV, j - 1, 1);
          }
          if (j < n1) {
            if (j == 0 && ack1) {
              if (!mbar_wait_bounded(p_full + 8, pph1, p.err, abort_flag, p.wait_ns)) {
                ok = false;
                break;
              }
              pph1 ^= 1;
              ack1 = false;
            }
            tc::fence_after_sync();
            issue_s(tmem + L::kColS + 128, loQ0 + kTileDesc, loK);
          }
          if (j <= n1 && (j < n1 || j > 0)) tc::commit(s_full + 8);
          // The item's Q buffers are free once its last Q.K^T completes.
          if (j == n_max - 1) tc::commit(q_empty);
          // ---- release the tiles this iteration consumed ----
          if (j >= 1) {  // V_{j-1}
            tc::commit(v_empty + 8 * sv);
            if (++sv == SV) {
              sv = 0;
              vph ^= 1;
            }
          }
          if (j < n_max) {  // K_j
            tc::commit(k_empty + 8 * sk);
            if (++sk == SK) {
              sk = 0;
              kph ^= 1;
            }
          }
        }
        ack0 = ack0 || n0 > 0;
        ack1 = ack1 || n1 > 0;
      }
      // Every MMA this thread issued has finished once `drain` completes.
      tc::commit(drain);
      mbar_wait_bounded(drain, 0, nullptr, nullptr, p.wait_ns);
    }
  } else {
    if constexpr (L::kSplitRegs) regs_inc<L::kRegsSoftmax>();
    // ============================ softmax warpgroups ============================
    const int t = warp >> 2;              // query tile of this warpgroup
    const int row = tid & 127;            // row of the tile = tensor-memory lane
    const uint32_t lane_base = tmem + (uint32_t((warp & 3) * 32) << 16);
    const uint32_t colS = L::kColS + 128 * t, colO = L::kColO + 128 * t;
    const uint32_t sbar = s_full + 8 * t, pbar = p_full + 8 * t;
    uint32_t sph = 0;  // parity of the next s_full phase of this tile (runs on across items)
    bool ok = true;
    for (int it = 0; ok && (kPersist || it < 1); ++it) {
      int n_t, lim;  // K/V tiles of this tile; last key this row may see (inclusive)
      {
        Work w;
        if (!consumer_item(it, w, ok)) break;
        n_t = t == 0 ? w.n0 : w.n1;
        const int q_idx = w.m0 + t * BM + row;
        lim = p.causal ? min(w.kv_len - 1, q_idx + w.offset) : w.kv_len - 1;
      }
      float m_used = -CUDART_INF_F, l_sum = 0.f;
      for (int j = 0; j < n_t; ++j) {
        if (!mbar_wait_bounded(sbar, sph, p.err, abort_flag, p.wait_ns)) {
          ok = false;
          break;
        }
        sph ^= 1;
        tc::fence_after_sync();
        float s[BN];
        {
          uint32_t r[BN / 32][32];
#pragma unroll
          for (int c = 0; c < BN / 32; ++c) tc::ld32(lane_base + colS + 32 * c, r[c]);
          tc::wait_ld();
#pragma unroll
          for (int c = 0; c < BN / 32; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i) s[32 * c + i] = __uint_as_float(r[c][i]);
        }
        const int kv0 = j * BN;
        if (kv0 + BN - 1 > lim) {
#pragma unroll
          for (int i = 0; i < BN; ++i) s[i] = (kv0 + i <= lim) ? s[i] : -CUDART_INF_F;
        }
        float mx;
        {
          // Four independent chains over the BN scores: blocks of 8 from 0.
          static_assert(BN % 8 == 0, "row max works on blocks of 8 scores");
          float a0 = fmaxf(s[0], s[4]), a1 = fmaxf(s[1], s[5]), a2 = fmaxf(s[2], s[6]), a3 = fmaxf(s[3], s[7]);
#pragma unroll
          for (int i = 8; i < BN; i += 8) {
            a0 = max3(a0, s[i], s[i + 4]);
            a1 = max3(a1, s[i + 1], s[i + 5]);
            a2 = max3(a2, s[i + 2], s[i + 6]);
            a3 = max3(a3, s[i + 3], s[i + 7]);
          }
          mx = fmaxf(max3(a0, a1, a2), a3);
        }
        mx *= p.scale_log2;
        float factor = 1.f;
        bool grow = false;
        if (mx > m_used + kRescaleThreshold) {
          factor = (m_used == -CUDART_INF_F) ? 1.f : fast_exp2(m_used - mx);
          grow = m_used != -CUDART_INF_F;
          m_used = mx;
          l_sum *= factor;
        }
        if (__any_sync(0xffffffffu, grow)) {
          // S_t(j) is complete, so O_t holds every earlier P.V: rescale in place.
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            tc::ld32(lane_base + colO + 32 * c, r);
            tc::wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
            tc::st32(lane_base + colO + 32 * c, r);
          }
        }
        const float msub = (m_used == -CUDART_INF_F) ? 0.f : m_used;
        float sum0 = 0.f, sum1 = 0.f, sum2 = 0.f, sum3 = 0.f;
        if constexpr (!kSplit) {
          // P rounded to the input dtype (prefill.py:128), packed over S's first 64 columns.
#pragma unroll
          for (int c = 0; c < BN / 64; ++c) {
            uint32_t packed[32];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float x0, x1, x2, x3;
              fma2(x0, x1, s[64 * c + 2 * i], s[64 * c + 2 * i + 1], p.scale_log2, -msub);
              fma2(x2, x3, s[64 * c + 2 * i + 2], s[64 * c + 2 * i + 3], p.scale_log2, -msub);
              const float p0 = fast_exp2(x0);
              const float p1 = fast_exp2(x1);
              const float p2 = fast_exp2(x2);
              const float p3 = fast_exp2(x3);
              add2(sum0, sum1, p0, p1);
              add2(sum2, sum3, p2, p3);
              packed[i] = pack2<PT>(p0, p1);
              packed[i + 1] = pack2<PT>(p2, p3);
            }
            tc::st32(lane_base + colS + 32 * c, packed);
          }
          l_sum += (sum0 + sum1) + (sum2 + sum3);
        } else {
          // Decided before the exponentials: the row's sum after this tile is at
          // least its sum so far plus the tile's largest p, so a key of an unsplit
          // tile still ends with weight <= kSplitTheta.
          bool split = p.p_split == 2;
          if (p.p_split == 1) {
            const float pmax = fast_exp2(mx - msub);
            split = __any_sync(0xffffffffu, pmax > kSplitTheta * (l_sum + pmax));
          }
          if (!split) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) {
              uint32_t packed[32];
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                float x0, x1, x2, x3;
                fma2(x0, x1, s[64 * c + 2 * i], s[64 * c + 2 * i + 1], p.scale_log2, -msub);
                fma2(x2, x3, s[64 * c + 2 * i + 2], s[64 * c + 2 * i + 3], p.scale_log2, -msub);
                const float p0 = fast_exp2(x0);
                const float p1 = fast_exp2(x1);
                const float p2 = fast_exp2(x2);
                const float p3 = fast_exp2(x3);
                add2(sum0, sum1, p0, p1);
                add2(sum2, sum3, p2, p3);
                packed[i] = pack2<T>(p0, p1);
                packed[i + 1] = pack2<T>(p2, p3);
              }
              tc::st32(lane_base + colS + 32 * c, packed);
            }
            if (p.p_split == 1) {
              // Another warp of this tile may vote to split: the remainder pass then
              // reads these rows' columns [64, 128), which must hold zeros.
              uint32_t zero[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) zero[i] = 0u;
              tc::st32(lane_base + colS + BN / 2, zero);
              tc::st32(lane_base + colS + BN / 2 + 32, zero);
            }
          } else {
            // Head in columns [0, 64), remainder p - head in [64, 128): every score
            // of this S row is already in registers, so those columns are free.
#pragma unroll
            for (int c = 0; c < BN / 32; ++c) {
              uint32_t hi[16], lo[16];
#pragma unroll
              for (int i = 0; i < 16; i += 2) {
                float x0, x1, x2, x3;
                fma2(x0, x1, s[32 * c + 2 * i], s[32 * c + 2 * i + 1], p.scale_log2, -msub);
                fma2(x2, x3, s[32 * c + 2 * i + 2], s[32 * c + 2 * i + 3], p.scale_log2, -msub);
                const float p0 = fast_exp2(x0);
                const float p1 = fast_exp2(x1);
                const float p2 = fast_exp2(x2);
                const float p3 = fast_exp2(x3);
                add2(sum0, sum1, p0, p1);
                add2(sum2, sum3, p2, p3);
                split_hi_lo<T>(p0, p1, hi[i], lo[i]);
                split_hi_lo<T>(p2, p3, hi[i + 1], lo[i + 1]);
              }
              tc::st16(lane_base + colS + 16 * c, hi);
              tc::st16(lane_base + colS + BN / 2 + 16 * c, lo);
            }
          }
          l_sum += (sum0 + sum1) + (sum2 + sum3);
          if (p.p_split == 1 && lane == 0) votes[t * 8 + (warp & 3) * 2 + (j & 1)] = split ? 1 : 0;
        }
        tc::wait_st();
        tc::fence_before_sync();
        mbar_arrive(pbar);
      }
      // ---- epilogue: O / l -> global, once the last P.V of this tile completed ----
      // (the item is described again here, so nothing of it stays live in the loop)
      const Work w = peek_item(it);
      const int q0 = w.q0, q_len = w.q_len, m0 = w.m0, h = w.h;
      // Only a CTA's single item (one CTA per item) may stage O in its Q buffers:
      // in the persistent grid the producer refills them for the next item.
      const bool last = !kPersist;
      const int q_idx = m0 + t * BM + row;
      bool fin = false;
      if (ok && n_t > 0) {
        fin = mbar_wait_bounded(sbar, sph, p.err, abort_flag, p.wait_ns);
        if (fin) {
          sph ^= 1;
          // Seen final: the issuer may now start this tile's next item (S_t only;
          // O_t is overwritten after this tile's next P arrives).
          mbar_arrive(pbar);
        } else {
          ok = false;
        }
      }
      // A warp whose 32 rows all belong to the sequence stages them, 16-bit and
      // 128-byte swizzled, in its rows of the tile's Q buffer (unused once the
      // tile's last MMA completed) and stores them with one TMA copy per 64
      // columns: whole 128-byte lines leave instead of each store instruction
      // touching 32 rows' lines with 16 bytes.  Rows of a partial group (the
      // next sequence's rows follow in out) take the direct stores below.
      const int wrow0 = m0 + t * BM + 32 * (warp & 3);
      if (p.o_tma && last && n_t > 0 && wrow0 + 32 <= q_len) {
        if (__all_sync(0xffffffffu, fin)) {
          tc::fence_after_sync();
          const float inv = (l_sum > 0.f ? 1.f / l_sum : 0.f) * pv_unscale<kHalfPV>(p, w);
          const uint32_t qt = sQ + uint32_t(t * L::kTile);
#pragma unroll
          for (int c = 0; c < D / 32; c += 2) {
            uint32_t r[2][32];
            tc::ld32(lane_base + colO + 32 * c, r[0]);
            tc::ld32(lane_base + colO + 32 * (c + 1), r[1]);
            tc::wait_ld();
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const uint32_t blk = qt + uint32_t(((c + u) >> 1) * BM * 128);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint32_t* x = r[u] + 8 * i;
                st_shared_v4(blk + swz128(uint32_t(row), uint32_t(((c + u) & 1) * 4 + i)),
                             pack2<T>(__uint_as_float(x[0]) * inv, __uint_as_float(x[1]) * inv),
                             pack2<T>(__uint_as_float(x[2]) * inv, __uint_as_float(x[3]) * inv),
                             pack2<T>(__uint_as_float(x[4]) * inv, __uint_as_float(x[5]) * inv),
                             pack2<T>(__uint_as_float(x[6]) * inv, __uint_as_float(x[7]) * inv));
              }
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
#pragma unroll
            for (int cb = 0; cb < L::kCB; ++cb)
              tma_store_3d(&tm_o, qt + uint32_t(cb * BM * 128 + (warp & 3) * 32 * 128), cb * 64, h, q0 + wrow0);
            bulk_commit_group();
            bulk_wait_read_all();
          }
        }
      } else if (fin) {
        tc::fence_after_sync();
        const float inv = (l_sum > 0.f ? 1.f / l_sum : 0.f) * pv_unscale<kHalfPV>(p, w);
        const bool store = q_idx < q_len;
        const long long base = (long long)(q0 + q_idx) * p.o_st + (long long)h * p.o_sh;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tc::ld32(lane_base + colO + 32 * c, r);
          tc::wait_ld();
          if (store) {
            if (p.out_f32) {
              float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + base + 32 * c);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                dst[i] = make_float4(__uint_as_float(r[4 * i]) * inv, __uint_as_float(r[4 * i + 1]) * inv,
                                     __uint_as_float(r[4 * i + 2]) * inv, __uint_as_float(r[4 * i + 3]) * inv);
            } else {
              uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + base + 32 * c);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                uint4 v;
                v.x = pack2<T>(__uint_as_float(r[8 * i + 0]) * inv, __uint_as_float(r[8 * i + 1]) * inv);
                v.y = pack2<T>(__uint_as_float(r[8 * i + 2]) * inv, __uint_as_float(r[8 * i + 3]) * inv);
                v.z = pack2<T>(__uint_as_float(r[8 * i + 4]) * inv, __uint_as_float(r[8 * i + 5]) * inv);
                v.w = pack2<T>(__uint_as_float(r[8 * i + 6]) * inv, __uint_as_float(r[8 * i + 7]) * inv);
                dst[i] = v;
              }
            }
          }
        }
      } else if (n_t == 0 && q_idx < q_len) {
        // No visible keys (only reachable with invalid causal inputs): zeros.
        const long long base = (long long)(q0 + q_idx) * p.o_st + (long long)h * p.o_sh;
        for (int d = 0; d < D; ++d) {
          if (p.out_f32) {
            reinterpret_cast<float*>(p.out)[base + d] = 0.f;
          } else {
            reinterpret_cast<T*>(p.out)[base + d] = from_float<T>(0.f);
          }
        }
      }
      __syncwarp();
      if (lane == 0) release_item(it);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == kMmaWarp) tc::tmem_dealloc(tmem, kTmemCols);
  if (kPersist && tid == 0) {
    // The last CTA to finish zeroes the counters for the next launch on this stream.
    __threadfence();
    if (atomicAdd(p.sched + 1, 1) == int(gridDim.x) - 1) {
      atomicExch(p.sched, 0);
      atomicExch(p.sched + 1, 0);
    }
  }
}

// ---- kHalfPV pre-pass: bf16 V -> fp16 copy scaled per (sequence, KV head) ----
// Block (x, y): tokens [64 x, 64 x + 64) of KV head y; thread i takes the
// 16-byte vectors i, i + 256, ... of that 64-row slab (all loads issued first).
// A slab inside one sequence (the common case) looks its sequence up once.
constexpr int kVRows = 64;
constexpr int kVThreads = 256;

// The sequence of packed token t: the largest b with cu[b] <= t.
__device__ __forceinline__ int seq_of_token(const int* cu, int batch, long long t) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(cu + mid) <= t) {
      lo = mid;
    } else {
      hi = mid - 1;
    }
  }
  return lo;
}

// A bf16 magnitude (sign cleared), or 0 for inf and NaN (exponent bits all ones).
__device__ __forceinline__ unsigned finite_mag(unsigned mag) { return mag < 0x7f80u ? mag : 0u; }

template <int D>
struct VSlab {
  static constexpr int kVecs = D / 8;                          // 16-byte vectors per token row
  static constexpr int kPerThread = kVRows * kVecs / kVThreads;  // vectors per thread
  static_assert(kVRows * kVecs % kVThreads == 0, "slab splits evenly");
};

// The slab's sequence when all its tokens belong to one, else -1.
__device__ __forceinline__ int slab_sequence(const int* cu_k, int batch, long long t0, long long total_k) {
  __shared__ int seq;
  if (threadIdx.x == 0) {
    const long long t1 = min(t0 + kVRows, total_k) - 1;
    const int b0 = seq_of_token(cu_k, batch, t0), b1 = seq_of_token(cu_k, batch, t1);
    seq = b0 == b1 ? b0 : -1;
  }
  __syncthreads();
  return seq;
}

// Largest finite |v| per (sequence, KV head) as bf16 bits without the sign (a
// bf16 magnitude orders like its bit pattern), into emax (zeroed before): one
// atomic per slab (per token in a slab that straddles sequences).  inf and NaN
// are left out: they convert to fp16 inf and NaN whatever the scale, and a
// scale set by them would flush every finite value of the sequence to zero.
template <int D>
__global__ void __launch_bounds__(kVThreads) v_absmax_kernel(const uint16_t* v, long long v_st, long long v_sh,
                                                             const int* cu_k, int batch, int num_kv_heads,
                                                             long long total_k, unsigned* emax) {
  using S = VSlab<D>;
  const int kvh = blockIdx.y;
  const long long t0 = (long long)blockIdx.x * kVRows;
  uint4 x[S::kPerThread];  // loads first: the sequence lookup overlaps their latency
#pragma unroll
  for (int i = 0; i < S::kPerThread; ++i) {
    const int idx = threadIdx.x + i * kVThreads, r = idx / S::kVecs, c = idx % S::kVecs;
    x[i] = make_uint4(0u, 0u, 0u, 0u);
    if (t0 + r < total_k) x[i] = __ldg(reinterpret_cast<const uint4*>(v + (t0 + r) * v_st + kvh * v_sh + c * 8));
  }
  const int seq = slab_sequence(cu_k, batch, t0, total_k);
  unsigned mt = 0;
#pragma unroll
  for (int i = 0; i < S::kPerThread; ++i) {
    const uint32_t w[4] = {x[i].x, x[i].y, x[i].z, x[i].w};
    unsigned m = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) m = max(m, max(finite_mag(w[k] & 0x7fffu), finite_mag((w[k] >> 16) & 0x7fffu)));
    if (seq >= 0) {
      mt = max(mt, m);
    } else {
      const int r = (threadIdx.x + i * kVThreads) / S::kVecs;
      if (t0 + r < total_k)
        atomicMax(emax + (long long)seq_of_token(cu_k, batch, t0 + r) * num_kv_heads + kvh, m);
    }
  }
  if (seq >= 0) {
    __shared__ unsigned red[kVThreads / 32];
    mt = __reduce_max_sync(0xffffffffu, mt);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mt;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned m = 0;
#pragma unroll
      for (int w = 0; w < kVThreads / 32; ++w) m = max(m, red[w]);
      atomicMax(emax + (long long)seq * num_kv_heads + kvh, m);
    }
  }
}

// v16[t, kvh, :] = fp16(v[t, kvh, :] * 2^-e), e = pv_exponent(emax[b, kvh]): the
// product is exact in fp32 (a power of two), below 2^15, and its fp16 rounding
// is exact down to 2^-14 (smaller values, under 2^-28 of the row's largest,
// keep an absolute error under 2^-25 of the scale).
template <int D>
__global__ void __launch_bounds__(kVThreads) v_to_half_kernel(const uint16_t* v, long long v_st, long long v_sh,
                                                              const int* cu_k, int batch, int num_kv_heads,
                                                              long long total_k, const unsigned* emax,
                                                              uint16_t* v16) {
  using S = VSlab<D>;
  const int kvh = blockIdx.y;
  const long long t0 = (long long)blockIdx.x * kVRows;
  uint4 x[S::kPerThread];  // loads first: the sequence lookup overlaps their latency
#pragma unroll
  for (int i = 0; i < S::kPerThread; ++i) {
    const int idx = threadIdx.x + i * kVThreads, r = idx / S::kVecs, c = idx % S::kVecs;
    x[i] = make_uint4(0u, 0u, 0u, 0u);
    if (t0 + r < total_k) x[i] = __ldg(reinterpret_cast<const uint4*>(v + (t0 + r) * v_st + kvh * v_sh + c * 8));
  }
  const int seq = slab_sequence(cu_k, batch, t0, total_k);
  const float f_slab = seq >= 0 ? __int_as_float((127 - pv_exponent(__ldg(emax + (long long)seq * num_kv_heads + kvh)))
                                                 << 23)
                                : 0.f;
#pragma unroll
  for (int i = 0; i < S::kPerThread; ++i) {
    const int idx = threadIdx.x + i * kVThreads, r = idx / S::kVecs, c = idx % S::kVecs;
    const long long t = t0 + r;
    if (t >= total_k) continue;
    float f = f_slab;  // 2^-e
    if (seq < 0)
      f = __int_as_float((127 - pv_exponent(__ldg(emax + (long long)seq_of_token(cu_k, batch, t) * num_kv_heads +
                                                   kvh)))
                         << 23);
    const uint32_t w[4] = {x[i].x, x[i].y, x[i].z, x[i].w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      o[k] = pack2<__half>(__uint_as_float(w[k] << 16) * f, __uint_as_float(w[k] & 0xffff0000u) * f);
    *reinterpret_cast<uint4*>(v16 + (t * num_kv_heads + kvh) * D + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace pre

// =============================================================================
// Host side
// =============================================================================
namespace {

// Work counters of the persistent grid, one pair {next rank, CTAs done} per
// (device, stream).  Launches on one stream run in order and the last CTA of
// each launch zeroes its pair, so every launch finds it zero.  Made on a
// stream's first prefill outside stream capture (a cudaMalloc, then a
// cudaMemsetAsync on that stream); a stream first seen while it is being
// captured gets none, and its launches use one CTA per item.  Never freed
// (8 bytes per stream).
int* prefill_counters(int device, cudaStream_t stream) {
  static std::mutex mu;
  static std::map<std::pair<int, uintptr_t>, int*> counters;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(device, reinterpret_cast<uintptr_t>(stream));
  const auto it = counters.find(key);
  if (it != counters.end()) return it->second;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return nullptr;
  }
  int* c = nullptr;
  if (cudaMalloc(&c, 2 * sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (cudaMemsetAsync(c, 0, 2 * sizeof(int), stream) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(c);
    return nullptr;
  }
  counters[key] = c;
  return c;
}

// Grid of a prefill launch.  Persistent (the default for rounded P): one CTA
// per SM, each claiming items from the stream's counters until none is left,
// so an item's Q and first K/V copies and its first Q.K^T overlap the previous
// item's last softmax and output stores, tensor memory and barriers are set up
// once per SM, and SMs that finish early take more items.  Otherwise one CTA
// per (head, sequence, pair), heaviest pairs first.  Returns the kernel.
using PrefillKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                               const pre::Params);

// p_split 3 (fp16 P.V) reaches here only for bf16 inputs with packed K/V.
template <typename T, int D, bool kPaged>
PrefillKernel plan_prefill(const PrefillArgs& a, int p_split, pre::Params& p, dim3* grid) {
  using L = pre::Layout<D>;
  constexpr bool kCanHalf = std::is_same<T, __nv_bfloat16>::value && !kPaged;
  const int pairs = (a.max_seqlen_q + L::kRowsPerCta - 1) / L::kRowsPerCta;
  p.batch = a.batch;
  p.num_pairs = pairs;
  const int device = current_device();
  const int g = sm_count(device);
  const bool rounded = p_split == 0 || p_split == 3;
  p.sched = (rounded && prefill_schedule() == 0 && g > 0) ? prefill_counters(device, a.stream) : nullptr;
  if (p.sched != nullptr) {
    *grid = dim3(unsigned(g));
    if constexpr (kCanHalf) {
      if (p_split == 3) return pre::prefill_kernel<T, D, kPaged, false, true, true>;
    }
    return pre::prefill_kernel<T, D, kPaged, false, true, false>;
  }
  *grid = dim3(unsigned(a.num_heads * a.batch), unsigned(pairs));
  if constexpr (kCanHalf) {
    if (p_split == 3) return pre::prefill_kernel<T, D, kPaged, false, false, true>;
  }
  return rounded ? pre::prefill_kernel<T, D, kPaged, false, false, false>
                 : pre::prefill_kernel<T, D, kPaged, true, false, false>;
}

// fp16 P.V scratch per (device, stream): the fp16 copy of V and the largest
// |v| per (sequence, KV head).  Grown on demand (after the stream's earlier
// work finished) and never freed; not grown while the stream is captured
// (false: the caller feeds P as head + remainder instead).
bool pv_scratch(int device, cudaStream_t stream, size_t v16_bytes, size_t emax_count, void** v16,
                unsigned** emax) {
  struct Buffers {
    void* v16 = nullptr;
    size_t v16_cap = 0;
    unsigned* emax = nullptr;
    size_t emax_cap = 0;
  };
  static std::mutex mu;
  static std::map<std::pair<int, uintptr_t>, Buffers> scratch;
  std::lock_guard<std::mutex> lock(mu);
  Buffers& s = scratch[std::make_pair(device, reinterpret_cast<uintptr_t>(stream))];
  if (s.v16_cap < v16_bytes || s.emax_cap < emax_count) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone ||
        cudaStreamSynchronize(stream) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    if (s.v16_cap < v16_bytes) {
      cudaFree(s.v16);
      s.v16 = nullptr;
      s.v16_cap = 0;
      const size_t cap = v16_bytes + v16_bytes / 4;
      if (cudaMalloc(&s.v16, cap) != cudaSuccess) {
        cudaGetLastError();
        return false;
      }
      s.v16_cap = cap;
    }
    if (s.emax_cap < emax_count) {
      cudaFree(s.emax);
      s.emax = nullptr;
      s.emax_cap = 0;
      const size_t cap = emax_count + emax_count / 4 + 64;
      if (cudaMalloc(&s.emax, cap * sizeof(unsigned)) != cudaSuccess) {
        cudaGetLastError();
        return false;
      }
      s.emax_cap = cap;
    }
  }
  *v16 = s.v16;
  *emax = s.emax;
  return true;
}

// Map of the 16-bit output {head_dim, head, token} in 64-column, 32-row boxes
// (the epilogue's TMA stores).  fp32 output, or a layout the map cannot
// describe, keeps the direct stores (the map is then a placeholder).
template <int D>
int encode_out_map(const PrefillArgs& a, const CUtensorMap& placeholder, CUtensorMap* to) {
  *to = placeholder;
  if (a.out_dtype == FAT_DTYPE_F32) return 0;
  std::string why;
  const uint32_t box[3] = {64u, 1u, 32u};
  const uint64_t dims[3] = {uint64_t(D), uint64_t(a.num_heads), uint64_t(a.total_q)};
  const uint64_t strides[2] = {uint64_t(a.o_sh) * 2, uint64_t(a.o_st) * 2};
  if (!encode_tiled(to, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, a.out, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                    &why)) {
    *to = placeholder;
    return 0;
  }
  return 1;
}

template <typename T, int D>
int launch_t(const PrefillArgs& a) {
  using L = pre::Layout<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  int p_split = prefill_p_split(kBf16);
  // fp16 P.V: V is read from an fp16 copy the pre-pass writes ([tokens, kv heads,
  // dim], contiguous) into this stream's scratch.
  PrefillArgs av = a;
  unsigned* emax = nullptr;
  if (p_split == 3) {
    void* v16 = nullptr;
    const size_t n_e = size_t(a.batch) * size_t(a.num_kv_heads);
    const size_t bytes = size_t(a.total_k) * size_t(a.num_kv_heads) * size_t(D) * 2;
    if (!kBf16) {
      p_split = 0;  // fp16 inputs: P.V already runs in fp16
    } else if (a.total_k > 0 && pv_scratch(current_device(), a.stream, bytes, n_e, &v16, &emax)) {
      av.v = v16;
      av.v_st = int64_t(a.num_kv_heads) * D;
      av.v_sh = D;
    } else {
      p_split = 1;  // no scratch (stream being captured, or out of memory): head + remainder
    }
  }
  pre::Params p{};
  dim3 grid;
  const PrefillKernel kern = plan_prefill<T, D, false>(a, p_split, p, &grid);
  static_assert(L::kSmem <= 227 * 1024, "prefill tiles exceed shared memory");
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), int(L::kSmem), current_device());
  if (e != cudaSuccess) return cuda_failure("cudaFuncSetAttribute(prefill)", e);
  std::string why;
  CUtensorMap tq, tk, tv;
  const uint32_t box[3] = {64u, 1u, uint32_t(pre::BM)};
  {
    const uint64_t dims[3] = {uint64_t(D), uint64_t(a.num_heads), uint64_t(a.total_q)};
    const uint64_t strides[2] = {uint64_t(a.q_sh) * 2, uint64_t(a.q_st) * 2};
    if (!encode_tiled(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, a.q, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B, &why))
      return invalid("prefill q: " + why);
  }
  {
    const uint64_t dims[3] = {uint64_t(D), uint64_t(a.num_kv_heads), uint64_t(a.total_k)};
    const uint64_t sk[2] = {uint64_t(a.k_sh) * 2, uint64_t(a.k_st) * 2};
    const uint64_t sv[2] = {uint64_t(av.v_sh) * 2, uint64_t(av.v_st) * 2};
    if (!encode_tiled(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, a.k, dims, sk, box, CU_TENSOR_MAP_SWIZZLE_128B,
                      &why))
      return invalid("prefill k: " + why);
    if (!encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, av.v, dims, sv, box, CU_TENSOR_MAP_SWIZZLE_128B,
                      &why))
      return invalid("prefill v: " + why);
  }
  CUtensorMap to;
  p.o_tma = encode_out_map<D>(a, tq, &to);
  p.cu_q = a.cu_q;
  p.cu_k = a.cu_k;
  p.out = a.out;
  p.o_st = a.o_st;
  p.o_sh = a.o_sh;
  p.num_heads = a.num_heads;
  p.group = a.num_heads / a.num_kv_heads;
  p.scale_log2 = float(double(a.softmax_scale) * 1.4426950408889634);
  p.causal = a.causal ? 1 : 0;
  p.out_f32 = a.out_dtype == FAT_DTYPE_F32;
  p.err = a.error_word;
  p.wait_ns = wait_limit_ns();
  p.expire = take_expire_request() ? 1 : 0;
  p.p_split = p_split;
  p.num_kv_heads = a.num_kv_heads;
  if (p_split == 3) {
    // Pre-pass: largest finite |v| per (sequence, KV head), then the scaled fp16 copy.
    p.pv_emax = emax;
    e = cudaMemsetAsync(emax, 0, size_t(a.batch) * size_t(a.num_kv_heads) * sizeof(unsigned), a.stream);
    if (e != cudaSuccess) return cuda_failure("prefill v pre-pass memset", e);
    const dim3 vgrid(unsigned((a.total_k + pre::kVRows - 1) / pre::kVRows), unsigned(a.num_kv_heads));
    const uint16_t* vsrc = static_cast<const uint16_t*>(a.v);
    pre::v_absmax_kernel<D><<<vgrid, pre::kVThreads, 0, a.stream>>>(vsrc, a.v_st, a.v_sh, a.cu_k, a.batch,
                                                                   a.num_kv_heads, a.total_k, emax);
    pre::v_to_half_kernel<D><<<vgrid, pre::kVThreads, 0, a.stream>>>(
        vsrc, a.v_st, a.v_sh, a.cu_k, a.batch, a.num_kv_heads, a.total_k, emax,
        static_cast<uint16_t*>(const_cast<void*>(av.v)));
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_failure("prefill v pre-pass launch", e);
  }
  kern<<<grid, L::kThreads, L::kSmem, a.stream>>>(tq, tk, tv, to, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_failure("prefill launch", e);
  return FAT_OK;
}

template <typename T, int D>
int launch_paged_t(const PrefillArgs& a) {
  using L = pre::Layout<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  int p_split = prefill_p_split(kBf16);
  // fp16 P.V needs a copy of V, which a paged cache does not get: bf16 feeds P
  // as head + remainder instead (fp16 inputs: P.V already runs in fp16).
  if (p_split == 3) p_split = kBf16 ? 1 : 0;
  pre::Params p{};
  dim3 grid;
  const PrefillKernel kern = plan_prefill<T, D, true>(a, p_split, p, &grid);
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), int(L::kSmem), current_device());
  if (e != cudaSuccess) return cuda_failure("cudaFuncSetAttribute(prefill paged)", e);
  std::string why;
  CUtensorMap tq, tk, tv;
  {
    const uint32_t box[3] = {64u, 1u, uint32_t(pre::BM)};
    const uint64_t dims[3] = {uint64_t(D), uint64_t(a.num_heads), uint64_t(a.total_q)};
    const uint64_t strides[2] = {uint64_t(a.q_sh) * 2, uint64_t(a.q_st) * 2};
    if (!encode_tiled(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, a.q, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B, &why))
      return invalid("prefill q: " + why);
  }
  const int rpb = a.page_size < pre::BN ? a.page_size : pre::BN;
  {
    // {head_dim, kv head, slot, page}: one box = rpb slots of one head of one page.
    const uint64_t dims[4] = {uint64_t(D), uint64_t(a.num_kv_heads), uint64_t(a.page_size), uint64_t(a.num_pages)};
    const uint64_t strides[3] = {uint64_t(a.kv_sh) * 2, uint64_t(a.kv_ss) * 2, uint64_t(a.kv_sp) * 2};
    const uint32_t box[4] = {64u, 1u, uint32_t(rpb), 1u};
    if (!encode_tiled(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, a.k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                      &why))
      return invalid("prefill k_cache: " + why);
    if (!encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, a.v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                      &why))
      return invalid("prefill v_cache: " + why);
  }
  CUtensorMap to;
  p.o_tma = encode_out_map<D>(a, tq, &to);
  p.cu_q = a.cu_q;
  p.out = a.out;
  p.o_st = a.o_st;
  p.o_sh = a.o_sh;
  p.num_heads = a.num_heads;
  p.group = a.num_heads / a.num_kv_heads;
  p.scale_log2 = float(double(a.softmax_scale) * 1.4426950408889634);
  p.causal = a.causal ? 1 : 0;
  p.out_f32 = a.out_dtype == FAT_DTYPE_F32;
  p.err = a.error_word;
  p.page_table = a.page_table;
  p.pt_sb = a.pt_sb;
  p.max_pages = int(a.max_pages);
  p.num_pages = int(a.num_pages);
  p.page_size = a.page_size;
  p.rows_per_box = rpb;
  p.cap_tokens = int(std::min<long long>((long long)a.max_pages * a.page_size, 1ll << 30));
  p.seq_lens_k = a.seq_lens_k;
  p.wait_ns = wait_limit_ns();
  p.expire = take_expire_request() ? 1 : 0;
  p.p_split = p_split;
  kern<<<grid, L::kThreads, L::kSmem, a.stream>>>(tq, tk, tv, to, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_failure("prefill paged launch", e);
  return FAT_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int launch_prefill_paged(const PrefillArgs& a) {
  if (a.batch < 0 || a.total_q < 0) return invalid("prefill_paged: sizes must be non-negative");
  if (a.num_heads <= 0 || a.num_kv_heads <= 0 || a.num_heads % a.num_kv_heads != 0)
    return invalid("prefill_paged: num_heads must be a positive multiple of num_kv_heads");
  if (a.dtype != FAT_DTYPE_F16 && a.dtype != FAT_DTYPE_BF16)
    return unsupported("prefill_paged: q and the cache must be fp16 or bf16");
  if (a.out_dtype != a.dtype && a.out_dtype != FAT_DTYPE_F32)
    return invalid("prefill_paged: out dtype must be the input dtype or fp32");
  if (a.batch == 0 || a.total_q == 0 || a.max_seqlen_q <= 0) return FAT_OK;
  if (a.q == nullptr || a.k == nullptr || a.v == nullptr || a.out == nullptr || a.cu_q == nullptr ||
      a.page_table == nullptr || a.seq_lens_k == nullptr)
    return invalid("prefill_paged: null pointer argument");
  if (a.num_pages <= 0 || a.max_pages <= 0) return invalid("prefill_paged: empty cache or page table");
  // One TMA box per (page, 128-byte column block): a page holds a power of two
  // of at least 8 token rows below 128, or whole 128-row tiles.
  const int ps = a.page_size;
  const bool pow2 = ps > 0 && (ps & (ps - 1)) == 0;
  if (!((pow2 && ps >= 8 && ps <= pre::BN) || (ps > pre::BN && ps % pre::BN == 0)))
    return unsupported("prefill_paged: page_size must be a power of two in [8, 128] or a multiple of 128, got " +
                       std::to_string(ps));
  if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || (a.q_st * 2) % 16 || (a.q_sh * 2) % 16 ||
      (a.kv_sp * 2) % 16 || (a.kv_ss * 2) % 16 || (a.kv_sh * 2) % 16)
    return unsupported("prefill_paged: q and the cache must be 16-byte aligned with 16-byte-multiple strides");
  if (!aligned16(a.out) || (a.o_st * (a.out_dtype == FAT_DTYPE_F32 ? 4 : 2)) % 16 ||
      (a.o_sh * (a.out_dtype == FAT_DTYPE_F32 ? 4 : 2)) % 16)
    return unsupported("prefill_paged: out must be 16-byte aligned with 16-byte-multiple strides");
  if (a.max_seqlen_q > 65535 * pre::BM) return unsupported("prefill_paged: max_seqlen_q too large");
  // One producer lane per (page, 128-byte column block) of a 128-row tile.
  if ((pre::BN / std::min(ps, pre::BN)) * (a.head_dim / 64) > 32)
    return unsupported("prefill_paged: head_dim " + std::to_string(a.head_dim) + " needs page_size >= " +
                       std::to_string(pre::BN * (a.head_dim / 64) / 32) + ", got " + std::to_string(ps));
  const bool bf = a.dtype == FAT_DTYPE_BF16;
  switch (a.head_dim) {
    case 64:
      return bf ? launch_paged_t<__nv_bfloat16, 64>(a) : launch_paged_t<__half, 64>(a);
    case 128:
      return bf ? launch_paged_t<__nv_bfloat16, 128>(a) : launch_paged_t<__half, 128>(a);
    case 256:
      return bf ? launch_paged_t<__nv_bfloat16, 256>(a) : launch_paged_t<__half, 256>(a);
    default:
      return unsupported("prefill_paged: head_dim must be 64, 128 or 256, got " + std::to_string(a.head_dim));
  }
}

int launch_prefill_varlen(const PrefillArgs& a) {
  if (a.batch < 0 || a.total_q < 0 || a.total_k < 0) return invalid("prefill_varlen: sizes must be non-negative");
  if (a.num_heads <= 0 || a.num_kv_heads <= 0 || a.num_heads % a.num_kv_heads != 0)
    return invalid("prefill_varlen: num_heads must be a positive multiple of num_kv_heads");
  if (a.dtype != FAT_DTYPE_F16 && a.dtype != FAT_DTYPE_BF16)
    return unsupported("prefill_varlen: q/k/v must be fp16 or bf16");
  if (a.out_dtype != a.dtype && a.out_dtype != FAT_DTYPE_F32)
    return invalid("prefill_varlen: out dtype must be the input dtype or fp32");
  if (a.batch == 0 || a.total_q == 0 || a.max_seqlen_q <= 0) return FAT_OK;
  if (a.q == nullptr || a.k == nullptr || a.v == nullptr || a.out == nullptr || a.cu_q == nullptr ||
      a.cu_k == nullptr)
    return invalid("prefill_varlen: null pointer argument");
  if (a.total_k == 0) return invalid("prefill_varlen: no keys");
  if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || (a.q_st * 2) % 16 || (a.q_sh * 2) % 16 ||
      (a.k_st * 2) % 16 || (a.k_sh * 2) % 16 || (a.v_st * 2) % 16 || (a.v_sh * 2) % 16)
    return unsupported("prefill_varlen: q/k/v must be 16-byte aligned with 16-byte-multiple strides");
  if (!aligned16(a.out) || (a.o_st * (a.out_dtype == FAT_DTYPE_F32 ? 4 : 2)) % 16 ||
      (a.o_sh * (a.out_dtype == FAT_DTYPE_F32 ? 4 : 2)) % 16)
    return unsupported("prefill_varlen: out must be 16-byte aligned with 16-byte-multiple strides");
  if (a.max_seqlen_q > 65535 * pre::BM) return unsupported("prefill_varlen: max_seqlen_q too large");
  const bool bf = a.dtype == FAT_DTYPE_BF16;
  switch (a.head_dim) {
    case 64:
      return bf ? launch_t<__nv_bfloat16, 64>(a) : launch_t<__half, 64>(a);
    case 128:
      return bf ? launch_t<__nv_bfloat16, 128>(a) : launch_t<__half, 128>(a);
    case 256:
      return bf ? launch_t<__nv_bfloat16, 256>(a) : launch_t<__half, 256>(a);
    default:
      return unsupported("prefill_varlen: head_dim must be 64, 128 or 256, got " + std::to_string(a.head_dim));
  }
}

}  // namespace fat
