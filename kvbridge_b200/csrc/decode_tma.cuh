#pragma once
// Split-K partial kernel for paged INT8 KV on sm_100a.
//
// Computes, for every piece of the split-K schedule (kvb_schedule.h), the
// partial (m, l, n[dim]) of reference src/attention_shared.cu:42-209 /
// include/kvbridge/partial_attention_mma.cuh:153-477: scores
// s = scale * kscale * q.k over the visible tokens of the piece, m = max s,
// l = sum exp(s - m), n = sum exp(s - m) * vscale * v.
//
// Structure (one CTA = 4 consumer warps + 1 producer warp):
//  * Data movement: the producer warp walks the CTA's pieces, looks the pages
//    of each 64-token stage up in the page table (a 64-entry register window
//    prefetched ahead), and issues one bulk asynchronous copy per (page, K|V|
//    kscale|vscale) into a STAGES-deep shared-memory ring guarded by
//    mbarriers. K and V are consumed exactly as stored (int8); nothing is
//    converted before it reaches shared memory.
//  * Math: each consumer warp owns whole stages (stage g goes to warp g % 4)
//    and keeps its own online-softmax state. QK and PV run on the int8
//    warp-level MMA (m16n8k32, exact s32 accumulation) with the query side
//    as the A operand, whose 16 rows are (query column, int8 limb) pairs, and
//    K / V as the B operand, used exactly as stored:
//        S[(col, limb)][token] = Q_limb[col][d] . K^T[d][token]
//        O[(col, limb)][d]     = P_limb[col][token] . V^T[token][d]
//    A thread's B fragment is then 8 contiguous bytes of one K row (dims) or
//    one V row (tokens), so every 16-byte shared load lands as two aligned B
//    register pairs, and both limbs of a column come back in the same
//    thread's C fragment. QK: each query row is a 22-bit fixed-point value
//    split into three signed int8 limbs (q = L0 + 2^8 L1 + 2^16 L2, scaled by
//    a power of two per row). PV: P = w * vscale is a 15-bit signed
//    fixed-point value per (stage, column) split into two signed int8 limbs;
//    the exact sums are folded into fp32 accumulators with the power-of-two
//    scale. Per-token kscale multiplies the fp32 scores and per-token vscale
//    rides on P, as in the reference MMA kernel. The QK n-tiles take their
//    tokens in the order that leaves each thread the scores of 16 contiguous
//    tokens of its column, which are exactly the tokens of its PV A operand,
//    so P never leaves the thread's registers.
//  * Precision: QK is exact up to the 2^-22 (relative to the row's largest
//    |q|) rounding of Q; P is exact up to 2^-15 of the stage's largest |P|
//    of the column (its power-of-two scale adapts per stage and column, so
//    any finite vscale works).
//  * Pieces end with an in-CTA log-sum-exp combine of the four warps'
//    states and one (m, l, n) write per query row.
#include <cuda.h>

#include <type_traits>

#include "kvb_device.cuh"
#include "kvb_schedule.h"

namespace kvb {

struct DecodeParams {
  const float* q;
  const int64_t* q_positions;  // single sequence: [rows]; batched: unused
  const int64_t* k_positions;  // single sequence: [tokens]; batched: unused
  const uint32_t* table;       // page table (single) or block table (batched)
  const int8_t* k;
  const int8_t* v;
  const float* k_scales;
  const float* v_scales;
  const uint32_t* seq_lens;  // batched: [batch]; nullptr for a single sequence
  float* part;               // partial output
  uint32_t batch, rows, q_heads, kv_heads, group, qr;
  uint32_t page_tokens, log2_page, pages, table_stride;
  uint32_t begin, end;    // single sequence token interval
  uint32_t seg_stages;    // single sequence: stages per segment
  uint32_t split_stride;  // single sequence: scratch splits per row-head
  uint32_t max_tokens;    // batched: clamp for seq_lens
  uint32_t ctas;
  uint64_t total_stages;  // single sequence only (batched computes it)
  float score_scale;
  // L2 prefetch of the CTA's first `prefetch_stages` stages before the
  // dependency wait on the preceding grid (0 = none).
  uint32_t prefetch_stages;
  // Single sequence: the query columns (rows * group per KV head) are cut
  // into col_groups groups of group_cols (= 8 * NT) columns; CTA c works on
  // group c % col_groups, so the CTAs of one KV range and different groups
  // run side by side and share its pages in L2. Batched: 1 and 8 * NT.
  uint32_t col_groups, group_cols;
  // Upper bound of every pipeline wait of the launch (kDefaultWaitLimitNs
  // unless the host set another).
  unsigned long long wait_limit_ns;
  // Test hook for the bounded waits: the producer of CTA 0 neither arms nor
  // loads its stage number `fault_stage` (0xffffffff = off), so the consumer
  // of that stage waits until wait_limit_ns, records the failure and the CTA
  // returns. No memory access depends on it.
  uint32_t fault_stage;
};

// Parameters of the small-page kernels. 16-token pages at dim <= 128
// (gather_kv = 1): the K and V pools as 2-D tensor maps of one row of
// page_tokens * dim bytes per (page, KV head), so that one gather load
// brings a stage's four pages. Only these kernels carry the maps (256
// bytes of parameters a launch otherwise).
struct DecodeParamsGather : DecodeParams {
  CUtensorMap tm_k, tm_v;
  uint32_t gather_kv;
};

template <bool SMALL_PAGES>
using KernelParams = typename std::conditional<SMALL_PAGES, DecodeParamsGather, DecodeParams>::type;

// Per-CTA timeline of these kernels (trace builds only, -DKVB_TC_TRACE): for
// the first kCtaTraceCtas CTAs of the latest launch, g_cta_trace[cta][event]
// with the events below. Entry and exit also carry the global timer (ns), so
// that CTAs on different SMs share one time axis; the other events are SM
// clock stamps (clock64), exact within a CTA.
constexpr int kCtaTraceCtas = 1024;
constexpr int kCtaTraceEvents = 20;
enum CtaTraceEvent : int {
  kCtaEntryNs = 0,      // thread 0 entered (global timer)
  kCtaEntryClk = 1,     // thread 0 entered (clock64)
  kCtaSm = 2,           // SM id
  kCtaDepWaitDone = 3,  // consumer warp 0 passed the dependency wait on the preceding grid
  kCtaFirstCopy = 4,    // producer armed its first stage (copies issued right after)
  kCtaLastCopy = 5,     // producer armed its last stage
  kCtaFirstStage = 6,   // the CTA's first stage had landed (its consumer's wait returned)
  kCtaWarpDone = 7,     // + w: consumer warp w finished its last stage (w < 4)
  kCtaPartialDone = 11, // partials written, the consumers' exit (clock64)
  kCtaExitNs = 12,      // the same moment on the global timer
  kCtaStages = 13,      // stages the producer issued
  kCtaLastStage = 14,   // the CTA's last stage had landed (its consumer's wait returned)
  // Kept from the first launch after the trace was cleared (later launches
  // leave them alone), so that two traced calls show call 1's exit beside
  // call 2's events:
  kCtaFirstEntryNs = 16,  // entry (global timer)
  kCtaFirstExitNs = 17,   // consumers' exit (global timer)
  kCtaProducerWait = 18,  // SM cycles the producer spent waiting for free ring slots
  kCtaConsumerWait = 19,  // SM cycles consumer warp 0 spent waiting for its stages to land
};
#ifdef KVB_TC_TRACE
#define KVB_WAIT_CLOCK_BEGIN() const long long kvb_wait_t0 = clock64()
#define KVB_WAIT_CLOCK_END(acc) (acc) += static_cast<unsigned long long>(clock64() - kvb_wait_t0)
#else
#define KVB_WAIT_CLOCK_BEGIN() \
  do {                         \
  } while (0)
#define KVB_WAIT_CLOCK_END(acc) \
  do {                          \
  } while (0)
#endif
#ifdef KVB_TC_TRACE
__device__ unsigned long long g_cta_trace[kCtaTraceCtas][kCtaTraceEvents];
#define KVB_CTA_MARK(event, value)                                          \
  do {                                                                      \
    if (blockIdx.x < kCtaTraceCtas) g_cta_trace[blockIdx.x][(event)] = (value); \
  } while (0)
#define KVB_CTA_MARK_FIRST(event, value)                                                     \
  do {                                                                                       \
    if (blockIdx.x < kCtaTraceCtas && g_cta_trace[blockIdx.x][(event)] == 0ull)                \
      g_cta_trace[blockIdx.x][(event)] = (value);                                            \
  } while (0)
#else
#define KVB_CTA_MARK(event, value) \
  do {                             \
  } while (0)
#define KVB_CTA_MARK_FIRST(event, value) \
  do {                                   \
  } while (0)
#endif

__device__ __forceinline__ unsigned long long sm_id() {
  uint32_t id;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(id));
  return id;
}

constexpr int kConsumerWarps = 4;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kDecodeThreads = 32 * (kConsumerWarps + 1);
constexpr int kStatusBadPage = 4;
constexpr int kStatusSeqLenClamped = 5;

template <int D>
struct StageLayout {
  static constexpr uint32_t kK = 0;
  static constexpr uint32_t kV = 64u * D;
  static constexpr uint32_t kKs = 128u * D + 128u;
  static constexpr uint32_t kVs = kKs + 256u;
  static constexpr uint32_t kBytes = kVs + 256u;
};

// V page pitch inside a stage. Small-page kernels: the pages of a stage sit
// back to back (as a gather load writes them); a warp's 16-byte V reads (row
// 8 dn + grp, tokens 16 tig..) take the minimum four wavefronts either way.
// The 64-token-page kernels (one page a stage) keep the expression they were
// tuned with: its register allocation measured ~0.1 us a call better at cfg2.
template <bool SMALL_PAGES>
__device__ __forceinline__ uint32_t v_page_pitch(uint32_t dim, uint32_t page_tokens) {
  if (SMALL_PAGES) return dim * page_tokens;
  return dim * page_tokens + (page_tokens < 64 ? 2u * page_tokens : 0u);
}

// RING_COMBINE: the warps' combine buffer reuses the start of the ring. A
// single-sequence CTA has one piece, so when it combines, every copy has
// landed and every stage has been read (the consumers meet at a barrier
// first); the freed shared memory holds one more stage. A batched CTA may
// already be loading its next piece and keeps a buffer of its own.
// Query columns of a CTA. NT >= 1: 8 NT columns, column grp + 8 nt of a
// warp's MMA fragments in lane (grp, tig). NT = 0: the four-column layout of
// query groups of at most 4 columns (one query row of a 32/8- or 64/16-head
// model): column grp & 3 in lanes grp and grp + 4, which split the int8
// digits of its query and probability rows between them, so that QK needs
// one m-tile instead of two and P carries three digits instead of two.
template <int NT>
constexpr int cta_cols() { return NT == 0 ? 4 : 8 * NT; }
// Column slots of the per-thread state arrays (one in the four-column layout).
template <int NT>
constexpr int nt_slots() { return NT == 0 ? 1 : NT; }

template <int D, int NT, int STAGES, bool RING_COMBINE>
struct DecodeSmem {
  static constexpr uint32_t kRing = STAGES * StageLayout<D>::kBytes;
  static constexpr uint32_t kCols = 8 * nt_slots<NT>();  // four-column layout: 4 of 8 used
  static constexpr uint32_t kPitch = D + 4;  // floats; breaks bank aliasing of columns
  static constexpr uint32_t kCombine = kConsumerWarps * kCols * kPitch * 4;
  static_assert(!RING_COMBINE || kCombine <= kRing, "combine buffer larger than the ring");
  static constexpr uint32_t kStats = kConsumerWarps * kCols * 2 * 4;
  static constexpr uint32_t kBarriers = 2 * STAGES * 8;
  static constexpr uint32_t kOffCombine = RING_COMBINE ? 0 : kRing;
  static constexpr uint32_t kOffStats = RING_COMBINE ? kRing : kOffCombine + kCombine;
  static constexpr uint32_t kOffBar = kOffStats + kStats;
  static constexpr uint32_t kOffAbort = kOffBar + kBarriers;
  // Stage tags: the CTA stage sequence number each ring slot is armed for.
  static constexpr uint32_t kOffTags = kOffAbort + 16;
  static constexpr uint32_t kBytes = kOffTags + 4 * STAGES;
};

// ---------------------------------------------------------------------------
// Piece walking (identical in producer and consumers).

struct Piece {
  uint32_t b, h;       // sequence and KV head
  uint32_t j0, j1;     // stage range within the segment
  uint32_t lo, hi;     // attended token interval of the sequence
  uint32_t slot;       // partial slot (see write_partial)
  uint32_t col0;       // first query column of the CTA's column group
};

// HINT: a read before the dependency wait on the preceding grid, through L2
// only (ld.global.cg), so that no possibly stale copy stays in L1 for the
// reads after the wait; such values only steer prefetches.
template <bool HINT = false>
__device__ __forceinline__ uint32_t clamped_len(const DecodeParams& p, uint32_t b) {
  const uint32_t len = HINT ? __ldcg(p.seq_lens + b) : p.seq_lens[b];
  return len > p.max_tokens ? p.max_tokens : len;
}

// Warp-cooperative: total stages of a batched call.
template <bool HINT = false>
__device__ __forceinline__ uint64_t batched_total(const DecodeParams& p) {
  const uint32_t lane = threadIdx.x & 31;
  uint64_t total = 0;
  for (uint32_t base = 0; base < p.batch; base += 32) {
    const uint32_t b = base + lane;
    const uint32_t t = b < p.batch ? stages_of_range(0, clamped_len<HINT>(p, b)) : 0;
    uint64_t s = t;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    total += s;
  }
  return total * p.kv_heads;
}

// Warp-cooperative: sequence b whose segments hold global stage x, and the
// number of stages of all earlier sequences (per KV head).
template <bool HINT = false>
__device__ __forceinline__ void batched_locate(const DecodeParams& p, uint64_t x, uint32_t& b_out,
                                               uint64_t& pref_out) {
  const uint32_t lane = threadIdx.x & 31;
  uint64_t pref = 0;
  for (uint32_t base = 0; base < p.batch; base += 32) {
    const uint32_t b = base + lane;
    const uint64_t t = b < p.batch ? stages_of_range(0, clamped_len<HINT>(p, b)) : 0;
    uint64_t incl = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= uint32_t(o)) incl += y;
    }
    const uint32_t hit = __ballot_sync(0xffffffffu, b < p.batch && (pref + incl) * p.kv_heads > x);
    if (hit) {
      const uint32_t l = __ffs(hit) - 1;
      b_out = base + l;
      const uint64_t incl_l = __shfl_sync(0xffffffffu, incl, l);
      const uint64_t t_l = __shfl_sync(0xffffffffu, t, l);
      pref_out = pref + incl_l - t_l;
      return;
    }
    pref += __shfl_sync(0xffffffffu, incl, 31);
  }
  b_out = p.batch;  // unreachable for x < total
  pref_out = pref;
}

// Single sequence (ctas = parts * kv_heads * col_groups): CTA c = (j *
// kv_heads + h) * col_groups + col_group owns piece j of head h, stages
// [floor(j*T/parts), floor((j+1)*T/parts)), T = seg_stages -- the global
// schedule of kvb_schedule.h restricted to a segment, in 32-bit arithmetic:
// floor(j*T/parts) = j*(T/parts) + floor(j*(T%parts)/parts). Heads are
// interleaved over the CTA index, so that every head has pieces among the
// first CTAs an SM takes and among the second ones, which run a little
// slower beside them (measured ~0.15 us a call at 64K tokens).
__device__ __forceinline__ Piece single_piece(const DecodeParams& p, uint32_t c) {
  const uint32_t groups = p.col_groups;
  const uint32_t parts = p.ctas / (p.kv_heads * groups);
  const uint32_t col_group = c % groups;
  c /= groups;
  const uint32_t h = c % p.kv_heads, j = c / p.kv_heads;
  const uint32_t T = p.seg_stages, q = T / parts, r = T - q * parts;
  Piece pc;
  pc.b = 0;
  pc.col0 = col_group * p.group_cols;
  pc.h = h;
  pc.j0 = j * q + (j * r) / parts;
  pc.j1 = (j + 1) * q + ((j + 1) * r) / parts;
  pc.lo = p.begin;
  pc.hi = p.end;
  pc.slot = j;
  return pc;
}

// The piece starting at global stage x of CTA c whose range ends at x_end.
template <bool BATCHED>
__device__ __forceinline__ Piece locate_piece(const DecodeParams& p, const Piece& only, uint64_t x,
                                              uint64_t x_end, uint64_t total, uint32_t c) {
  if (!BATCHED) return only;
  Piece pc;
  pc.col0 = 0;
  uint64_t seg_base;
  uint32_t seg_len;
  if (!BATCHED) {
    pc.b = 0;
    pc.lo = p.begin;
    pc.hi = p.end;
    seg_base = 0;
    seg_len = p.seg_stages;
  } else {
    uint64_t pref;
    batched_locate(p, x, pc.b, pref);
    pc.lo = 0;
    pc.hi = clamped_len(p, pc.b);
    seg_base = pref * p.kv_heads;
    seg_len = stages_of_range(0, pc.hi);
  }
  pc.h = static_cast<uint32_t>((x - seg_base) / seg_len);
  const uint64_t seg_off = seg_base + uint64_t(pc.h) * seg_len;
  pc.j0 = static_cast<uint32_t>(x - seg_off);
  const uint64_t rem = x_end - seg_off;
  pc.j1 = rem < seg_len ? static_cast<uint32_t>(rem) : seg_len;
  if (!BATCHED)
    pc.slot = c - cta_of_stage(seg_off, total, p.ctas);
  else
    pc.slot = c + pc.b * p.kv_heads + pc.h;
  return pc;
}

__device__ __forceinline__ uint64_t piece_end_stage(const DecodeParams& p, const Piece& pc,
                                                    uint64_t x) {
  return x + (pc.j1 - pc.j0);
}

// The CTA's global stage range [x0, x1) and the call's stage count. A batched
// call reads the sequence lengths, so this runs after the dependency wait.
template <bool BATCHED>
__device__ __forceinline__ void cta_stage_range(const DecodeParams& p, const Piece& only,
                                                uint64_t& total, uint64_t& x0, uint64_t& x1) {
  if (!BATCHED) {
    total = p.total_stages;
    x0 = uint64_t(only.h) * p.seg_stages + only.j0;
    x1 = x0 + (only.j1 - only.j0);
  } else {
    total = batched_total(p);
    x0 = cta_stage_begin(blockIdx.x, total, p.ctas);
    x1 = cta_stage_begin(blockIdx.x + 1, total, p.ctas);
  }
}

// ---------------------------------------------------------------------------
// Producer: one warp, bulk copies of whole pages.

// Single sequence, before the dependency wait on the preceding grid: L2
// prefetch of the K/V pages and scales of the CTA's first `count` stages.
// The preceding grid may still be writing the page table or the pages, so
// nothing read here is used as data: table entries only steer prefetches
// (read through L2, so that no stale copy stays in L1), out-of-range entries
// are skipped, and the copies proper re-read everything after the wait.
template <int D>
__device__ void prefetch_first_stages(const DecodeParams& p, const Piece& pc, uint32_t count) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t first_stage = pc.lo / kStageTokens;
  const uint32_t j_end = min(pc.j1, pc.j0 + count);
  const uint32_t tok_lo = max(pc.lo, (first_stage + pc.j0) * kStageTokens);
  const uint32_t tok_hi = min(pc.hi, (first_stage + j_end) * kStageTokens);
  if (tok_hi <= tok_lo) return;
  // The table entries of the producer's first two batches of 8 pages.
  const uint32_t piece_hi =
      (min(pc.hi, (first_stage + pc.j1) * kStageTokens) - 1) >> p.log2_page;
  const uint32_t batch_pg = (first_stage + pc.j0) * (kStageTokens >> p.log2_page) + lane;
  if (lane < 16 && batch_pg >= (tok_lo >> p.log2_page) && batch_pg <= piece_hi)
    prefetch_line_l2(p.table + batch_pg);
  const uint32_t P = p.page_tokens;
  const uint32_t pg1 = (tok_hi - 1) >> p.log2_page;
  for (uint32_t pg = (tok_lo >> p.log2_page) + lane; pg <= pg1; pg += 32) {
    const uint32_t phys = __ldcg(p.table + pg);
    if (phys >= p.pages) continue;
    const size_t unit = size_t(phys) * p.kv_heads + pc.h;
    prefetch_l2(p.k + unit * P * D, P * D);
    prefetch_l2(p.v + unit * D * P, D * P);
    prefetch_l2(p.k_scales + unit * P, 4 * P);
    prefetch_l2(p.v_scales + unit * P, 4 * P);
  }
}

// Batched, before the dependency wait on the preceding grid: L2 prefetch of
// the K/V pages and scales of the CTA's first `count` stages (within its
// first piece). The preceding grid may still be writing seq_lens, the block
// table or the pages, so everything here is read through L2 only and steers
// prefetches alone (entries that point outside the pool are skipped); the
// producer locates its pieces and reads the table again after the wait.
template <int D>
__device__ void prefetch_first_stages_batched(const DecodeParams& p, uint32_t count) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t total = batched_total<true>(p);
  const uint64_t x0 = cta_stage_begin(blockIdx.x, total, p.ctas);
  const uint64_t x1 = cta_stage_begin(blockIdx.x + 1, total, p.ctas);
  if (x0 >= x1) return;
  uint32_t b;
  uint64_t pref;
  batched_locate<true>(p, x0, b, pref);
  if (b >= p.batch) return;
  const uint32_t len = clamped_len<true>(p, b);
  const uint32_t t = stages_of_range(0, len);
  if (t == 0) return;
  const uint64_t seg_base = pref * p.kv_heads;
  const uint32_t h = static_cast<uint32_t>((x0 - seg_base) / t);
  if (h >= p.kv_heads) return;
  const uint32_t j0 = static_cast<uint32_t>(x0 - seg_base - uint64_t(h) * t);
  const uint32_t j1 = static_cast<uint32_t>(min(uint64_t(t), uint64_t(j0) + min(uint64_t(count), x1 - x0)));
  const uint32_t tok_lo = j0 * kStageTokens, tok_hi = min(len, j1 * kStageTokens);
  if (tok_hi <= tok_lo) return;
  const uint32_t* trow = p.table + size_t(b) * p.table_stride;
  const uint32_t P = p.page_tokens;
  const uint32_t pg1 = (tok_hi - 1) >> p.log2_page;
  for (uint32_t pg = (tok_lo >> p.log2_page) + lane; pg <= pg1; pg += 32) {
    const uint32_t phys = __ldcg(trow + pg);
    if (phys >= p.pages) continue;
    const size_t unit = size_t(phys) * p.kv_heads + h;
    prefetch_l2(p.k + unit * P * D, P * D);
    prefetch_l2(p.v + unit * D * P, D * P);
    prefetch_l2(p.k_scales + unit * P, 4 * P);
    prefetch_l2(p.v_scales + unit * P, 4 * P);
  }
}

// Single sequence, before the dependency wait: L2 prefetch of the query rows
// of the CTA's columns and of the two position words the piece setup reads.
// A hint only: the setup loads them again after the wait. (Under a streaming
// call those lines are often no longer in L2, and a miss behind the first
// copies of every CTA took ~1.5 us.)
template <int D, int NT>
__device__ void prefetch_query_lines(const DecodeParams& p, const Piece& pc) {
  const uint32_t lane = threadIdx.x & 31;
  if (pc.j1 <= pc.j0) return;
  constexpr uint32_t kLines = D * 4 / 128;  // 128-byte lines of one fp32 query row
  for (uint32_t i = lane; i < uint32_t(cta_cols<NT>()) * kLines; i += 32) {
    const uint32_t col = pc.col0 + i / kLines;
    if (col >= p.qr) break;
    const uint32_t r = col / p.group, g = col % p.group;
    prefetch_line_l2(p.q + (size_t(r) * p.q_heads + size_t(pc.h) * p.group + g) * D + (i % kLines) * 32);
  }
  if (lane == 0) {
    const uint32_t first_stage = pc.lo / kStageTokens;
    prefetch_line_l2(p.k_positions + (min(pc.hi, (first_stage + pc.j1) * kStageTokens) - 1));
    prefetch_line_l2(p.q_positions + pc.col0 / p.group);
  }
}

// Drain: every copy the producer issued (stages 0..g-1) must land before the
// CTA can exit; only the last STAGES of them can still be in flight.
template <int STAGES>
__device__ __forceinline__ void drain_copies(uint64_t* full, uint32_t g,
                                             unsigned long long limit_ns) {
  const uint32_t first = g > STAGES ? g - STAGES : 0u;
  for (uint32_t s = first; s < g; ++s) {
    // Copies land whatever the consumers do, so this wait ignores an abort.
    volatile int no_abort = 0;
    if (mbar_wait_bounded(&full[s % STAGES], (s / STAGES) & 1u, &no_abort, kStatusDrainTimeout,
                          int(s), limit_ns) != kWaitOk)
      break;
  }
}

// Single sequence: splits [parts, split_stride) of the CTA's row-heads are
// written as empty partials (m = -inf, l = 0; n is left as it is), so that
// the scratch holds a complete reference layout for a merge over all splits.
// They are spread over the CTAs by slot (split parts + slot + k * parts) and
// written by the producer warp once its copies are issued, off the path of
// the call's last stage and of the merge that follows.
template <int D>
__device__ void mark_empty_splits(const DecodeParams& p, const Piece& pc) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t parts = p.ctas / (p.kv_heads * p.col_groups);
  if (p.split_stride <= parts + pc.slot) return;
  const uint32_t count = (p.split_stride - parts - pc.slot - 1) / parts + 1;
  const uint32_t cols = min(p.group_cols, p.qr - pc.col0);
  for (uint32_t w = lane; w < cols * count; w += 32) {
    const uint32_t col = pc.col0 + w % cols;
    const uint32_t split = parts + pc.slot + (w / cols) * parts;
    const uint32_t r = col / p.group, gq = col % p.group;
    const size_t rh = size_t(r) * p.q_heads + size_t(pc.h) * p.group + gq;
    float* e = p.part + (rh * p.split_stride + split) * (D + 2);
    e[0] = -INFINITY;
    e[1] = 0.f;
  }
}

// Producer for pages shorter than a stage (16 or 32 tokens). Each bulk copy
// costs the SM's copy engine about as much time as a small one, and with
// 16-token pages the four copies per page (K, V and two 64-byte scale runs)
// made that the streaming limit. Here only K and V are bulk-copied; per
// stage, lane l loads the 16 bytes of scales of tokens 4*(l%16) .. +3 (K
// scales for l < 16, V scales above) with a plain load and stores them to the
// stage before the barrier is armed, and the lane holding a page's first
// four tokens starts the bulk copy of that page's K (l < 16) or V (l >= 16).
// A lane's table entries and scales are fetched 8 and 5 stages ahead in
// registers that take turns (no register copies, which would wait for the
// loads). With 64-token pages the extra per-stage work costs more than the
// two copies it saves, so produce() keeps those.
template <int D, int STAGES, bool BATCHED>
__device__ void produce_small_pages(const DecodeParamsGather& p, const Piece& only, uint8_t* ring,
                                    uint64_t* full, uint64_t* empty, volatile uint32_t* tags,
                                    volatile int* abort_flag) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t policy = l2_evict_first_policy();
  const uint32_t P = p.page_tokens;
  const uint32_t kv_bytes = 2u * P * D;  // bulk-copied bytes per page
  const uint32_t vpitch = v_page_pitch<true>(D, P);
  const uint32_t pps = kStageTokens >> p.log2_page;  // pages per stage: 2 or 4
  const uint32_t tok4 = 4u * (lane & 15u);
  const uint32_t q = tok4 >> p.log2_page;  // the lane's page within a stage
  const bool is_v = lane >= 16;
  const bool copier = (tok4 & (P - 1u)) == 0u;
  const float* scale_base = is_v ? p.v_scales : p.k_scales;
  const uint32_t scale_off = is_v ? StageLayout<D>::kVs : StageLayout<D>::kKs;
  grid_dependency_wait();
  uint64_t total, x0, x1;
  cta_stage_range<BATCHED>(p, only, total, x0, x1);
  uint32_t g = 0;  // stages issued so far (CTA stage sequence number)
  bool failed = false;
  unsigned long long empty_wait = 0;  // trace builds only
  (void)empty_wait;
  for (uint64_t x = x0; x < x1 && !failed;) {
    const Piece pc = locate_piece<BATCHED>(p, only, x, x1, total, blockIdx.x);
    const uint32_t first_stage = pc.lo / kStageTokens;
    const uint32_t page_lo = max(pc.lo, (first_stage + pc.j0) * kStageTokens) >> p.log2_page;
    const uint32_t page_hi = (min(pc.hi, (first_stage + pc.j1) * kStageTokens) - 1) >> p.log2_page;
    const uint32_t* trow =
        !BATCHED ? p.table : p.table + size_t(pc.b) * p.table_stride;
    // Table entry of this lane's page of stage j (in flight after return).
    auto table_load = [&](uint32_t j, uint32_t& t, bool& mine) {
      const uint32_t pg = (first_stage + j) * pps + q;
      mine = j < pc.j1 && pg >= page_lo && pg <= page_hi;
      t = mine ? __ldg(trow + pg) : 0u;
    };
    // This lane's 16 bytes of scales of the stage whose table entry is t.
    auto scale_load = [&](uint32_t t, bool mine, float4& sc) {
      const bool ok = mine && t < p.pages;
      const size_t unit = size_t(ok ? t : 0u) * p.kv_heads + pc.h;  // (page, kv head)
      sc = ok ? __ldcs(reinterpret_cast<const float4*>(scale_base + unit * P + (tok4 & (P - 1u))))
              : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    // One stage: wait for its slot, store the scales, arm the barrier,
    // start the bulk copies. False if the slot wait gave up.
    auto issue_stage = [&](uint32_t t, bool mine, const float4& sc) -> bool {
      const bool ok = mine && t < p.pages;
      if (__ballot_sync(0xffffffffu, mine && !ok) && lane == 0)
        atomicMax(&g_kvb_status, kStatusBadPage);
      const uint32_t okpages = __popc(__ballot_sync(0xffffffffu, ok && copier && !is_v));
      // Lanes 0..15 and 16..31 each cover the stage's pages (four lanes a page).
      const bool gather = pps == 4 && p.gather_kv != 0 && __all_sync(0xffffffffu, ok);
      const int32_t unit32 = int32_t(uint32_t(ok ? t : 0u) * p.kv_heads + pc.h);
      const uint32_t slot = g % STAGES;
      KVB_WAIT_CLOCK_BEGIN();
      if (mbar_wait_bounded(&empty[slot], ((g / STAGES) & 1u) ^ 1u, abort_flag,
                            kStatusEmptyWaitTimeout, int(g), p.wait_limit_ns) != kWaitOk)
        return false;
      KVB_WAIT_CLOCK_END(empty_wait);
      if (g == p.fault_stage && blockIdx.x == 0) {
        // Test hook: the stage is never published (no tag) and loads nothing;
        // its barrier phase completes with zero bytes so that the ring, and
        // the drain at exit, stay in step.
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], 0u);
        ++g;
        return true;
      }
      uint8_t* st = ring + size_t(slot) * StageLayout<D>::kBytes;
      *reinterpret_cast<float4*>(st + scale_off + tok4 * 4u) = sc;
      // The warp's scale stores come before lane 0's arrive (release).
      __syncwarp();
      if (lane == 0) {
        // Tag protocol as in produce().
        tags[slot] = g;
        mbar_arrive_expect_tx(&full[slot], okpages * kv_bytes);
        if (g == 0) KVB_CTA_MARK(kCtaFirstCopy, clock64());
        KVB_CTA_MARK(kCtaLastCopy, clock64());
      }
      __syncwarp();
      if (gather) {
        // All four pages of the stage are valid: two four-row gathers (K, V)
        // instead of eight page copies (the bulk-copy request rate, not HBM,
        // bounds 16-token pages).
        const int32_t u0 = __shfl_sync(0xffffffffu, unit32, 0), u1 = __shfl_sync(0xffffffffu, unit32, 4);
        const int32_t u2 = __shfl_sync(0xffffffffu, unit32, 8), u3 = __shfl_sync(0xffffffffu, unit32, 12);
        if (lane == 0) {
          tma_gather4(st + StageLayout<D>::kK, &p.tm_k, u0, u1, u2, u3, &full[slot], policy);
          tma_gather4(st + StageLayout<D>::kV, &p.tm_v, u0, u1, u2, u3, &full[slot], policy);
        }
      } else if (ok && copier) {
        const size_t unit = size_t(t) * p.kv_heads + pc.h;
        if (is_v)
          bulk_copy_g2s(st + StageLayout<D>::kV + q * vpitch, p.v + unit * D * P, D * P,
                        &full[slot], policy);
        else
          bulk_copy_g2s(st + StageLayout<D>::kK + q * P * D, p.k + unit * P * D, P * D,
                        &full[slot], policy);
      }
      ++g;
      return true;
    };
    // Table entries 8 stages ahead, scales 5 (their loads go to DRAM under a
    // streaming HBM; at cfg4 a lead of 3 was 1.5 % slower, and 7 leaves the
    // table entry too little time before its scale load needs it).
    uint32_t t[8];
    bool mine[8];
    float4 sc[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) table_load(pc.j0 + u, t[u], mine[u]);
#pragma unroll
    for (int u = 0; u < 5; ++u) scale_load(t[u], mine[u], sc[u]);
    for (uint32_t jb = pc.j0; jb < pc.j1 && !failed; jb += 8) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (jb + u >= pc.j1) break;
        scale_load(t[(u + 5) & 7], mine[(u + 5) & 7], sc[(u + 5) & 7]);
        if (!issue_stage(t[u], mine[u], sc[u & 7])) {
          failed = true;
          break;
        }
        table_load(jb + u + 8, t[u], mine[u]);
      }
    }
    x = piece_end_stage(p, pc, x);
  }
  if (!BATCHED && !failed) mark_empty_splits<D>(p, only);
  if (lane == 0) {
    KVB_CTA_MARK(kCtaStages, g);
    KVB_CTA_MARK(kCtaProducerWait, empty_wait);
  }
  drain_copies<STAGES>(full, g, p.wait_limit_ns);
}

template <int D, int STAGES, bool BATCHED>
__device__ void produce(const DecodeParams& p, const Piece& only, uint8_t* ring, uint64_t* full,
                        uint64_t* empty, volatile uint32_t* tags, volatile int* abort_flag) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t policy = l2_evict_first_policy();
  const uint32_t P = p.page_tokens;
  const uint32_t page_bytes = 2u * P * D + 8u * P;
  const uint32_t vpitch = v_page_pitch<false>(D, P);
  // Work is handed out 8 pages at a time, four lanes per page: lane l
  // copies part l % 4 (K, V, K scales, V scales) of page l / 4 of the batch.
  // A batch covers spb stages of pps pages each. Table entries, page checks
  // and copy addresses are worked out for the whole batch at once, so that
  // issuing a stage is only: wait for its slot, arm its barrier, and one
  // warp instruction that starts all of the stage's copies.
  const uint32_t pps = kStageTokens >> p.log2_page;  // 1, 2 or 4
  const uint32_t spb = 8u / pps;
  const uint32_t lane_page = lane >> 2, part = lane & 3;
  const uint32_t lane_stage = lane_page / pps;
  const uint32_t page_in_stage = lane_page - lane_stage * pps;
  uint32_t part_bytes, dst_off;
  if (part == 0) {
    part_bytes = P * D;
    dst_off = StageLayout<D>::kK + page_in_stage * P * D;
  } else if (part == 1) {
    part_bytes = D * P;
    dst_off = StageLayout<D>::kV + page_in_stage * vpitch;
  } else {
    part_bytes = 4 * P;
    dst_off = (part == 2 ? StageLayout<D>::kKs : StageLayout<D>::kVs) + page_in_stage * P * 4;
  }
  grid_dependency_wait();
  uint64_t total, x0, x1;
  cta_stage_range<BATCHED>(p, only, total, x0, x1);
  uint32_t g = 0;  // stages issued so far (CTA stage sequence number)
  bool failed = false;
  unsigned long long empty_wait = 0;  // trace builds only
  (void)empty_wait;
  for (uint64_t x = x0; x < x1 && !failed;) {
    const Piece pc = locate_piece<BATCHED>(p, only, x, x1, total, blockIdx.x);
    const uint32_t first_stage = pc.lo / kStageTokens;
    const uint32_t page_lo = max(pc.lo, (first_stage + pc.j0) * kStageTokens) >> p.log2_page;
    const uint32_t page_hi = (min(pc.hi, (first_stage + pc.j1) * kStageTokens) - 1) >> p.log2_page;
    const uint32_t* trow =
        !BATCHED ? p.table : p.table + size_t(pc.b) * p.table_stride;
    // This lane's page of the batch starting at stage j, if the piece reads it.
    auto batch_page = [&](uint32_t j, uint32_t& pg) {
      pg = (first_stage + j) * pps + lane_page;
      return j < pc.j1 && pg >= page_lo && pg <= page_hi;
    };
    uint32_t pg;
    bool mine = batch_page(pc.j0, pg);
    uint32_t cur = mine ? __ldg(trow + pg) : 0u;
    bool in_nxt = batch_page(pc.j0 + spb, pg);
    uint32_t nxt = in_nxt ? __ldg(trow + pg) : 0u;
    for (uint32_t jb = pc.j0; jb < pc.j1 && !failed; jb += spb) {
      const uint32_t phys = cur;
      const bool ok = mine && phys < p.pages;
      if (__ballot_sync(0xffffffffu, mine && !ok) && lane == 0)
        atomicMax(&g_kvb_status, kStatusBadPage);
      const uint32_t okmask = __ballot_sync(0xffffffffu, ok && part == 0);
      // Table entries two batches ahead, so that they are in registers in time.
      cur = nxt;
      mine = in_nxt;
      in_nxt = batch_page(jb + 2 * spb, pg);
      nxt = in_nxt ? __ldg(trow + pg) : 0u;
      const size_t unit = size_t(ok ? phys : 0u) * p.kv_heads + pc.h;  // (page, kv head)
      const uint8_t* src;
      if (part == 0)
        src = reinterpret_cast<const uint8_t*>(p.k + unit * P * D);
      else if (part == 1)
        src = reinterpret_cast<const uint8_t*>(p.v + unit * D * P);
      else
        src = reinterpret_cast<const uint8_t*>((part == 2 ? p.k_scales : p.v_scales) + unit * P);
      const uint32_t nstages = min(spb, pc.j1 - jb);
      for (uint32_t sb = 0; sb < nstages; ++sb) {
        const uint32_t slot = g % STAGES;
        const uint32_t use = g / STAGES;
        KVB_WAIT_CLOCK_BEGIN();
        if (mbar_wait_bounded(&empty[slot], (use & 1u) ^ 1u, abort_flag, kStatusEmptyWaitTimeout,
                              int(g), p.wait_limit_ns) != kWaitOk) {
          failed = true;
          break;
        }
        KVB_WAIT_CLOCK_END(empty_wait);
        if (g == p.fault_stage && blockIdx.x == 0) {
          // Test hook: the stage is never published (no tag) and loads
          // nothing; its barrier phase completes with zero bytes so that the
          // ring, and the drain at exit, stay in step.
          if (lane == 0) mbar_arrive_expect_tx(&full[slot], 0u);
          ++g;
          continue;
        }
        if (lane == 0) {
          // The slot is free, so its full barrier has completed the phase of
          // stage g - STAGES; publishing g tells the consumer of stage g that
          // the barrier's parity now refers to stage g (see the consumer loop).
          tags[slot] = g;
          const uint32_t stage_lanes = (pps == 4 ? 0xffffu : (1u << (4 * pps)) - 1u) << (4 * pps * sb);
          mbar_arrive_expect_tx(&full[slot], __popc(okmask & stage_lanes) * page_bytes);
          if (g == 0) KVB_CTA_MARK(kCtaFirstCopy, clock64());
          KVB_CTA_MARK(kCtaLastCopy, clock64());
        }
        __syncwarp();
        if (ok && lane_stage == sb)
          bulk_copy_g2s(ring + size_t(slot) * StageLayout<D>::kBytes + dst_off, src, part_bytes,
                        &full[slot], policy);
        ++g;
      }
    }
    x = piece_end_stage(p, pc, x);
  }
  if (!BATCHED && !failed) mark_empty_splits<D>(p, only);
  if (lane == 0) {
    KVB_CTA_MARK(kCtaStages, g);
    KVB_CTA_MARK(kCtaProducerWait, empty_wait);
  }
  drain_copies<STAGES>(full, g, p.wait_limit_ns);
}

// ---------------------------------------------------------------------------
// Consumers.

template <int D, int NT>
struct WarpState {
  // O fragments: column grp + 8 nt, dims 8 dn + 2 tig + e. Four-column
  // layout: lanes grp and grp + 4 each hold a part of column grp & 3 (their
  // digit rows' sums), added together when the warp flushes.
  float acc[D / 8][nt_slots<NT>()][2];
  float m[nt_slots<NT>()];  // running max (log2 units) of the column
  float l[nt_slots<NT>()];  // thread-partial denominator of that column
};

// QK m-tiles: rows (column c, limb k) are numbered 3 c + k (c < 8 NT taken
// as 8 nt + row-in-group), eight to a half-tile: m-tile mt holds row sets
// 2 mt (rows 0-7) and 2 mt + 1 (rows 8-15). With NT = 1 the last half-tile
// is zero. Four-column layout: one m-tile, rows grp < 4 limb 0 of column
// grp, rows 8 + grp limb 1, rows 4 + c limb 2 of column c, rows 12-15 zero.
template <int NT>
constexpr int qk_tiles() { return NT == 0 ? 1 : (3 * NT + 1) / 2; }

// Per-piece query operands of one warp: the A fragments of the QK MMA for
// every k-step (k-step j covers dims 64*(j/2) + 16*tig + 8*(j%2) + [0,8) for
// lane tig; a thread holds the limbs of its own column grp + 8 nt), and the
// fp32 factor turning combined limb dots into log2-unit scores.
template <int D, int NT>
struct QueryFrags {
  uint32_t a[qk_tiles<NT>()][D / 32][4];
  float cf[nt_slots<NT>()];      // score factor of the thread's column (log2 units)
  int64_t qpos[nt_slots<NT>()];  // query position of that column
};

// Loads the piece's query operands and, for a single sequence, returns
// whether every token of the piece is visible to every query row of the
// CTA's columns (k_positions is nondecreasing, so it is enough that the
// piece's last token `last_token` is). Every global load of this setup (Q
// rows, their positions, the last key position) is issued before any is
// used, so the setup costs one memory round trip.
template <int D, int NT, bool BATCHED>
__device__ __forceinline__ bool load_query(const DecodeParams& p, const Piece& pc,
                                           uint32_t last_token, QueryFrags<D, NT>& qf) {
  constexpr int kNt = nt_slots<NT>();
  const uint32_t lane = threadIdx.x & 31, grp = lane >> 2, tig = lane & 3;
  // Visibility: lane j < cta_cols checks the row of column col0 + j.
  int64_t kp_last = 0, qp_own = INT64_MAX;
  if (!BATCHED) {
    kp_last = __ldg(p.k_positions + last_token);
    const uint32_t ocol = pc.col0 + lane;
    if (lane < uint32_t(cta_cols<NT>()) && ocol < p.qr) qp_own = __ldg(p.q_positions + ocol / p.group);
  }
  float vals[kNt][D / 64][16];
  int64_t qp[kNt];
#pragma unroll
  for (int nt = 0; nt < kNt; ++nt) {
    const uint32_t col = pc.col0 + (NT == 0 ? (grp & 3u) : 8 * nt + grp);
    const bool valid = col < p.qr;
    const uint32_t r = valid ? col / p.group : 0, g = valid ? col % p.group : 0;
    const uint32_t row = !BATCHED ? r : pc.b;
    const float* qrow = p.q + (size_t(row) * p.q_heads + size_t(pc.h) * p.group + g) * D;
#pragma unroll
    for (int c = 0; c < D / 64; ++c) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 f = valid ? __ldg(reinterpret_cast<const float4*>(qrow + 64 * c + 16 * tig) + i)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        vals[nt][c][4 * i + 0] = f.x;
        vals[nt][c][4 * i + 1] = f.y;
        vals[nt][c][4 * i + 2] = f.z;
        vals[nt][c][4 * i + 3] = f.w;
      }
    }
    qp[nt] = (!BATCHED && valid) ? __ldg(p.q_positions + r) : INT64_MAX;
  }
#pragma unroll
  for (int nt = 0; nt < kNt; ++nt) {
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < D / 64; ++c)
#pragma unroll
      for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(vals[nt][c][i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    // 2^e > max|q|; q * 2^(22-e) rounds to an integer of magnitude <= 2^22.
    int e = 0;
    if (amax > 0.f) e = int((__float_as_uint(amax) >> 23) & 0xffu) - 126;
    e = max(-100, min(100, e));
    const float up = __uint_as_float(uint32_t(127 + 22 - e) << 23);
    // q = rint(v * up), |q| <= 2^22, is split into signed base-256 digits
    // q = l0 + 256 l1 + 65536 l2 with l0, l1 in [-128, 127] (unique, so the
    // same limbs as a sequential split). v * up is exact (a power-of-two
    // scale), so fma(v, up, 1.5 * 2^23) rounds it to the nearest integer
    // (ties to even) in the low mantissa bits; subtracting the sum's bias and
    // adding 0x808080 leaves q + 0x808080, whose bytes 0..2 are l0..l2 + 128.
    // Byte permutes gather digit k of four values and xor 0x80 removes the 128.
    constexpr float kRoundInt = 12582912.0f;  // 1.5 * 2^23
    constexpr uint32_t kBias = 0x808080u - 0x4B400000u;
#pragma unroll
    for (int c = 0; c < D / 64; ++c) {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            w[i] = __float_as_uint(fmaf(vals[nt][c][8 * jj + 4 * half + i], up, kRoundInt)) + kBias;
          const uint32_t a = __byte_perm(w[0], w[1], 0x5140), b = __byte_perm(w[2], w[3], 0x5140);
          const uint32_t c2 = __byte_perm(w[0], w[1], 0x0062), d2 = __byte_perm(w[2], w[3], 0x0062);
          const uint32_t limb[3] = {__byte_perm(a, b, 0x5410) ^ 0x80808080u,
                                    __byte_perm(a, b, 0x7632) ^ 0x80808080u,
                                    __byte_perm(c2, d2, 0x5410) ^ 0x80808080u};
          if constexpr (NT == 0) {
            // a0/a2 (row grp): limb 0, or limb 2 in lanes grp >= 4; a1/a3
            // (row grp + 8): limb 1, or zero.
            const bool upper = grp >= 4;
            qf.a[0][2 * c + jj][2 * half] = upper ? limb[2] : limb[0];
            qf.a[0][2 * c + jj][1 + 2 * half] = upper ? 0u : limb[1];
          } else {
            // Row set 3 nt + k of the A fragment: a0/a2 (rows 0-7, k-lo/hi),
            // a1/a3 (rows 8-15).
#pragma unroll
            for (int k = 0; k < 3; ++k) {
              const int rs = 3 * nt + k;
              qf.a[rs / 2][2 * c + jj][(rs % 2) + 2 * half] = limb[k];
            }
          }
        }
      }
    }
    qf.cf[nt] = p.score_scale * kLog2e * __uint_as_float(uint32_t(127 + e - 22) << 23);
    qf.qpos[nt] = qp[nt];
  }
  if constexpr (NT != 0 && 3 * NT % 2 == 1) {
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      qf.a[qk_tiles<NT>() - 1][j][1] = 0u;
      qf.a[qk_tiles<NT>() - 1][j][3] = 0u;
    }
  }
  if (BATCHED) return true;
  return __all_sync(0xffffffffu, kp_last <= qp_own);
}

// One 64-token stage for one warp. The thread (grp, tig) works on columns
// grp + 8 nt and on the stage's tokens 16 tig + [0, 16) (local index t).
template <int D, int NT, bool SMALL_PAGES>
__device__ __forceinline__ void consume_stage(const DecodeParams& p, const uint8_t* st,
                                              uint32_t tb, uint32_t lo, uint32_t hi,
                                              bool all_visible, const QueryFrags<D, NT>& qf,
                                              WarpState<D, NT>& ws) {
  constexpr int kQk = qk_tiles<NT>();
  constexpr int kNt = nt_slots<NT>();
  const uint32_t lane = threadIdx.x & 31, grp = lane >> 2, tig = lane & 3;
  const uint8_t* sk = st + StageLayout<D>::kK;
  const uint8_t* sv = st + StageLayout<D>::kV;
  const float* sks = reinterpret_cast<const float*>(st + StageLayout<D>::kKs);
  const float* svs = reinterpret_cast<const float*>(st + StageLayout<D>::kVs);

  // ---- S = Q K^T. N-tile j holds tokens 16*(n/2) + 2j + n%2 (n = 0..7): the
  //      thread supplies the K row of token n = grp and gets back columns
  //      n = 2 tig + e, i.e. tokens 16 tig + 2 j + e (t = 2 j + e).
  float sc[kNt][16];
  // K rows are read one n-tile ahead of the MMAs that use them; the compiler
  // fence after each read keeps it from hoisting further (register pressure).
  uint4 kw[2][D / 64];
#pragma unroll
  for (int c = 0; c < D / 64; ++c)
    kw[0][c] = *reinterpret_cast<const uint4*>(sk + (16 * (grp >> 1) + (grp & 1)) * D + 64 * c + 16 * tig);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j + 1 < 8) {
      const uint32_t tk = 16 * (grp >> 1) + 2 * (j + 1) + (grp & 1);
#pragma unroll
      for (int c = 0; c < D / 64; ++c)
        kw[(j + 1) & 1][c] = *reinterpret_cast<const uint4*>(sk + tk * D + 64 * c + 16 * tig);
    }
    asm volatile("" ::: "memory");
    int acc[kQk][4];
#pragma unroll
    for (int mt = 0; mt < kQk; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][i] = 0;
#pragma unroll
    for (int c = 0; c < D / 64; ++c) {
      const uint4 k4 = kw[j & 1][c];
#pragma unroll
      for (int mt = 0; mt < kQk; ++mt) {
        const uint32_t* a0 = qf.a[mt][2 * c];
        const uint32_t* a1 = qf.a[mt][2 * c + 1];
        imma_16832(acc[mt], a0[0], a0[1], a0[2], a0[3], k4.x, k4.y);
        imma_16832(acc[mt], a1[0], a1[1], a1[2], a1[3], k4.z, k4.w);
      }
    }
    if constexpr (NT == 0) {
      // Rows grp (c0, c1) and grp + 8 (c2, c3): limbs 0 and 1 of the column
      // in lanes grp < 4 (l0 + 256 l1, exact in s32: |dot| <= 2^22 at dim
      // 256), limb 2 in lanes grp >= 4 (its second row is zero). The lane
      // pair adds the two parts (the same sum in both lanes: fp32 addition
      // is commutative).
      const float wgt = grp >= 4 ? 65536.f : 1.f;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float part = float(acc[0][e] + 256 * acc[0][2 + e]) * wgt;
        sc[0][2 * j + e] = part + __shfl_xor_sync(0xffffffffu, part, 16);
      }
    } else {
      // Limb k of column grp + 8 nt is row set 3 nt + k: C rows 0-7 (c0, c1)
      // or 8-15 (c2, c3) of m-tile (3 nt + k) / 2. Limb dots are exact
      // integers (|dot| < 2^21); combine in fp32.
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int r0 = 3 * nt, r1 = 3 * nt + 1, r2 = 3 * nt + 2;
          const int d0 = acc[r0 / 2][2 * (r0 % 2) + e], d1 = acc[r1 / 2][2 * (r1 % 2) + e];
          const int d2 = acc[r2 / 2][2 * (r2 % 2) + e];
          sc[nt][2 * j + e] = fmaf(float(d2), 65536.f, fmaf(float(d1), 256.f, float(d0)));
        }
    }
  }

  // ---- scores in log2 units, masking.
  const bool full = all_visible && tb >= lo && tb + kStageTokens <= hi;
  const uint32_t t0 = tb + 16 * tig;  // sequence index of local token 0
  {
    float ks[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 f = reinterpret_cast<const float4*>(sks + 16 * tig)[i];
      ks[4 * i + 0] = f.x;
      ks[4 * i + 1] = f.y;
      ks[4 * i + 2] = f.z;
      ks[4 * i + 3] = f.w;
    }
#pragma unroll
    for (int nt = 0; nt < kNt; ++nt)
#pragma unroll
      for (int t = 0; t < 16; ++t) sc[nt][t] *= ks[t] * qf.cf[nt];
  }
  if (!full) {
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      const bool in = t0 + t >= lo && t0 + t < hi;
      const int64_t kp = (in && !all_visible) ? __ldg(p.k_positions + t0 + t) : 0;
#pragma unroll
      for (int nt = 0; nt < kNt; ++nt)
        if (!in || (!all_visible && kp > qf.qpos[nt])) sc[nt][t] = -INFINITY;
    }
  }

  // ---- online softmax update per column (its 64 tokens sit in the four
  //      lanes of the thread's quad).
  {
    bool rescale = false;
    float fac[kNt];
#pragma unroll
    for (int nt = 0; nt < kNt; ++nt) {
      float cm = sc[nt][0];
#pragma unroll
      for (int t = 1; t < 16; ++t) cm = fmaxf(cm, sc[nt][t]);
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 1));
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 2));
      const float mold = ws.m[nt];
      const float mnew = fmaxf(mold, cm);
      const float alpha = mnew == -INFINITY ? 1.f : fast_exp2(mold - mnew);
      ws.m[nt] = mnew;
      const float msub = mnew == -INFINITY ? 0.f : mnew;
      float lsum = 0.f;
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        sc[nt][t] = fast_exp2(sc[nt][t] - msub);
        lsum += sc[nt][t];
      }
      ws.l[nt] = ws.l[nt] * alpha + lsum;
      fac[nt] = alpha;
      rescale |= alpha != 1.f;
    }
    if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
      for (int dn = 0; dn < D / 8; ++dn)
#pragma unroll
        for (int nt = 0; nt < kNt; ++nt) {
          ws.acc[dn][nt][0] *= fac[nt];
          ws.acc[dn][nt][1] *= fac[nt];
        }
    }
  }

  // ---- P = w * vscale in fp32 (tokens outside [lo, hi) take vscale 0: their
  //      slots may hold anything), and per column the power of two that puts
  //      the stage's largest |P| in [2^13, 2^14) (four-column layout: in
  //      [2^21, 2^22), for three digits): pscale scales P into the fixed
  //      point below, inv_pscale scales the exact sums back.
  float pscale[kNt], inv_pscale[kNt];
  {
    float vs[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 f = reinterpret_cast<const float4*>(svs + 16 * tig)[i];
      vs[4 * i + 0] = f.x;
      vs[4 * i + 1] = f.y;
      vs[4 * i + 2] = f.z;
      vs[4 * i + 3] = f.w;
    }
    if (!full) {
#pragma unroll
      for (int t = 0; t < 16; ++t)
        if (!(t0 + t >= lo && t0 + t < hi)) vs[t] = 0.f;
    }
#pragma unroll
    for (int nt = 0; nt < kNt; ++nt) {
      float pm = 0.f;
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        sc[nt][t] *= vs[t];
        pm = fmaxf(pm, fabsf(sc[nt][t]));
      }
      pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 1));
      pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 2));
      // pm < 2^(x - 126) for biased exponent x; pscale = 2^(140 - x) (2^(148
      // - x) for three digits), kept a normal float (stages with |P| below
      // ~2^-113 lose precision).
      const int x = int((__float_as_uint(pm) >> 23) & 0xffu);
      const int sh = max(-126, min(126, (NT == 0 ? 148 : 140) - x));
      pscale[nt] = pm > 0.f ? __uint_as_float(uint32_t(127 + sh) << 23) : 1.f;
      inv_pscale[nt] = pm > 0.f ? __uint_as_float(uint32_t(127 - sh) << 23) : 1.f;
    }
  }

  // ---- P as signed fixed point per (stage, column): u = rint(P * pscale),
  //      |u| < 2^14, split into signed base-256 digits u = lo + 256 hi
  //      (lo in [-128, 127], |hi| <= 64) as for the query limbs: the fma
  //      with 1.5 * 2^23 rounds the exact product to an integer (ties to
  //      even), and after the bias u + 0x8080 holds lo + 128 and hi + 128
  //      in its two low bytes. The PV A fragment of k-step kb is rows
  //      (column, lo) and (column, hi) over tokens 8 kb + [0, 8) of the
  //      thread: a0 / a2 = lo of tokens +0..3 / +4..7, a1 / a3 = hi.
  //      Four-column layout: |u| <= 2^22 in three digits u = d0 + 256 d1 +
  //      65536 d2 (the query's split); lanes grp < 4 supply rows (column,
  //      d0) and (column, d1), lanes grp >= 4 rows (column, d2) and zero.
  constexpr float kRoundInt = 12582912.0f;  // 1.5 * 2^23
  constexpr uint32_t kBias = (NT == 0 ? 0x808080u : 0x8080u) - 0x4B400000u;
  const bool upper = NT == 0 && grp >= 4;
  uint32_t pa[kNt][2][4];
#pragma unroll
  for (int nt = 0; nt < kNt; ++nt)
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          w[i] = __float_as_uint(fmaf(sc[nt][8 * kb + 4 * half + i], pscale[nt], kRoundInt)) + kBias;
        const uint32_t t01 = __byte_perm(w[0], w[1], 0x5140), t23 = __byte_perm(w[2], w[3], 0x5140);
        const uint32_t d0 = __byte_perm(t01, t23, 0x5410) ^ 0x80808080u;
        const uint32_t d1 = __byte_perm(t01, t23, 0x7632) ^ 0x80808080u;
        if constexpr (NT == 0) {
          const uint32_t c2 = __byte_perm(w[0], w[1], 0x0062), e2 = __byte_perm(w[2], w[3], 0x0062);
          const uint32_t d2 = __byte_perm(c2, e2, 0x5410) ^ 0x80808080u;
          pa[nt][kb][2 * half + 0] = upper ? d2 : d0;
          pa[nt][kb][2 * half + 1] = upper ? 0u : d1;
        } else {
          pa[nt][kb][2 * half + 0] = d0;
          pa[nt][kb][2 * half + 1] = d1;
        }
      }

  // ---- O += P V on the int8 MMA (exact s32). k-step kb covers the thread's
  //      tokens 16 tig + 8 kb + [0, 8): k = 4 tig + i is token +i, k = 16 +
  //      4 tig + i is token +4+i, so the B fragment is bytes 8 kb .. 8 kb + 7
  //      of the thread's 16-byte slice of V row d = 8 dn + grp, used as stored.
  const uint32_t P = p.page_tokens;
  const uint32_t vpitch = v_page_pitch<SMALL_PAGES>(D, P);
  const uint8_t* vslice = sv + ((16 * tig) >> p.log2_page) * vpitch + ((16 * tig) & (P - 1));
  // V rows are read two n-tiles ahead of their MMAs, fenced like K.
  uint4 vw[2];
  vw[0] = *reinterpret_cast<const uint4*>(vslice + grp * P);
#pragma unroll
  for (int dn = 0; dn < D / 8; ++dn) {
    if (dn + 1 < D / 8) vw[(dn + 1) & 1] = *reinterpret_cast<const uint4*>(vslice + (8 * (dn + 1) + grp) * P);
    if (dn % 2 == 0) asm volatile("" ::: "memory");
    const uint4 v4 = vw[dn & 1];
#pragma unroll
    for (int nt = 0; nt < kNt; ++nt) {
      int c4[4] = {0, 0, 0, 0};
      imma_16832(c4, pa[nt][0][0], pa[nt][0][1], pa[nt][0][2], pa[nt][0][3], v4.x, v4.y);
      imma_16832(c4, pa[nt][1][0], pa[nt][1][1], pa[nt][1][2], pa[nt][1][3], v4.z, v4.w);
      // c0, c1: lo-digit sums of dims 8 dn + 2 tig + e; c2, c3: hi-digit
      // sums (four-column layout, lanes grp >= 4: d2 sums and zero, weight
      // 65536). |digit sums| <= 64 * 128 * 128, so hi * 256 + lo (< 2^29)
      // is exact in s32.
#pragma unroll
      for (int e = 0; e < 2; ++e)
        ws.acc[dn][nt][e] = fmaf(float(c4[2 + e] * 256 + c4[e]), upper ? inv_pscale[nt] * 65536.f : inv_pscale[nt],
                                 ws.acc[dn][nt][e]);
    }
  }
}

// SMALL_PAGES: pages shorter than a stage (produce_small_pages); a separate
// instantiation, so that the 64-token-page kernel does not carry that code
// (which cost it ~0.6 us a call at cfg2 when both producers were compiled in).
// Register cap per variant. Registers are split between an SM's four
// sub-partitions (16K each, allocated per warp in 256-register units), and a
// CTA's five warps are spread over them, so one sub-partition holds three
// warps of two resident CTAs: <= 168 registers (3 x 21 units) keeps two
// CTAs per SM at dims 64 and 128. The merge kernel that follows a call needs
// room for one of its warps (10 units) in every sub-partition: at 168 an SM
// still holding a merge CTA admitted one partial CTA instead of two, and at
// 64K tokens the call's last 32 CTAs started ~3 us late. The dim-128,
// 8-column kernels are therefore held to 144 (3 x 18 + 10 units; no
// spills). At dim 256 one CTA has the SM to itself: 216 (2 x 27 + 10).
template <int D, int NT, bool BATCHED>
constexpr int decode_max_regs() {
  return D == 256 ? 216 : (D == 128 && NT <= 1) ? 144 : 168;
}

template <int D, int NT, int STAGES, bool SMALL_PAGES, bool BATCHED>
__device__ __forceinline__ void decode_partial_body(const KernelParams<SMALL_PAGES>& p) {
  using L = DecodeSmem<D, NT, STAGES, !BATCHED>;
  constexpr int kNt = nt_slots<NT>();
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  float* combine = reinterpret_cast<float*>(smem + L::kOffCombine);
  float* stats = reinterpret_cast<float*>(smem + L::kOffStats);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* empty = full + STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);
  volatile uint32_t* tags = reinterpret_cast<volatile uint32_t*>(smem + L::kOffTags);

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    KVB_CTA_MARK_FIRST(kCtaFirstEntryNs, global_ns());
    KVB_CTA_MARK(kCtaEntryNs, global_ns());
    KVB_CTA_MARK(kCtaEntryClk, clock64());
    KVB_CTA_MARK(kCtaSm, sm_id());
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) tags[s] = 0xffffffffu;
    fence_barrier_init();
  }
  __syncthreads();
  // A single sequence's piece depends on the launch parameters only, so it
  // is worked out before the dependency wait on the preceding grid (which
  // may still be writing the inputs); each role waits just before its first
  // read of an input.
  const Piece only = !BATCHED ? single_piece(p, blockIdx.x) : Piece{};
  if (warp == kProducerWarp) {
    if (!BATCHED && p.prefetch_stages != 0) prefetch_first_stages<D>(p, only, p.prefetch_stages);
    if (BATCHED && p.prefetch_stages != 0) prefetch_first_stages_batched<D>(p, p.prefetch_stages);
    if constexpr (SMALL_PAGES)
      produce_small_pages<D, STAGES, BATCHED>(p, only, ring, full, empty, tags, abort_flag);
    else
      produce<D, STAGES, BATCHED>(p, only, ring, full, empty, tags, abort_flag);
    return;
  }
  if (warp == 0 && !BATCHED && p.prefetch_stages != 0) prefetch_query_lines<D, NT>(p, only);
  grid_dependency_wait();
  if (threadIdx.x == 0) KVB_CTA_MARK(kCtaDepWaitDone, clock64());
  uint64_t total, x0, x1;
  cta_stage_range<BATCHED>(p, only, total, x0, x1);

  const uint32_t grp = lane >> 2, tig = lane & 3;
  uint32_t g_base = 0;  // CTA stage sequence number of the piece's first stage
  unsigned long long full_wait = 0;  // trace builds only
  (void)full_wait;
  for (uint64_t x = x0; x < x1;) {
    const Piece pc = locate_piece<BATCHED>(p, only, x, x1, total, blockIdx.x);
    const uint32_t first_stage = pc.lo / kStageTokens;
    QueryFrags<D, NT> qf;
    const uint32_t last = min(pc.hi, (first_stage + pc.j1) * kStageTokens) - 1;
    const bool all_visible = load_query<D, NT, BATCHED>(p, pc, last, qf);
    WarpState<D, NT> ws;
#pragma unroll
    for (int dn = 0; dn < D / 8; ++dn)
#pragma unroll
      for (int nt = 0; nt < kNt; ++nt) ws.acc[dn][nt][0] = ws.acc[dn][nt][1] = 0.f;
#pragma unroll
    for (int nt = 0; nt < kNt; ++nt) {
      ws.m[nt] = -INFINITY;
      ws.l[nt] = 0.f;
    }

    const uint32_t n = pc.j1 - pc.j0;
    const uint32_t first = (warp + kConsumerWarps - g_base % kConsumerWarps) % kConsumerWarps;
    for (uint32_t i = first; i < n; i += kConsumerWarps) {
      const uint32_t g = g_base + i;
      const uint32_t slot = g % STAGES;
      // Consecutive uses of a slot go to different warps, so this warp may
      // arrive here while the slot still holds stage g - STAGES in flight:
      // the full barrier is then one phase behind, and a parity test alone
      // would mistake that phase for this one. Wait for the producer to tag
      // the slot with g first; from then on the barrier is in the phase of
      // stage g or past it, and the parity test is exact.
      KVB_WAIT_CLOCK_BEGIN();
      if (wait_tag_bounded(&tags[slot], g, abort_flag, kStatusFullWaitTimeout, int(g),
                           p.wait_limit_ns) == kWaitOk)
        mbar_wait_bounded(&full[slot], (g / STAGES) & 1u, abort_flag, kStatusFullWaitTimeout,
                          int(g), p.wait_limit_ns);
      KVB_WAIT_CLOCK_END(full_wait);
      if (g == 0 && lane == 0) KVB_CTA_MARK(kCtaFirstStage, clock64());
      if (i + 1 == n && x + n >= x1 && lane == 0) KVB_CTA_MARK(kCtaLastStage, clock64());
      const uint32_t tb = (first_stage + pc.j0 + i) * kStageTokens;
      consume_stage<D, NT, SMALL_PAGES>(p, ring + size_t(slot) * StageLayout<D>::kBytes, tb, pc.lo, pc.hi,
                           all_visible, qf, ws);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    g_base += n;
    if (lane == 0) KVB_CTA_MARK(kCtaWarpDone + int(warp), clock64());

    // ---- flush this warp's state.
    float* cw = combine + size_t(warp) * L::kCols * L::kPitch;
    if constexpr (NT == 0) {
      // Lanes grp and grp + 4 hold the two digit parts of one column.
#pragma unroll
      for (int dn = 0; dn < D / 8; ++dn)
#pragma unroll
        for (int e = 0; e < 2; ++e) ws.acc[dn][0][e] += __shfl_xor_sync(0xffffffffu, ws.acc[dn][0][e], 16);
    }
    float lsums[kNt];
#pragma unroll
    for (int nt = 0; nt < kNt; ++nt) {
      float lsum = ws.l[nt];
      lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
      lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
      lsums[nt] = lsum;
    }
    // The combine buffer overlays ring slots that other warps may still read.
    if (!BATCHED) named_barrier(1, 32 * kConsumerWarps);
    const bool writer = NT != 0 || grp < 4;
#pragma unroll
    for (int nt = 0; nt < kNt; ++nt) {
      const uint32_t col = 8 * nt + grp;
      if (tig == 0 && writer) {
        stats[(warp * L::kCols + col) * 2 + 0] = ws.m[nt];
        stats[(warp * L::kCols + col) * 2 + 1] = lsums[nt];
      }
      if (writer) {
#pragma unroll
        for (int dn = 0; dn < D / 8; ++dn)
          *reinterpret_cast<float2*>(cw + col * L::kPitch + 8 * dn + 2 * tig) =
              make_float2(ws.acc[dn][nt][0], ws.acc[dn][nt][1]);
      }
    }
    if (x + n >= x1) grid_launch_dependents();
    named_barrier(1, 32 * kConsumerWarps);

    // ---- combine the four warps and write one partial per query row.
    constexpr uint32_t kTpc = 32 * kConsumerWarps / L::kCols;  // threads per column
    constexpr uint32_t kDpt = D / kTpc;                          // dims per thread
    const uint32_t col = threadIdx.x / kTpc, part = threadIdx.x % kTpc;
    const uint32_t gcol = pc.col0 + col;  // the column among all p.qr
    if (gcol < p.qr) {
      float mw[kConsumerWarps], M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        mw[w] = stats[(w * L::kCols + col) * 2 + 0];
        M = fmaxf(M, mw[w]);
      }
      float ew[kConsumerWarps], Lsum = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        ew[w] = (M == -INFINITY || mw[w] == -INFINITY) ? 0.f : fast_exp2(mw[w] - M);
        Lsum += ew[w] * stats[(w * L::kCols + col) * 2 + 1];
      }
      size_t base;
      if (!BATCHED) {
        const uint32_t r = gcol / p.group, gq = gcol % p.group;
        const size_t rh = size_t(r) * p.q_heads + size_t(pc.h) * p.group + gq;
        base = (rh * p.split_stride + pc.slot) * (D + 2);
      } else {
        base = (size_t(pc.slot) * p.qr + gcol) * (D + 2);
      }
      float* out = p.part + base;
      if (part == 0) {
        out[0] = M == -INFINITY ? -INFINITY : M * kLn2;
        out[1] = Lsum;
      }
#pragma unroll
      for (uint32_t i = 0; i < kDpt; i += 2) {
        const uint32_t d = part * kDpt + i;
        float2 v = make_float2(0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float* src = combine + (size_t(w) * L::kCols + col) * L::kPitch + d;
          v.x += ew[w] * src[0];
          v.y += ew[w] * src[1];
        }
        *reinterpret_cast<float2*>(out + 2 + d) = v;
      }
    }
    named_barrier(1, 32 * kConsumerWarps);
    x += n;
  }
  if (threadIdx.x == 0) {
    KVB_CTA_MARK(kCtaConsumerWait, full_wait);
    KVB_CTA_MARK(kCtaPartialDone, clock64());
    KVB_CTA_MARK(kCtaExitNs, global_ns());
    KVB_CTA_MARK_FIRST(kCtaFirstExitNs, global_ns());
  }
}

// The kernels. 64-token pages take their parameters by value, as they always
// have; the small-page kernels take theirs as a __grid_constant__ parameter,
// whose tensor maps the gather loads read in place.
template <int D, int NT, int STAGES, bool SMALL_PAGES, bool BATCHED>
__global__ void __maxnreg__((decode_max_regs<D, NT, BATCHED>())) decode_partial_kernel(DecodeParams p) {
  static_assert(!SMALL_PAGES, "small pages use decode_partial_kernel_gather");
  decode_partial_body<D, NT, STAGES, false, BATCHED>(p);
}

template <int D, int NT, int STAGES, bool BATCHED>
__global__ void __maxnreg__((decode_max_regs<D, NT, BATCHED>()))
    decode_partial_kernel_gather(const __grid_constant__ DecodeParamsGather p) {
  decode_partial_body<D, NT, STAGES, true, BATCHED>(p);
}

}  // namespace kvb
