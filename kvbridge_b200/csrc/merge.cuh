#pragma once
// Log-sum-exp merge of split-K partials (reference src/attention_shared.cu:
// 295-335): for each (row, head)
//   M = max over partials with l_p > 0 of m_p
//   L = sum_p exp(m_p - M) * l_p,   N[d] = sum_p exp(m_p - M) * n_p[d]
// with m = -inf, l = 0, n = 0 when no partial has l_p > 0. The optional
// fp16 and bf16 epilogues write out = N / L (0 for empty rows), rounded to
// nearest even.
//
// The same kernel serves three partial layouts:
//   kScratch - the reference scratch layout [rh][split][dim+2]
//   kBatched - the batched workspace [piece][qrow][dim+2] (kvb_schedule.h)
//   kShards  - shard-major m/l/n triples from several GPUs
#include <cuda_bf16.h>

#include "kvb_device.cuh"
#include "kvb_schedule.h"

namespace kvb {

enum MergeMode : int { kMergeScratch = 0, kMergeBatched = 1, kMergeShards = 2 };

struct MergeParams {
  float* part;  // kScratch / kBatched (kScratch may write empty splits)
  const float* m_parts;  // kShards
  const float* l_parts;
  const float* n_parts;
  float* m;
  float* l;
  float* n;
  __half* out;
  __nv_bfloat16* out_bf16;
  uint32_t row_heads, dim;
  uint32_t np;            // kScratch: partials per row-head; kShards: shards
  uint32_t split_stride;  // kScratch: S of the layout
  uint32_t fill_empty;    // kScratch: write empty partials into splits [np, S)
  // kShards: floats from one shard's m (l, n) to the next shard's; 0 = the
  // separate arrays [shard][row_head] and [shard][row_head][dim]. A packed
  // exchange buffer [shard][m | l | n] uses row_heads * (dim + 2).
  uint64_t shard_stride;
  // kBatched
  const uint32_t* seq_lens;
  uint32_t batch, q_heads, kv_heads, group, max_tokens, ctas;
};

// Merge timeline (trace builds only, -DKVB_TC_TRACE): per CTA of the first
// merge launch after the trace was cleared, the global timer (ns) at entry
// (0), after the dependency wait on the partial kernel (1), at exit (2),
// after the first chunk's loads were used (3) and after the warps' fold (4).
constexpr int kMergeTraceCtas = 1024;
constexpr int kMergeTraceEvents = 5;
#ifdef KVB_TC_TRACE
__device__ unsigned long long g_merge_trace[kMergeTraceCtas][kMergeTraceEvents];
#define KVB_MERGE_MARK(event)                                                                 \
  do {                                                                                        \
    if (threadIdx.x == 0 && blockIdx.x < kMergeTraceCtas && g_merge_trace[blockIdx.x][(event)] == 0ull) \
      g_merge_trace[blockIdx.x][(event)] = global_ns();                                       \
  } while (0)
#else
#define KVB_MERGE_MARK(event) \
  do {                        \
  } while (0)
#endif

// Four warps per CTA with at most 80 registers a thread, so that a merge CTA
// fits on an SM beside two partial-kernel CTAs: with programmatic dependent
// launch it becomes resident early without holding back a partial CTA.
constexpr int kMergeWarps = 4;

// Warp-cooperative prefix of per-sequence stages for the batched layout.
__device__ __forceinline__ void merge_batched_geometry(const MergeParams& p, uint32_t b,
                                                       uint64_t& pref, uint64_t& total) {
  const uint32_t lane = threadIdx.x & 31;
  uint64_t before = 0, all = 0;
  for (uint32_t base = 0; base < p.batch; base += 32) {
    const uint32_t s = base + lane;
    uint32_t t = 0;
    if (s < p.batch) {
      const uint32_t len = min(p.seq_lens[s], p.max_tokens);
      t = stages_of_range(0, len);
    }
    uint64_t x = s < b ? t : 0, y = t;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      x += __shfl_xor_sync(0xffffffffu, x, o);
      y += __shfl_xor_sync(0xffffffffu, y, o);
    }
    before += x;
    all += y;
  }
  pref = before;
  total = all * p.kv_heads;
}

// One CTA of kMergeWarps warps merges one row-head. Partials are taken in
// chunks of kMergeWarps * kPerWarp: every thread issues the loads of all its
// partials (m, l and its KD dims of n, d = lane + 32k) before using any, so
// a chunk costs one memory round trip; chunks are folded with a running max.
// KD = ceil(dim / 32) is 2, 4 or 8; kPerWarp keeps up to 40 n values a
// thread in flight (fewer where the registers would not hold them).
template <int MODE, int KD>
__global__ void __launch_bounds__(32 * kMergeWarps, 6) merge_kernel(MergeParams p) {
  constexpr int kPerWarp = KD == 2 ? 12 : (MODE == kMergeBatched ? 32 : 40) / KD;
  __shared__ float red_m[kMergeWarps];
  __shared__ float red_l[kMergeWarps];
  __shared__ float red_n[kMergeWarps][256];
  // The next kernel on the stream may start its prologue now; its own
  // dependency wait still waits for this grid to finish.
  KVB_MERGE_MARK(0);
  grid_launch_dependents();
  grid_dependency_wait();
  KVB_MERGE_MARK(1);
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t rh = blockIdx.x;
  const uint32_t D = p.dim;

  const float *mb, *lb, *nb;
  size_t ms, ls, ns;
  uint32_t np = p.np;
  // kBatched: the pieces of a segment are those of CTAs c_first..c_last that
  // own at least one stage (with fewer stages than CTAs some ranges are empty).
  uint32_t c_first = 0;
  uint64_t total = 0;
  if (MODE == kMergeScratch) {
    mb = p.part + size_t(rh) * p.split_stride * (D + 2);
    lb = mb + 1;
    nb = mb + 2;
    ms = ls = ns = D + 2;
  } else if (MODE == kMergeShards) {
    mb = p.m_parts + rh;
    lb = p.l_parts + rh;
    nb = p.n_parts + size_t(rh) * D;
    ms = ls = p.shard_stride ? p.shard_stride : p.row_heads;
    ns = p.shard_stride ? p.shard_stride : size_t(p.row_heads) * D;
  } else {
    const uint32_t b = rh / p.q_heads, hq = rh % p.q_heads;
    const uint32_t h = hq / p.group, g = hq % p.group;
    uint64_t pref;
    merge_batched_geometry(p, b, pref, total);
    const uint32_t len = min(p.seq_lens[b], p.max_tokens);
    const uint32_t t = stages_of_range(0, len);
    np = 0;
    if (t > 0) {
      const uint64_t seg_off = pref * p.kv_heads + uint64_t(h) * t;
      c_first = cta_of_stage(seg_off, total, p.ctas);
      np = cta_of_stage(seg_off + t - 1, total, p.ctas) - c_first + 1;
    }
    const uint32_t seg = b * p.kv_heads + h;
    mb = p.part + (size_t(c_first + seg) * p.group + g) * (D + 2);
    lb = mb + 1;
    nb = mb + 2;
    ms = ls = ns = size_t(p.group) * (D + 2);
  }

  constexpr int kMaxK = KD;
  float acc[kMaxK];
#pragma unroll
  for (int k = 0; k < kMaxK; ++k) acc[k] = 0.f;
  float M = -INFINITY, Lw = 0.f;  // running max (block-uniform), warp-partial denominator
  for (uint32_t base = 0; base < np; base += kMergeWarps * kPerWarp) {
    float mv[kPerWarp], lv[kPerWarp], nv[kPerWarp][kMaxK];
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
      const uint32_t i = base + warp + kMergeWarps * j;
      bool ok = i < np;
      if (MODE == kMergeBatched && ok)
        ok = cta_stage_begin(c_first + i + 1, total, p.ctas) > cta_stage_begin(c_first + i, total, p.ctas);
      lv[j] = ok ? lb[i * ls] : 0.f;
      mv[j] = ok ? mb[i * ms] : -INFINITY;
#pragma unroll
      for (int k = 0; k < kMaxK; ++k) {
        const uint32_t d = lane + 32 * k;
        nv[j][k] = (ok && d < D) ? nb[i * ns + d] : 0.f;
      }
    }
    float cm = -INFINITY;
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j)
      if (lv[j] > 0.f) cm = fmaxf(cm, mv[j]);
    if (lane == 0) red_m[warp] = cm;
    __syncthreads();
    KVB_MERGE_MARK(3);
    float mnew = M;
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) mnew = fmaxf(mnew, red_m[w]);
    __syncthreads();
    if (mnew == -INFINITY) continue;
    const float alpha = M == -INFINITY ? 0.f : expf(M - mnew);
    Lw *= alpha;
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) acc[k] *= alpha;
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
      // A partial with l = 0 contributes nothing; its n is not read (an
      // empty-split marker leaves n undefined).
      const bool live = lv[j] > 0.f;
      const float e = live ? expf(mv[j] - mnew) : 0.f;
      Lw = fmaf(e, lv[j], Lw);
#pragma unroll
      for (int k = 0; k < kMaxK; ++k) acc[k] = live ? fmaf(e, nv[j][k], acc[k]) : acc[k];
    }
    M = mnew;
  }
  // Fold the warps.
  if (lane == 0) red_l[warp] = Lw;
#pragma unroll
  for (int k = 0; k < kMaxK; ++k) {
    const uint32_t d = lane + 32 * k;
    if (d < D) red_n[warp][d] = acc[k];
  }
  __syncthreads();
  KVB_MERGE_MARK(4);
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < kMergeWarps; ++w) L += red_l[w];
  if (threadIdx.x == 0) {
    p.m[rh] = L > 0.f ? M : -INFINITY;
    p.l[rh] = L;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (uint32_t d = threadIdx.x; d < D; d += 32 * kMergeWarps) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) v += red_n[w][d];
    v = L > 0.f ? v : 0.f;
    p.n[size_t(rh) * D + d] = v;
    if (p.out != nullptr) p.out[size_t(rh) * D + d] = __float2half_rn(v * inv);
    if (p.out_bf16 != nullptr) p.out_bf16[size_t(rh) * D + d] = __float2bfloat16_rn(v * inv);
  }
  if (MODE == kMergeScratch && p.fill_empty) {
    float* row = p.part + size_t(rh) * p.split_stride * (D + 2);
    for (uint32_t i = np + threadIdx.x; i < p.split_stride; i += 32 * kMergeWarps) {
      row[size_t(i) * (D + 2) + 0] = -INFINITY;
      row[size_t(i) * (D + 2) + 1] = 0.f;
    }
  }
  KVB_MERGE_MARK(2);
}

// Number of partials above which a row-head's merge takes merge_wide_kernel:
// merge_kernel reads at most kMergeWarps * 10 partials a round at dim 128.
constexpr uint32_t kMergeWideAbove = 40;

// Warps of a merge_wide_kernel CTA, and the partials it folds per round
// (32 a warp).
constexpr int kMergeWideWarps = 8;
constexpr uint32_t kMergeWideRound = 32 * kMergeWideWarps;

// Merge of many partials per row-head (kScratch, kShards): CTA c merges dims
// [32 s, 32 s + 32) of row-head c / S, S = ceil(dim / 32), so that the S
// slices of a row-head read its partials on S SMs. Partials go in rounds of
// 32 a warp (256 a CTA): lane j loads m and l of the warp's partial j, and
// every lane loads each of those 32 partials' n at its own dim, all before
// any is used; the partials' weights reach the lanes by shuffles. With up to
// 256 partials per row-head (one KV head of cfg2 per GPU) that is one round,
// each round costing one memory round trip (with 4 warps, 128 a round, one
// KV head of cfg2 at 256 partitions took 8.84 us a call).
template <int MODE>
__global__ void __launch_bounds__(32 * kMergeWideWarps, 3) merge_wide_kernel(MergeParams p) {
  static_assert(MODE != kMergeBatched, "the batched layout takes merge_kernel");
  __shared__ float red_m[kMergeWideWarps];
  __shared__ float red_l[kMergeWideWarps];
  __shared__ float red_n[kMergeWideWarps][32];
  KVB_MERGE_MARK(0);
  grid_launch_dependents();
  grid_dependency_wait();
  KVB_MERGE_MARK(1);
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t D = p.dim, slices = (D + 31) / 32;
  const uint32_t rh = blockIdx.x / slices, slice = blockIdx.x % slices;
  const uint32_t d = 32 * slice + lane;
  const bool has_d = d < D;
  const uint32_t np = p.np;

  const float *mb, *lb, *nb;
  size_t ms, ls, ns;
  if (MODE == kMergeScratch) {
    mb = p.part + size_t(rh) * p.split_stride * (D + 2);
    lb = mb + 1;
    nb = mb + 2;
    ms = ls = ns = D + 2;
  } else {
    mb = p.m_parts + rh;
    lb = p.l_parts + rh;
    nb = p.n_parts + size_t(rh) * D;
    ms = ls = p.shard_stride ? p.shard_stride : p.row_heads;
    ns = p.shard_stride ? p.shard_stride : size_t(p.row_heads) * D;
  }

  float acc = 0.f, M = -INFINITY, Lw = 0.f;  // Lw: this lane's partials' share of L
  for (uint32_t base = 0; base < np; base += 32 * kMergeWideWarps) {
    const uint32_t first = base + 32 * warp;
    const uint32_t i = first + lane;  // this lane's partial
    const bool ok = i < np;
    const float lv = ok ? lb[i * ls] : 0.f;
    const float mv = ok ? mb[i * ms] : -INFINITY;
    const uint32_t okmask = __ballot_sync(0xffffffffu, ok);
    float nv[32];
#pragma unroll
    for (int j = 0; j < 32; ++j)
      nv[j] = (((okmask >> j) & 1u) != 0u && has_d) ? nb[size_t(first + j) * ns + d] : 0.f;
    const float cm = warp_max(lv > 0.f ? mv : -INFINITY);
    if (lane == 0) red_m[warp] = cm;
    __syncthreads();
    KVB_MERGE_MARK(3);
    float mnew = M;
#pragma unroll
    for (int w = 0; w < kMergeWideWarps; ++w) mnew = fmaxf(mnew, red_m[w]);
    __syncthreads();
    if (mnew == -INFINITY) continue;
    const float alpha = M == -INFINITY ? 0.f : expf(M - mnew);
    Lw *= alpha;
    acc *= alpha;
    // A partial with l = 0 contributes nothing (an empty-split marker leaves
    // its n undefined).
    const bool live = lv > 0.f;
    const float e = live ? expf(mv - mnew) : 0.f;
    Lw = fmaf(e, lv, Lw);
    const uint32_t livemask = __ballot_sync(0xffffffffu, live);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float ej = __shfl_sync(0xffffffffu, e, j);
      acc = ((livemask >> j) & 1u) != 0u ? fmaf(ej, nv[j], acc) : acc;
    }
    M = mnew;
  }
  Lw = warp_sum(Lw);
  if (lane == 0) red_l[warp] = Lw;
  red_n[warp][lane] = acc;
  __syncthreads();
  KVB_MERGE_MARK(4);
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < kMergeWideWarps; ++w) L += red_l[w];
  if (threadIdx.x == 0 && slice == 0) {
    p.m[rh] = L > 0.f ? M : -INFINITY;
    p.l[rh] = L;
  }
  if (warp == 0 && has_d) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kMergeWideWarps; ++w) v += red_n[w][lane];
    v = L > 0.f ? v : 0.f;
    const float inv = L > 0.f ? 1.f / L : 0.f;
    p.n[size_t(rh) * D + d] = v;
    if (p.out != nullptr) p.out[size_t(rh) * D + d] = __float2half_rn(v * inv);
    if (p.out_bf16 != nullptr) p.out_bf16[size_t(rh) * D + d] = __float2bfloat16_rn(v * inv);
  }
  if (MODE == kMergeScratch && p.fill_empty && slice == 0) {
    float* row = p.part + size_t(rh) * p.split_stride * (D + 2);
    for (uint32_t j = np + threadIdx.x; j < p.split_stride; j += 32 * kMergeWideWarps) {
      row[size_t(j) * (D + 2) + 0] = -INFINITY;
      row[size_t(j) * (D + 2) + 1] = 0.f;
    }
  }
  KVB_MERGE_MARK(2);
}

}  // namespace kvb
