#pragma once
// Split-K work schedule shared by the host launcher, the partial kernel and
// the merge kernel.
//
// The attended KV of a call is a list of segments, one per (sequence, KV
// head), each a run of 64-token stages. Concatenating the segments gives
// `total` global stages, which are cut into `ctas` contiguous, equally sized
// ranges: CTA c owns global stages [floor(c*total/ctas), floor((c+1)*total/ctas)).
// Every (CTA range, segment) intersection is one "piece" and produces one
// split-K partial. Work per CTA is balanced to one stage regardless of how
// ragged the segments are.
//
// For a single sequence launched with ctas = partitions * kv_heads every
// segment has exactly `partitions` pieces, piece i of head h being CTA
// h * partitions + i (the CTA boundaries c*T/partitions land on segment
// boundaries for c a multiple of partitions).
#include <cstdint>

#if defined(__CUDACC__)
#define KVB_HD __host__ __device__ __forceinline__
#else
#define KVB_HD inline
#endif

namespace kvb {

constexpr uint32_t kStageTokens = 64;

// First global stage of CTA c.
KVB_HD uint64_t cta_stage_begin(uint32_t c, uint64_t total, uint32_t ctas) {
  return (uint64_t(c) * total) / ctas;
}

// The CTA whose range holds global stage x (0 <= x < total): the largest c
// with floor(c*total/ctas) <= x, i.e. c*total < (x+1)*ctas.
KVB_HD uint32_t cta_of_stage(uint64_t x, uint64_t total, uint32_t ctas) {
  return static_cast<uint32_t>(((x + 1) * uint64_t(ctas) - 1) / total);
}

// Stages covering the logical token interval [lo, hi) (0 when empty).
KVB_HD uint32_t stages_of_range(uint32_t lo, uint32_t hi) {
  if (hi <= lo) return 0;
  return (hi + kStageTokens - 1) / kStageTokens - lo / kStageTokens;
}

}  // namespace kvb
