#pragma once
// kvbridge-b200: host shape layer of the paged INT8-KV decode-attention path.
//
// Drop-in for the reference's include/kvbridge/attention_shape.h:1-37
// (dkeryyyy/kvbridge v0.1.0-research). The struct layout, constant and every
// function name/signature are kept identical so code written against the
// reference compiles unchanged; the implementation lives in
// kvbridge_b200/csrc/attention_shape.cpp. No CUDA toolkit is needed for this
// header or its implementation.
#include <cstddef>
#include <cstdint>

namespace kvbridge {

// Token granularity of the reference's split-K scratch layout. The B200
// launcher may use fewer, larger partitions, but scratch is always sized and
// indexed in units of this split (reference attention_shape.h:7).
constexpr unsigned kSplitTokens = 256;

// Geometry of one decode-attention call (reference attention_shape.h:9-13).
//   rows        query rows of ONE sequence that share page table and positions
//   q_heads     query heads per row; kv_heads divides q_heads (GQA group)
//   kv_heads    KV heads stored per physical page
//   dim         head dimension (1..256)
//   page_tokens KV slots per page
//   pages       page-table length == allocated physical pages
//   tokens      logical backing length (<= pages * page_tokens)
//   [begin,end) logical token interval attended by this call
//   scale       finite score scale applied after QK (e.g. 1/sqrt(dim))
//   int8        true: INT8 K/V with per-(page, kv_head, slot) fp32 scales;
//               false: fp32 K/V
struct Shape {
  uint32_t rows, q_heads, kv_heads, dim, page_tokens, pages, tokens, begin, end;
  float scale;
  bool int8;
};

// Metadata validation; never touches device memory or the CUDA runtime.
// attention_shape_error returns nullptr for a valid shape, else a static
// message; validate_shape throws std::invalid_argument with that message.
const char* attention_shape_error(const Shape&) noexcept;
bool attention_shape_valid(const Shape&) noexcept;
void validate_shape(const Shape&);

// Sizing helpers (element counts, not bytes); each validates first and throws
// std::invalid_argument on invalid metadata. An empty [begin,end) still has
// one split whose output is m=-inf, l=0, n=0.
unsigned split_count(const Shape&);
size_t scratch_elements(const Shape&);           // floats of split scratch
size_t output_scalar_elements(const Shape&);     // floats in EACH of m and l
size_t output_numerator_elements(const Shape&);  // floats in n (and in q)

// The reference tensor-core geometry predicate, kept with the reference's
// exact domain (int8, rows 8, group 6, dim 256, page 32, page-aligned begin).
// False for invalid metadata. The B200 kernels accept a wider domain; see
// kvbridge/attention_b200.h for the predicate of the fast path.
bool attention_mma_supported(const Shape&) noexcept;

}  // namespace kvbridge
