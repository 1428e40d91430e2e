// Host shape validation and sizing for the decode-attention path.
//
// Restates the reference's metadata rules (src/attention_shape.cpp:20-70) so
// that every integer result and every accept/reject decision is bit-identical:
// the checks run in the same order and return the same messages, because
// callers of the reference may match on them. Products are evaluated in 64
// bits with explicit overflow guards.
#include "kvbridge/attention_shape.h"

#include <cmath>
#include <cstdint>
#include <limits>
#include <stdexcept>

namespace kvbridge {
namespace {

constexpr uint64_t kU32Max = std::numeric_limits<uint32_t>::max();
constexpr uint64_t kFloatsMax = std::numeric_limits<size_t>::max() / sizeof(float);

// Number of kSplitTokens splits covering [begin,end); an empty interval keeps
// one split (reference attention_shape.cpp:9-12).
uint64_t raw_splits(const Shape& s) noexcept {
  const uint64_t span = uint64_t(s.end) - uint64_t(s.begin);
  if (span == 0) return 1;
  return (span + kSplitTokens - 1) / kSplitTokens;
}

// acc *= factor unless the product would exceed `limit`.
bool scaled_within(uint64_t& acc, uint64_t factor, uint64_t limit) noexcept {
  if (factor != 0 && acc > limit / factor) return false;
  acc *= factor;
  return true;
}

}  // namespace

const char* attention_shape_error(const Shape& s) noexcept {
  if (s.rows == 0 || s.q_heads == 0 || s.kv_heads == 0)
    return "rows and head counts must be positive";
  if (s.q_heads % s.kv_heads != 0) return "q_heads must be divisible by kv_heads";
  if (s.dim == 0 || s.dim > 256) return "dim must be in [1,256]";
  if (s.page_tokens == 0 || s.pages == 0 || s.tokens == 0)
    return "page_tokens, pages and tokens must be positive";
  if (s.begin > s.end || s.end > s.tokens) return "require begin <= end <= tokens";
  if (uint64_t(s.tokens) > uint64_t(s.pages) * uint64_t(s.page_tokens))
    return "tokens exceed allocated page capacity";
  if (!std::isfinite(s.scale)) return "score scale must be finite";
  if (raw_splits(s) > 65535) return "range exceeds CUDA grid-y split limit";
  if (uint64_t(s.rows) * uint64_t(s.q_heads) > 0x7fffffffull)
    return "row/head product exceeds CUDA grid-x limit";
  // Physical KV element extent pages*kv_heads*page_tokens*dim must stay a
  // 32-bit offset (it indexes int8 K/V).
  uint64_t extent = s.pages;
  if (!scaled_within(extent, s.kv_heads, kU32Max) ||
      !scaled_within(extent, s.page_tokens, kU32Max) ||
      !scaled_within(extent, s.dim, kU32Max))
    return "physical KV extent exceeds 32-bit kernel offsets";
  uint64_t scratch = uint64_t(s.rows) * uint64_t(s.q_heads);
  if (!scaled_within(scratch, raw_splits(s), kFloatsMax) ||
      !scaled_within(scratch, uint64_t(s.dim) + 2, kFloatsMax))
    return "scratch byte size exceeds size_t";
  if (extent > kFloatsMax ||
      uint64_t(s.tokens) > std::numeric_limits<size_t>::max() / sizeof(int64_t) ||
      uint64_t(s.pages) > std::numeric_limits<size_t>::max() / sizeof(uint32_t))
    return "input byte size exceeds size_t";
  return nullptr;
}

bool attention_shape_valid(const Shape& s) noexcept { return attention_shape_error(s) == nullptr; }

void validate_shape(const Shape& s) {
  const char* why = attention_shape_error(s);
  if (why != nullptr) throw std::invalid_argument(why);
}

unsigned split_count(const Shape& s) {
  validate_shape(s);
  return static_cast<unsigned>(raw_splits(s));
}

size_t scratch_elements(const Shape& s) {
  validate_shape(s);
  return size_t(s.rows) * size_t(s.q_heads) * size_t(raw_splits(s)) * (size_t(s.dim) + 2);
}

size_t output_scalar_elements(const Shape& s) {
  validate_shape(s);
  return size_t(s.rows) * size_t(s.q_heads);
}

size_t output_numerator_elements(const Shape& s) {
  return output_scalar_elements(s) * size_t(s.dim);
}

bool attention_mma_supported(const Shape& s) noexcept {
  if (!attention_shape_valid(s)) return false;
  return s.int8 && s.rows == 8 && s.dim == 256 && s.page_tokens == 32 &&
         s.q_heads / s.kv_heads == 6 && s.begin % 32 == 0;
}

}  // namespace kvbridge
