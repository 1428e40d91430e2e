#pragma once
// Pre-launch buffer checks with the reference's error behaviour
// (src/attention_launch_checks.h:8-27): metadata and null/misaligned buffers
// throw std::invalid_argument before anything is enqueued; CUDA failures
// throw std::runtime_error naming the operation.
#include <cstdint>
#include <stdexcept>
#include <string>

#include "kvbridge/attention_common.h"

namespace kvbridge::detail {

inline bool aligned_to(const void* p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

inline void check_outputs(const Shape& s, const void* scratch, const float* m, const float* l,
                          const float* n) {
  validate_shape(s);
  if (scratch == nullptr || m == nullptr || l == nullptr || n == nullptr)
    throw std::invalid_argument("scratch, m, l and n must be non-null device buffers");
}

inline void check_inputs(const Shape& s, const DeviceInput& in, const void* scratch,
                         const float* m, const float* l, const float* n) {
  check_outputs(s, scratch, m, l, n);
  const bool missing = in.q == nullptr || in.q_positions == nullptr ||
                       in.k_positions == nullptr || in.page_table == nullptr ||
                       in.k == nullptr || in.v == nullptr ||
                       (s.int8 && (in.k_scales == nullptr || in.v_scales == nullptr));
  if (missing) throw std::invalid_argument("attention input device buffers must be non-null");
  // The reference vectorises int8 K/V with 4-byte loads under these conditions
  // and rejects unaligned buffers there; keep the same acceptance rule.
  if (s.int8 && s.dim % 4 == 0 && s.page_tokens % 4 == 0 &&
      (!aligned_to(in.k, 4) || !aligned_to(in.v, 4)))
    throw std::invalid_argument("vectorized INT8 K/V buffers must be 4-byte aligned");
}

inline void cuda_ok(cudaError_t code, const char* what) {
  if (code != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(code));
}

}  // namespace kvbridge::detail
