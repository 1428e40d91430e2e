// TEST INFRASTRUCTURE - C wrapper around the reference repository's own CUDA
// launchers (src/attention_shared.cu:339-374 SIMT + merge, src/attention_mma.cu:
// 33-45 MMA), compiled for sm_100a from the reference's sources by
// oracle/Makefile into oracle/_ref/. GPU tests use it to compare this
// repository's kernels with the reference's own kernels on identical device
// inputs. Nothing in the product links it.
#include <cstdint>
#include <exception>
#include <stdexcept>

#include "kvbridge/attention_common.h"

namespace {
kvbridge::Shape make_shape(const uint32_t* d, float scale, int int8) {
  return kvbridge::Shape{d[0], d[1], d[2], d[3], d[4], d[5], d[6], d[7], d[8], scale, int8 != 0};
}
kvbridge::DeviceInput make_input(void* const* p) {
  return kvbridge::DeviceInput{static_cast<const float*>(p[0]),   static_cast<const int64_t*>(p[1]),
                               static_cast<const int64_t*>(p[2]), static_cast<const uint32_t*>(p[3]),
                               p[4],                              p[5],
                               static_cast<const float*>(p[6]),   static_cast<const float*>(p[7])};
}
template <class F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::invalid_argument&) {
    return 1;
  } catch (const std::exception&) {
    return 2;
  }
}
}  // namespace

extern "C" {

// dims = {rows, q_heads, kv_heads, dim, page_tokens, pages, tokens, begin, end};
// ptrs = {q, q_positions, k_positions, page_table, k, v, k_scales, v_scales}.
int kvbref_cuda_launch_attention(const uint32_t* dims, float scale, int int8, void* const* ptrs,
                                 float* scratch, float* m, float* l, float* n, void* stream) {
  return guarded([&] {
    kvbridge::launch_attention(make_shape(dims, scale, int8), make_input(ptrs), scratch, m, l, n,
                               static_cast<cudaStream_t>(stream));
  });
}

int kvbref_cuda_launch_attention_mma(const uint32_t* dims, float scale, int int8,
                                     void* const* ptrs, float* scratch, float* m, float* l,
                                     float* n, void* stream) {
  return guarded([&] {
    kvbridge::launch_attention_mma(make_shape(dims, scale, int8), make_input(ptrs), scratch, m, l,
                                   n, static_cast<cudaStream_t>(stream));
  });
}

int kvbref_cuda_preload_reference(void) {
  return int(kvbridge::preload_attention_reference_kernels());
}

}  // extern "C"
