#pragma once
// kvbridge-b200: public C++ interface of the paged INT8-KV grouped-query
// split-K decode-attention path, drop-in for the reference's
// include/kvbridge/attention_common.h:1-97. Names, argument order, ownership
// and error behaviour are unchanged; the kernels behind them are new sm_100a
// code (kvbridge_b200/csrc).
//
// Memory formats (device pointers, all caller-owned):
//   q           float[rows * q_heads * dim]      row-major fp32 query
//   q_positions int64[rows]                      absolute position of each row
//   k_positions int64[tokens]                    position of each logical token,
//                                                nondecreasing in token order
//   page_table  uint32[pages]                    logical page -> physical page
//   k           int8[((page * kv_heads + kv) * page_tokens + slot) * dim + d]
//   v           int8[((page * kv_heads + kv) * dim + d) * page_tokens + slot]
//   k_scales    float[(page * kv_heads + kv) * page_tokens + slot]
//   v_scales    float[same index as k_scales]
// (fp32 KV, Shape::int8 == false: k and v are float[] in the same index order
// and the scale pointers are ignored.)
//
// A key token t in [begin,end) is visible to query row r iff
// k_positions[t] <= q_positions[r]. Per (row, head) the call produces
//   m = max visible score, l = sum exp(score - m), n[d] = sum exp(score - m) * v[d]
// with score = scale * sum_d q[d] * k[d] * k_scale and v = code * v_scale.
// The caller normalises out = n / l where l > 0; empty or fully masked rows
// return m = -inf, l = 0, n = 0.
//
// Sizes (floats): m, l: output_scalar_elements; n: output_numerator_elements;
// scratch: scratch_elements. Scratch layout (reference attention_common.h:43-46):
//   scratch[((row * q_heads + head) * splits + split) * (dim + 2) + col]
//   col 0 = split max, 1 = split denominator, 2.. = split numerator,
// with splits = split_count(shape). After launch_attention the B200 launcher
// leaves a valid decomposition there: its partitions occupy the leading split
// slots and the remaining slots hold empty partials (m = -inf, l = 0), so
// merge_attention(shape, scratch, split_count(shape), ...) reproduces m/l/n.
//
// Buffers must be sized as above, must not overlap, and stay valid until the
// caller synchronises the stream. The library allocates nothing.
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include "kvbridge/attention_shape.h"

namespace kvbridge {

// Device pointers of one call (reference attention_common.h:54-63).
struct DeviceInput {
  const float* q;
  const int64_t* q_positions;
  const int64_t* k_positions;
  const uint32_t* page_table;
  const void* k;            // int8[] (or float[] when Shape::int8 is false)
  const void* v;
  const float* k_scales;    // ignored for fp32 KV
  const float* v_scales;
};

// Eager module load of every kernel in the current context (reference
// attention_common.h:69-72). Return the first CUDA failure; the B200 library
// returns cudaErrorNotSupported on a device other than sm_100.
cudaError_t preload_attention_kernels();
cudaError_t preload_attention_reference_kernels();
cudaError_t preload_attention_mma_kernels();

// Decode attention for a valid Shape (reference attention_common.h:80-81).
// INT8 KV runs the sm_100a TMA/tensor-core split-K kernel wherever its
// geometry allows it, and an sm_100a SIMT kernel otherwise (fp32 KV,
// unaligned buffers, head dims that are not a multiple of 16, ...).
// Invalid metadata or null/misaligned buffers throw std::invalid_argument
// before anything is enqueued; CUDA launch failures throw std::runtime_error.
void launch_attention(const Shape&, const DeviceInput&, float* scratch,
                      float* m, float* l, float* n, cudaStream_t);

// Same contract as the reference (attention_common.h:90-91): throws
// std::invalid_argument unless attention_mma_supported(shape); there is no
// implicit fallback. Runs the same B200 kernels as launch_attention.
void launch_attention_mma(const Shape&, const DeviceInput&, float* scratch,
                          float* m, float* l, float* n, cudaStream_t);

// Merge `splits` partials of the scratch layout above into m/l/n
// (reference attention_common.h:95-96). splits must equal split_count(shape).
void merge_attention(const Shape&, const float* scratch, unsigned splits,
                     float* m, float* l, float* n, cudaStream_t);

}  // namespace kvbridge
