#pragma once
// kvbridge-b200 extensions beyond the reference interface. Everything here is
// additive: the reference entry points in attention_common.h keep their
// contract, and these functions reuse the same memory formats.
//
//   * launch_attention_ex     - the single-sequence call with an explicit
//                               split-K partition count and a fused fp16
//                               normalised-output epilogue.
//   * launch_attention_batched- ragged batch of decode sequences over one
//                               shared page pool (block table per sequence).
//   * merge_attention_shards  - log-sum-exp merge of per-GPU (m, l, n)
//                               triples for sequence-sharded decode.
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include "kvbridge/attention_common.h"

namespace kvbridge {

struct LaunchOptions {
  // Split-K partitions per KV head. 0 lets the launcher choose from the SM
  // count; otherwise clamped to [1, split_count(shape)] and to the number of
  // 64-token stages in [begin,end).
  unsigned partitions;
  // Optional __half[rows * q_heads * dim]: out = n / l where l > 0, else 0.
  void* out_f16;
  // Optional __nv_bfloat16[rows * q_heads * dim], the same n / l in bf16 (for
  // an out-projection that takes bf16 activations). Either, both or neither.
  void* out_bf16 = nullptr;
};

// True when launch_attention(_ex) will use the TMA/tensor-core kernel for this
// shape and these buffers (int8 KV, dim in {64,128,256}, page_tokens 16, 32
// or 64, rows*group <= 64, 16-byte aligned K/V/scale buffers). Host-only.
bool attention_b200_supported(const Shape&, const DeviceInput&) noexcept;

// Partition count launch_attention_ex will use (host-only; needs the SM count
// of the current device, which it queries once per device).
unsigned attention_partitions(const Shape&, unsigned requested);

void launch_attention_ex(const Shape&, const DeviceInput&, const LaunchOptions&,
                         float* scratch, float* m, float* l, float* n, cudaStream_t);

// The two halves of launch_attention_ex on the tensor-core path, for callers
// that merge partials themselves (e.g. across GPUs). launch_attention_partials
// writes one (m, l, n) partial per partition into the leading splits of the
// scratch layout of attention_common.h, marks the remaining splits as empty
// partials, and returns the partition count used
// (0 for an empty range, where nothing is launched); it throws
// std::invalid_argument unless attention_b200_supported(shape, input).
// merge_attention_ex merges the leading `partitions` splits of every
// row-head (partitions <= split_count(shape)), marks the remaining splits as
// empty partials, and optionally writes the fp16 output n / l.
unsigned launch_attention_partials(const Shape&, const DeviceInput&, unsigned partitions,
                                   float* scratch, cudaStream_t);
void merge_attention_ex(const Shape&, const float* scratch, unsigned partitions, float* m,
                        float* l, float* n, void* out_f16, cudaStream_t);
// The same with an optional bf16 output beside (or instead of) the fp16 one.
void merge_attention_ex(const Shape&, const float* scratch, unsigned partitions, float* m,
                        float* l, float* n, void* out_f16, void* out_bf16, cudaStream_t);

// Ragged batch: sequence b attends its tokens [0, seq_lens[b]) (all visible;
// the query is the next token). Logical page j of sequence b lives at physical
// page block_table[b * table_stride + j] of the shared pool, whose K/V/scale
// layout is the one of attention_common.h with `pages` physical pages. Unlike
// the single-sequence Shape, the pool may exceed 2^32 elements (64-bit offsets).
struct BatchShape {
  uint32_t batch, q_heads, kv_heads, dim, page_tokens, pages, table_stride;
  uint32_t max_tokens;  // host-known upper bound of every seq_lens[b]
  float scale;
};
struct BatchInput {
  const float* q;               // float[batch * q_heads * dim]
  const uint32_t* seq_lens;     // uint32[batch], each <= max_tokens
  const uint32_t* block_table;  // uint32[batch * table_stride]
  const int8_t* k;
  const int8_t* v;
  const float* k_scales;
  const float* v_scales;
};
const char* batch_shape_error(const BatchShape&) noexcept;
// Bytes of caller-owned workspace launch_attention_batched needs on the
// current device (partials of every CTA/sequence piece).
size_t batch_workspace_bytes(const BatchShape&);
// Outputs: m, l float[batch * q_heads]; n float[batch * q_heads * dim];
// out_f16 optional __half[batch * q_heads * dim].
void launch_attention_batched(const BatchShape&, const BatchInput&, void* workspace,
                              size_t workspace_bytes, float* m, float* l, float* n,
                              void* out_f16, cudaStream_t);
// The same with an optional bf16 output beside (or instead of) the fp16 one.
void launch_attention_batched(const BatchShape&, const BatchInput&, void* workspace,
                              size_t workspace_bytes, float* m, float* l, float* n,
                              void* out_f16, void* out_bf16, cudaStream_t);

// Merge `shards` partial results, shard-major: m_parts/l_parts
// float[shards * row_heads], n_parts float[shards * row_heads * dim]. The
// result uses the same m/l/n convention (m = -inf, l = 0, n = 0 when no shard
// saw a visible token).
void merge_attention_shards(unsigned shards, unsigned row_heads, unsigned dim,
                            const float* m_parts, const float* l_parts, const float* n_parts,
                            float* m, float* l, float* n, void* out_f16, cudaStream_t);
// The same with a shard stride and an optional bf16 output. shard_stride is
// the distance in floats from one shard's m (and l, and n) to the next
// shard's: 0 keeps the layout above; row_heads * (dim + 2) reads a packed
// exchange buffer [shard][m | l | n] (one all-gather of every rank's
// partial, m at 0, l at row_heads, n at 2 * row_heads of each block).
void merge_attention_shards_ex(unsigned shards, unsigned row_heads, unsigned dim,
                               const float* m_parts, const float* l_parts, const float* n_parts,
                               size_t shard_stride, float* m, float* l, float* n, void* out_f16,
                               void* out_bf16, cudaStream_t);

// Cross-GPU merge of sequence shards over NVLink peer memory, in place of an
// all-gather followed by merge_attention_shards_ex: one kernel exchanges and
// merges. Each of the `world` ranks (one process per GPU, at most 8) owns a
// peer buffer of peer_buffer_bytes(row_heads, dim) bytes from
// peer_buffer_alloc, exported to the other ranks by its 64-byte CUDA IPC
// handle and mapped there with peer_buffer_open. Call number `epoch` (1, 2,
// ... counted by each rank alike) writes the rank's partials (m, l, n as in
// the packed layout above) into peer_slot(own buffer, epoch, ...) and then
// calls merge_attention_peers with every rank's buffer base (its own at
// [rank]) on the same stream: the kernel publishes the slot to every rank,
// waits (up to the wait limit, status 7 when it runs out) until every rank
// has published this epoch, reads their slots over NVLink and writes the
// merged m, l, n (and fp16 / bf16 outputs) of all row_heads. A rank must
// not start call epoch + 2 before its call epoch + 1 returned on the stream.
size_t peer_buffer_bytes(unsigned row_heads, unsigned dim);
float* peer_slot(void* buffer, unsigned epoch, unsigned row_heads, unsigned dim);
void peer_buffer_alloc(size_t bytes, void** buffer, unsigned char handle[64]);
void peer_buffer_open(const unsigned char handle[64], void** peer_buffer);
void peer_buffer_close(void* peer_buffer);
void peer_buffer_free(void* buffer);
void merge_attention_peers(const void* const* buffers, unsigned world, unsigned rank, unsigned epoch,
                           unsigned row_heads, unsigned dim, float* m, float* l, float* n, void* out_f16,
                           void* out_bf16, cudaStream_t);

// Paged KV append (the step before decode; no counterpart in the reference,
// whose fixtures write codes and scales directly): quantises new K and V rows
// with the symmetric per-(token, kv-head) absmax rule -- scale = max|x| / 127,
// code = clamp(rint(x / scale), -127, 127), fp32, ties to even; scale 0 and
// codes 0 for an all-zero row -- and writes codes and scales into the pool
// layout of attention_common.h. Row t goes to physical slot slots[t] =
// page * page_tokens + position in page (negative: skipped); a slot at or
// beyond pages * page_tokens is skipped and reported through
// read_device_status. Rows of one call must target distinct slots.
struct AppendShape {
  uint32_t tokens;  // rows to append (0: nothing is launched)
  uint32_t kv_heads, dim, page_tokens, pages;
};
struct AppendInput {
  const float* k_new;    // float[tokens * kv_heads * dim]
  const float* v_new;    // float[tokens * kv_heads * dim]
  const int64_t* slots;  // int64[tokens]
  int8_t* k;             // the pool (attention_common.h layout)
  int8_t* v;
  float* k_scales;
  float* v_scales;
};
const char* append_shape_error(const AppendShape&) noexcept;
void append_kv(const AppendShape&, const AppendInput&, cudaStream_t);

// Status word written by the kernels' bounded waits (0 = ok). Reading clears
// it. A nonzero value means a pipeline wait gave up and that call's outputs
// are invalid.
cudaError_t read_device_status(int* status);
// The first bounded wait that gave up since the last read (all zero if none):
// {status code, block, warp, stage, waited ns, waited SM cycles}. Reading
// clears it.
cudaError_t read_wait_failure(long long* record6);

// Upper bound, in nanoseconds, of any single pipeline wait inside the kernels
// launched after this call (process-wide; 0 restores the default of 2 s). A
// correct call never waits more than microseconds; the bound only turns a
// broken pipeline into a status code instead of a held GPU.
void set_wait_limit_ns(unsigned long long ns) noexcept;
unsigned long long wait_limit_ns() noexcept;

namespace detail {
// Test hooks for the failure paths (no effect unless armed; both are
// thread-local and one-shot).
//  * fail_launch(nth, code): the nth kernel launch this library makes on the
//    calling thread after the call (1 = the next one) is not made; the call
//    that would make it throws std::runtime_error with cudaGetErrorString(code)
//    as if the launch had failed. nth = 0 disarms.
//  * skip_stage(stage): in the next tensor-core partial launch on the calling
//    thread, the producer of CTA 0 leaves its pipeline stage `stage` unarmed,
//    so that a consumer wait runs into the wait limit and the kernel reports
//    status 1 and returns.
void fail_launch(unsigned nth, cudaError_t code) noexcept;
void skip_stage(unsigned stage) noexcept;
// Which single-sequence partial kernel later calls use (process-wide): 0 =
// chosen by shape (default), 1 = the warp-level MMA kernel, 2 = the tcgen05
// (TMEM accumulator) kernel wherever it has a variant for the shape, 3 = the
// general CUDA-core kernel for every launch_attention / launch_attention_ex
// call (int8 or fp32 KV; the partials-only entry points keep the
// tensor-core kernels). For side-by-side measurements and tests; results
// agree within the tolerance.
void set_decode_kernel(int choice) noexcept;
int decode_kernel() noexcept;
}  // namespace detail

}  // namespace kvbridge
