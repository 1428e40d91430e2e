/* kvbridge-b200 C ABI: plain pointers, sizes and status codes, no C++ types
 * and no exceptions. Each function mirrors one entry point of the reference's
 * C++ interface (dkeryyyy/kvbridge, include/kvbridge/attention_common.h and
 * attention_shape.h) or of the B200 extensions in kvbridge/attention_b200.h.
 *
 * Status codes: KVB_OK on success; KVB_EINVAL where the C++ API throws
 * std::invalid_argument (bad metadata, null or misaligned buffers, nothing was
 * enqueued); KVB_ECUDA where it throws std::runtime_error (CUDA launch or
 * setup failure). kvb_last_error() returns the message of the calling
 * thread's last failure.
 *
 * Streams are passed as `void*` (a cudaStream_t; NULL = legacy default
 * stream). All buffers are device pointers owned by the caller. */
#ifndef KVBRIDGE_C_H
#define KVBRIDGE_C_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVB_OK 0
#define KVB_EINVAL 1
#define KVB_ECUDA 2

/* Same field order and layout as kvbridge::Shape
 * (reference include/kvbridge/attention_shape.h:9-13). */
typedef struct kvb_shape {
  uint32_t rows, q_heads, kv_heads, dim, page_tokens, pages, tokens, begin, end;
  float scale;
  bool int8;
} kvb_shape;

/* Same field order as kvbridge::DeviceInput
 * (reference include/kvbridge/attention_common.h:54-63). */
typedef struct kvb_device_input {
  const float* q;
  const int64_t* q_positions;
  const int64_t* k_positions;
  const uint32_t* page_table;
  const void* k;
  const void* v;
  const float* k_scales;
  const float* v_scales;
} kvb_device_input;

/* Message of the calling thread's last failed call ("" if none). */
const char* kvb_last_error(void);

/* ---- shape layer: reference src/attention_shape.cpp:20-70 ---- */
/* attention_shape_error: NULL when valid, else a static message. */
const char* kvb_attention_shape_error(const kvb_shape* s);
bool kvb_attention_shape_valid(const kvb_shape* s);
/* validate_shape / split_count / scratch_elements / output_*_elements:
 * KVB_EINVAL (with the validation message) instead of throwing. */
int kvb_validate_shape(const kvb_shape* s);
int kvb_split_count(const kvb_shape* s, unsigned* splits);
int kvb_scratch_elements(const kvb_shape* s, size_t* elements);
int kvb_output_scalar_elements(const kvb_shape* s, size_t* elements);
int kvb_output_numerator_elements(const kvb_shape* s, size_t* elements);
bool kvb_attention_mma_supported(const kvb_shape* s);

/* ---- kernels: reference include/kvbridge/attention_common.h:69-96 ---- */
/* preload_*: return the cudaError_t value (0 = cudaSuccess). */
int kvb_preload_attention_kernels(void);
int kvb_preload_attention_reference_kernels(void);
int kvb_preload_attention_mma_kernels(void);
/* reference launch_attention (src/attention_shared.cu:339) */
int kvb_launch_attention(const kvb_shape* s, const kvb_device_input* in, float* scratch,
                         float* m, float* l, float* n, void* stream);
/* reference launch_attention_mma (src/attention_mma.cu:33) */
int kvb_launch_attention_mma(const kvb_shape* s, const kvb_device_input* in, float* scratch,
                             float* m, float* l, float* n, void* stream);
/* reference merge_attention (src/attention_shared.cu:368) */
int kvb_merge_attention(const kvb_shape* s, const float* scratch, unsigned splits,
                        float* m, float* l, float* n, void* stream);

/* ---- B200 extensions (kvbridge/attention_b200.h) ---- */
bool kvb_attention_b200_supported(const kvb_shape* s, const kvb_device_input* in);
/* partitions the launcher will use for `requested` (0 = automatic) */
int kvb_attention_partitions(const kvb_shape* s, unsigned requested, unsigned* partitions);
/* launch_attention with explicit partitions and optional fp16 output n/l */
int kvb_launch_attention_ex(const kvb_shape* s, const kvb_device_input* in, unsigned partitions,
                            void* out_f16, float* scratch, float* m, float* l, float* n,
                            void* stream);

/* kvb_launch_attention_ex with an optional bf16 output beside (or instead
 * of) the fp16 one (kvbridge::LaunchOptions::out_bf16); either may be NULL. */
int kvb_launch_attention_ex2(const kvb_shape* s, const kvb_device_input* in, unsigned partitions,
                             void* out_f16, void* out_bf16, float* scratch, float* m, float* l,
                             float* n, void* stream);

/* the two halves of kvb_launch_attention_ex (partial kernel; merge of the
 * leading `partitions` splits). *partitions_used may be NULL. */
int kvb_launch_attention_partials(const kvb_shape* s, const kvb_device_input* in,
                                  unsigned partitions, float* scratch, unsigned* partitions_used,
                                  void* stream);
int kvb_merge_attention_ex(const kvb_shape* s, const float* scratch, unsigned partitions,
                           float* m, float* l, float* n, void* out_f16, void* stream);
/* kvb_merge_attention_ex with an optional bf16 output as well. */
int kvb_merge_attention_ex2(const kvb_shape* s, const float* scratch, unsigned partitions,
                            float* m, float* l, float* n, void* out_f16, void* out_bf16,
                            void* stream);

typedef struct kvb_batch_shape {
  uint32_t batch, q_heads, kv_heads, dim, page_tokens, pages, table_stride, max_tokens;
  float scale;
} kvb_batch_shape;

typedef struct kvb_batch_input {
  const float* q;
  const uint32_t* seq_lens;
  const uint32_t* block_table;
  const int8_t* k;
  const int8_t* v;
  const float* k_scales;
  const float* v_scales;
} kvb_batch_input;

const char* kvb_batch_shape_error(const kvb_batch_shape* s);
int kvb_batch_workspace_bytes(const kvb_batch_shape* s, size_t* bytes);
int kvb_launch_attention_batched(const kvb_batch_shape* s, const kvb_batch_input* in,
                                 void* workspace, size_t workspace_bytes, float* m, float* l,
                                 float* n, void* out_f16, void* stream);
/* kvb_launch_attention_batched with an optional bf16 output as well. */
int kvb_launch_attention_batched2(const kvb_batch_shape* s, const kvb_batch_input* in,
                                  void* workspace, size_t workspace_bytes, float* m, float* l,
                                  float* n, void* out_f16, void* out_bf16, void* stream);
/* paged KV append: quantise and write new K/V rows (kvbridge/attention_b200.h) */
typedef struct kvb_append_shape {
  uint32_t tokens, kv_heads, dim, page_tokens, pages;
} kvb_append_shape;

typedef struct kvb_append_input {
  const float* k_new;
  const float* v_new;
  const int64_t* slots;
  int8_t* k;
  int8_t* v;
  float* k_scales;
  float* v_scales;
} kvb_append_input;

const char* kvb_append_shape_error(const kvb_append_shape* s);
int kvb_append_kv(const kvb_append_shape* s, const kvb_append_input* in, void* stream);

int kvb_merge_attention_shards(unsigned shards, unsigned row_heads, unsigned dim,
                               const float* m_parts, const float* l_parts,
                               const float* n_parts, float* m, float* l, float* n,
                               void* out_f16, void* stream);
/* kvb_merge_attention_shards with a shard stride (floats from one shard's m,
 * l and n to the next shard's; 0 = the layout above) and an optional bf16
 * output. A packed all-gather buffer [shard][m | l | n] is read with
 * m_parts = buf, l_parts = buf + row_heads, n_parts = buf + 2 * row_heads and
 * shard_stride = row_heads * (dim + 2). */
int kvb_merge_attention_shards_ex(unsigned shards, unsigned row_heads, unsigned dim,
                                  const float* m_parts, const float* l_parts,
                                  const float* n_parts, size_t shard_stride, float* m, float* l,
                                  float* n, void* out_f16, void* out_bf16, void* stream);
/* Cross-GPU merge of sequence shards over NVLink peer memory, in place of an
 * all-gather followed by kvb_merge_attention_shards_ex (one kernel exchanges
 * and merges). Each rank (one process per GPU, at most 8) allocates a peer
 * buffer of kvb_peer_buffer_bytes(row_heads, dim) bytes with
 * kvb_peer_buffer_alloc, which also returns its 64-byte CUDA IPC handle; the
 * ranks exchange handles (any host channel) and map each other's buffers
 * with kvb_peer_buffer_open. Call number `epoch` (1, 2, ..., counted alike on
 * every rank) writes the rank's partials into kvb_peer_slot(own buffer,
 * epoch, row_heads, dim) - packed [m | l | n]: m at 0, l at row_heads, n at
 * 2 * row_heads floats - and then calls kvb_merge_attention_peers on the same
 * stream with every rank's buffer ([rank] = its own). The kernel publishes
 * the slot to every rank, waits until every rank published this epoch (up
 * to the wait limit; status 7 and no output when it runs out), reads their
 * slots over NVLink and writes the merged m, l, n and optional fp16 / bf16
 * outputs. A rank starts call epoch + 2 only after its call epoch + 1 has
 * returned on its stream (the two slots alternate). kvb_peer_buffer_close
 * unmaps a peer's buffer and kvb_peer_buffer_free releases one's own.
 * kvb_peer_buffer_bytes returns 0 for an invalid shape. */
size_t kvb_peer_buffer_bytes(unsigned row_heads, unsigned dim);
float* kvb_peer_slot(void* buffer, unsigned epoch, unsigned row_heads, unsigned dim);
int kvb_peer_buffer_alloc(size_t bytes, void** buffer, unsigned char* handle64);
int kvb_peer_buffer_open(const unsigned char* handle64, void** peer_buffer);
int kvb_peer_buffer_close(void* peer_buffer);
int kvb_peer_buffer_free(void* buffer);
int kvb_merge_attention_peers(const void* const* buffers, unsigned world, unsigned rank, unsigned epoch,
                              unsigned row_heads, unsigned dim, float* m, float* l, float* n, void* out_f16,
                              void* out_bf16, void* stream);
/* Test hook: copies `bytes` from host memory to a device address (for
 * instance a peer buffer's flag or slot, which no tensor library wraps). */
int kvb_debug_copy_to_device(void* dst, const void* src, size_t bytes);
/* Reads and clears the kernels' device status word (0 = ok). Returns the
 * cudaError_t of the read. */
int kvb_read_device_status(int* status);
/* The first bounded wait that gave up since the last read: six values
 * {code, block, warp, stage, waited ns, waited SM cycles}; all zero if none.
 * Reading clears it. Returns the cudaError_t of the read. */
int kvb_read_wait_failure(long long* record6);
/* Upper bound in ns of any single pipeline wait in kernels launched after
 * the call (process-wide; 0 = the default 2 s). */
void kvb_set_wait_limit_ns(unsigned long long ns);
unsigned long long kvb_wait_limit_ns(void);

/* Test hooks for the failure paths; thread-local and one-shot.
 * kvb_debug_fail_launch: the nth kernel launch (1 = the next) this library
 * makes on the calling thread is not made and the call that would make it
 * returns KVB_ECUDA with cudaGetErrorString(cuda_error) in its message; 0
 * disarms. kvb_debug_skip_stage: in the next tensor-core partial launch on
 * the calling thread, the producer of CTA 0 leaves pipeline stage `stage`
 * unarmed, so a consumer wait runs into the wait limit, status 1 is recorded
 * (kvb_read_device_status, kvb_read_wait_failure) and the kernel returns. */
int kvb_debug_fail_launch(unsigned nth, int cuda_error);
int kvb_debug_skip_stage(unsigned stage);

/* Which single-sequence partial kernel later calls use (process-wide):
 * KVB_KERNEL_AUTO chooses by shape, KVB_KERNEL_WARP_MMA the warp-level int8
 * MMA kernel, KVB_KERNEL_TCGEN05 the TMEM-accumulator tcgen05 kernel wherever
 * it has a variant for the shape (else the warp-level one), KVB_KERNEL_GENERAL
 * the general CUDA-core kernel for every kvb_launch_attention(_ex) call, int8
 * or fp32 KV. For side-by-side measurements and tests; results agree within
 * the path tolerance. kvb_decode_kernel returns the current choice. */
#define KVB_KERNEL_AUTO 0
#define KVB_KERNEL_WARP_MMA 1
#define KVB_KERNEL_TCGEN05 2
#define KVB_KERNEL_GENERAL 3
int kvb_set_decode_kernel(int choice);
int kvb_decode_kernel(void);

/* Event timeline of the tcgen05 partial kernel, in libraries built with the
 * trace flag (python -m kvbridge_b200.build --trace): copies up to `count`
 * SM clock stamps [16 CTAs][16 tiles][18 events] of the latest launches
 * and clears them. Other builds return KVB_EINVAL. */
int kvb_debug_read_tc_trace(unsigned long long* out, size_t count);

/* Per-CTA timeline of the warp-level partial kernels, in libraries built
 * with the trace flag: copies up to `count` stamps [1024 CTAs][20 events]
 * of the latest launches (entry and exit on the global timer in ns, the
 * rest SM clock stamps; events 16-17 are kept from the first launch after
 * the previous read; the event list is in decode_tma.cuh, CtaTraceEvent)
 * and clears them. Other builds return KVB_EINVAL. */
int kvb_debug_read_cta_trace(unsigned long long* out, size_t count);

/* Merge timeline in trace builds: [1024 CTAs][5] global-timer stamps (ns) -
 * entry, dependency wait passed, exit, first loads used, warps folded - of
 * the first merge launch after the previous read, then clears them. Other
 * builds return KVB_EINVAL. */
int kvb_debug_read_merge_trace(unsigned long long* out, size_t count);

/* Decode call that allocates nothing. It has no counterpart in the
 * reference. kvb_launch_attention_ex needs a caller-provided scratch buffer
 * of scratch_elements(shape) floats; callers that cannot call cudaMalloc
 * when they decode - an inference server whose memory pool reserved all of
 * HBM up front for its KV cache, or a host whose decode path must not
 * allocate - use this one instead. It is kvb_launch_attention_ex (same
 * inputs, outputs, partitions and optional fp16 output) with the split-K
 * partials kept in a static device array of KVB_NOALLOC_SCRATCH_FLOATS
 * floats (2 MiB) that every GPU loading the library holds until process
 * exit.
 *   - Limits: the tensor-core geometry only (kvb_attention_b200_supported);
 *     partitions are clamped so rows * q_heads * partitions * (dim + 2)
 *     fits the array; a shape whose single partition does not fit returns
 *     KVB_EINVAL with a message.
 *   - The first call in each CUDA context looks up the array's device
 *     address (cudaGetSymbolAddress); make that first call before any
 *     stream capture.
 *   - It calls no cudaMalloc, cudaFree or other allocating routine.
 *   - All calls share the array: calls that can overlap on the GPU (other
 *     streams) race and must be serialised. No part of the array needs
 *     clearing between calls. */
#define KVB_NOALLOC_SCRATCH_FLOATS 524288
int kvb_launch_attention_noalloc(const kvb_shape* s, const kvb_device_input* in,
                                 unsigned partitions, float* m, float* l, float* n,
                                 void* out_f16, void* stream);

/* Host-side schedule of the split-K kernel, exported for tests: the CTA that
 * owns global stage `stage` when `total` stages are split over `ctas` CTAs. */
uint32_t kvb_schedule_cta_of(uint64_t stage, uint64_t total, uint32_t ctas);

#ifdef __cplusplus
}
#endif

#endif /* KVBRIDGE_C_H */
