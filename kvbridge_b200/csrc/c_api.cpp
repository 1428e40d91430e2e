// extern "C" boundary of kvbridge-b200 (include/kvbridge_c.h). Each function
// converts the C structs to the kvbridge:: types, calls the C++ entry point
// and turns its exceptions into status codes plus a thread-local message; no
// exception crosses this boundary.
#include <cstddef>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>

#include "kvbridge/attention_b200.h"
#include "kvbridge/attention_common.h"
#include "kvbridge_c.h"
#include "kvb_schedule.h"

namespace kvbridge::detail {
cudaError_t read_tc_trace(unsigned long long* out, size_t count, bool* available) noexcept;
cudaError_t read_cta_trace(unsigned long long* out, size_t count, bool* available) noexcept;
cudaError_t read_merge_trace(unsigned long long* out, size_t count, bool* available) noexcept;
void launch_attention_noalloc(const Shape&, const DeviceInput&, unsigned partitions, float* m,
                              float* l, float* n, void* out_f16, cudaStream_t);
}  // namespace kvbridge::detail

namespace {

thread_local std::string g_last_error;

static_assert(sizeof(kvb_shape) == sizeof(kvbridge::Shape), "kvb_shape must mirror Shape");
static_assert(offsetof(kvb_shape, scale) == offsetof(kvbridge::Shape, scale), "Shape layout");
static_assert(offsetof(kvb_shape, int8) == offsetof(kvbridge::Shape, int8), "Shape layout");
static_assert(sizeof(kvb_device_input) == sizeof(kvbridge::DeviceInput), "DeviceInput layout");

kvbridge::Shape to_shape(const kvb_shape* s) {
  if (s == nullptr) throw std::invalid_argument("shape pointer is null");
  kvbridge::Shape out;
  out.rows = s->rows;
  out.q_heads = s->q_heads;
  out.kv_heads = s->kv_heads;
  out.dim = s->dim;
  out.page_tokens = s->page_tokens;
  out.pages = s->pages;
  out.tokens = s->tokens;
  out.begin = s->begin;
  out.end = s->end;
  out.scale = s->scale;
  out.int8 = s->int8;
  return out;
}

kvbridge::DeviceInput to_input(const kvb_device_input* in) {
  if (in == nullptr) throw std::invalid_argument("input pointer is null");
  return kvbridge::DeviceInput{in->q,       in->q_positions, in->k_positions, in->page_table,
                               in->k,       in->v,           in->k_scales,    in->v_scales};
}

kvbridge::BatchShape to_batch_shape(const kvb_batch_shape* s) {
  if (s == nullptr) throw std::invalid_argument("shape pointer is null");
  return kvbridge::BatchShape{s->batch,       s->q_heads,      s->kv_heads,
                              s->dim,         s->page_tokens,  s->pages,
                              s->table_stride, s->max_tokens,  s->scale};
}

kvbridge::BatchInput to_batch_input(const kvb_batch_input* in) {
  if (in == nullptr) throw std::invalid_argument("input pointer is null");
  return kvbridge::BatchInput{in->q, in->seq_lens, in->block_table, in->k,
                              in->v, in->k_scales, in->v_scales};
}

template <class F>
int guarded(F&& body) {
  try {
    body();
    g_last_error.clear();
    return KVB_OK;
  } catch (const std::invalid_argument& e) {
    g_last_error = e.what();
    return KVB_EINVAL;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return KVB_ECUDA;
  } catch (...) {
    g_last_error = "unknown error";
    return KVB_ECUDA;
  }
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

extern "C" {

const char* kvb_last_error(void) { return g_last_error.c_str(); }

const char* kvb_attention_shape_error(const kvb_shape* s) {
  if (s == nullptr) return "shape pointer is null";
  return kvbridge::attention_shape_error(to_shape(s));
}

bool kvb_attention_shape_valid(const kvb_shape* s) {
  return s != nullptr && kvbridge::attention_shape_valid(to_shape(s));
}

int kvb_validate_shape(const kvb_shape* s) {
  return guarded([&] { kvbridge::validate_shape(to_shape(s)); });
}

int kvb_split_count(const kvb_shape* s, unsigned* splits) {
  return guarded([&] {
    const unsigned v = kvbridge::split_count(to_shape(s));
    if (splits == nullptr) throw std::invalid_argument("output pointer is null");
    *splits = v;
  });
}

int kvb_scratch_elements(const kvb_shape* s, size_t* elements) {
  return guarded([&] {
    const size_t v = kvbridge::scratch_elements(to_shape(s));
    if (elements == nullptr) throw std::invalid_argument("output pointer is null");
    *elements = v;
  });
}

int kvb_output_scalar_elements(const kvb_shape* s, size_t* elements) {
  return guarded([&] {
    const size_t v = kvbridge::output_scalar_elements(to_shape(s));
    if (elements == nullptr) throw std::invalid_argument("output pointer is null");
    *elements = v;
  });
}

int kvb_output_numerator_elements(const kvb_shape* s, size_t* elements) {
  return guarded([&] {
    const size_t v = kvbridge::output_numerator_elements(to_shape(s));
    if (elements == nullptr) throw std::invalid_argument("output pointer is null");
    *elements = v;
  });
}

bool kvb_attention_mma_supported(const kvb_shape* s) {
  return s != nullptr && kvbridge::attention_mma_supported(to_shape(s));
}

int kvb_preload_attention_kernels(void) { return int(kvbridge::preload_attention_kernels()); }
int kvb_preload_attention_reference_kernels(void) {
  return int(kvbridge::preload_attention_reference_kernels());
}
int kvb_preload_attention_mma_kernels(void) {
  return int(kvbridge::preload_attention_mma_kernels());
}

int kvb_launch_attention(const kvb_shape* s, const kvb_device_input* in, float* scratch, float* m,
                         float* l, float* n, void* stream) {
  return guarded([&] {
    kvbridge::launch_attention(to_shape(s), to_input(in), scratch, m, l, n, as_stream(stream));
  });
}

int kvb_launch_attention_mma(const kvb_shape* s, const kvb_device_input* in, float* scratch,
                             float* m, float* l, float* n, void* stream) {
  return guarded([&] {
    kvbridge::launch_attention_mma(to_shape(s), to_input(in), scratch, m, l, n,
                                   as_stream(stream));
  });
}

int kvb_merge_attention(const kvb_shape* s, const float* scratch, unsigned splits, float* m,
                        float* l, float* n, void* stream) {
  return guarded([&] {
    kvbridge::merge_attention(to_shape(s), scratch, splits, m, l, n, as_stream(stream));
  });
}

bool kvb_attention_b200_supported(const kvb_shape* s, const kvb_device_input* in) {
  if (s == nullptr || in == nullptr) return false;
  return kvbridge::attention_b200_supported(to_shape(s), to_input(in));
}

int kvb_attention_partitions(const kvb_shape* s, unsigned requested, unsigned* partitions) {
  return guarded([&] {
    const unsigned v = kvbridge::attention_partitions(to_shape(s), requested);
    if (partitions == nullptr) throw std::invalid_argument("output pointer is null");
    *partitions = v;
  });
}

int kvb_launch_attention_ex(const kvb_shape* s, const kvb_device_input* in, unsigned partitions,
                            void* out_f16, float* scratch, float* m, float* l, float* n,
                            void* stream) {
  return guarded([&] {
    kvbridge::launch_attention_ex(to_shape(s), to_input(in),
                                  kvbridge::LaunchOptions{partitions, out_f16}, scratch, m, l, n,
                                  as_stream(stream));
  });
}

int kvb_launch_attention_ex2(const kvb_shape* s, const kvb_device_input* in, unsigned partitions,
                             void* out_f16, void* out_bf16, float* scratch, float* m, float* l,
                             float* n, void* stream) {
  return guarded([&] {
    kvbridge::LaunchOptions opt{partitions, out_f16};
    opt.out_bf16 = out_bf16;
    kvbridge::launch_attention_ex(to_shape(s), to_input(in), opt, scratch, m, l, n,
                                  as_stream(stream));
  });
}

int kvb_launch_attention_partials(const kvb_shape* s, const kvb_device_input* in,
                                  unsigned partitions, float* scratch, unsigned* partitions_used,
                                  void* stream) {
  return guarded([&] {
    const unsigned used = kvbridge::launch_attention_partials(to_shape(s), to_input(in), partitions,
                                                              scratch, as_stream(stream));
    if (partitions_used != nullptr) *partitions_used = used;
  });
}

int kvb_merge_attention_ex(const kvb_shape* s, const float* scratch, unsigned partitions, float* m,
                           float* l, float* n, void* out_f16, void* stream) {
  return guarded([&] {
    kvbridge::merge_attention_ex(to_shape(s), scratch, partitions, m, l, n, out_f16,
                                 as_stream(stream));
  });
}

int kvb_merge_attention_ex2(const kvb_shape* s, const float* scratch, unsigned partitions,
                            float* m, float* l, float* n, void* out_f16, void* out_bf16,
                            void* stream) {
  return guarded([&] {
    kvbridge::merge_attention_ex(to_shape(s), scratch, partitions, m, l, n, out_f16, out_bf16,
                                 as_stream(stream));
  });
}

const char* kvb_batch_shape_error(const kvb_batch_shape* s) {
  if (s == nullptr) return "shape pointer is null";
  return kvbridge::batch_shape_error(to_batch_shape(s));
}

int kvb_batch_workspace_bytes(const kvb_batch_shape* s, size_t* bytes) {
  return guarded([&] {
    const size_t v = kvbridge::batch_workspace_bytes(to_batch_shape(s));
    if (bytes == nullptr) throw std::invalid_argument("output pointer is null");
    *bytes = v;
  });
}

int kvb_launch_attention_batched(const kvb_batch_shape* s, const kvb_batch_input* in,
                                 void* workspace, size_t workspace_bytes, float* m, float* l,
                                 float* n, void* out_f16, void* stream) {
  return guarded([&] {
    kvbridge::launch_attention_batched(to_batch_shape(s), to_batch_input(in), workspace,
                                       workspace_bytes, m, l, n, out_f16, as_stream(stream));
  });
}

int kvb_launch_attention_batched2(const kvb_batch_shape* s, const kvb_batch_input* in,
                                  void* workspace, size_t workspace_bytes, float* m, float* l,
                                  float* n, void* out_f16, void* out_bf16, void* stream) {
  return guarded([&] {
    kvbridge::launch_attention_batched(to_batch_shape(s), to_batch_input(in), workspace,
                                       workspace_bytes, m, l, n, out_f16, out_bf16,
                                       as_stream(stream));
  });
}

const char* kvb_append_shape_error(const kvb_append_shape* s) {
  if (s == nullptr) return "shape pointer is null";
  return kvbridge::append_shape_error(
      kvbridge::AppendShape{s->tokens, s->kv_heads, s->dim, s->page_tokens, s->pages});
}

int kvb_append_kv(const kvb_append_shape* s, const kvb_append_input* in, void* stream) {
  return guarded([&] {
    if (s == nullptr) throw std::invalid_argument("shape pointer is null");
    if (in == nullptr) throw std::invalid_argument("input pointer is null");
    kvbridge::append_kv(
        kvbridge::AppendShape{s->tokens, s->kv_heads, s->dim, s->page_tokens, s->pages},
        kvbridge::AppendInput{in->k_new, in->v_new, in->slots, in->k, in->v, in->k_scales,
                              in->v_scales},
        as_stream(stream));
  });
}

int kvb_merge_attention_shards(unsigned shards, unsigned row_heads, unsigned dim,
                               const float* m_parts, const float* l_parts, const float* n_parts,
                               float* m, float* l, float* n, void* out_f16, void* stream) {
  return guarded([&] {
    kvbridge::merge_attention_shards(shards, row_heads, dim, m_parts, l_parts, n_parts, m, l, n,
                                     out_f16, as_stream(stream));
  });
}

int kvb_merge_attention_shards_ex(unsigned shards, unsigned row_heads, unsigned dim,
                                  const float* m_parts, const float* l_parts,
                                  const float* n_parts, size_t shard_stride, float* m, float* l,
                                  float* n, void* out_f16, void* out_bf16, void* stream) {
  return guarded([&] {
    kvbridge::merge_attention_shards_ex(shards, row_heads, dim, m_parts, l_parts, n_parts,
                                        shard_stride, m, l, n, out_f16, out_bf16,
                                        as_stream(stream));
  });
}

size_t kvb_peer_buffer_bytes(unsigned row_heads, unsigned dim) {
  try {
    return kvbridge::peer_buffer_bytes(row_heads, dim);
  } catch (...) {
    return 0;
  }
}

float* kvb_peer_slot(void* buffer, unsigned epoch, unsigned row_heads, unsigned dim) {
  return buffer == nullptr ? nullptr : kvbridge::peer_slot(buffer, epoch, row_heads, dim);
}

int kvb_peer_buffer_alloc(size_t bytes, void** buffer, unsigned char* handle64) {
  return guarded([&] { kvbridge::peer_buffer_alloc(bytes, buffer, handle64); });
}

int kvb_peer_buffer_open(const unsigned char* handle64, void** peer_buffer) {
  return guarded([&] { kvbridge::peer_buffer_open(handle64, peer_buffer); });
}

int kvb_peer_buffer_close(void* peer_buffer) {
  return guarded([&] { kvbridge::peer_buffer_close(peer_buffer); });
}

int kvb_peer_buffer_free(void* buffer) {
  return guarded([&] { kvbridge::peer_buffer_free(buffer); });
}

int kvb_merge_attention_peers(const void* const* buffers, unsigned world, unsigned rank, unsigned epoch,
                              unsigned row_heads, unsigned dim, float* m, float* l, float* n, void* out_f16,
                              void* out_bf16, void* stream) {
  return guarded([&] {
    kvbridge::merge_attention_peers(buffers, world, rank, epoch, row_heads, dim, m, l, n, out_f16, out_bf16,
                                    as_stream(stream));
  });
}

int kvb_debug_copy_to_device(void* dst, const void* src, size_t bytes) {
  return guarded([&] {
    if (dst == nullptr || src == nullptr) throw std::invalid_argument("null pointer");
    const cudaError_t code = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
    if (code != cudaSuccess) throw std::runtime_error(std::string("copy: ") + cudaGetErrorString(code));
  });
}

int kvb_read_device_status(int* status) { return int(kvbridge::read_device_status(status)); }

void kvb_set_wait_limit_ns(unsigned long long ns) { kvbridge::set_wait_limit_ns(ns); }

unsigned long long kvb_wait_limit_ns(void) { return kvbridge::wait_limit_ns(); }

int kvb_debug_fail_launch(unsigned nth, int cuda_error) {
  kvbridge::detail::fail_launch(nth, static_cast<cudaError_t>(cuda_error));
  return KVB_OK;
}

int kvb_debug_read_tc_trace(unsigned long long* out, size_t count) {
  return guarded([&] {
    if (out == nullptr) throw std::invalid_argument("output pointer is null");
    bool available = false;
    const cudaError_t code = kvbridge::detail::read_tc_trace(out, count, &available);
    if (!available)
      throw std::invalid_argument("this library was built without the tcgen05 event trace (KVB_TC_TRACE)");
    if (code != cudaSuccess) throw std::runtime_error(std::string("trace read: ") + cudaGetErrorString(code));
  });
}

int kvb_debug_read_cta_trace(unsigned long long* out, size_t count) {
  return guarded([&] {
    if (out == nullptr) throw std::invalid_argument("output pointer is null");
    bool available = false;
    const cudaError_t code = kvbridge::detail::read_cta_trace(out, count, &available);
    if (!available)
      throw std::invalid_argument("this library was built without the event trace (KVB_TC_TRACE)");
    if (code != cudaSuccess) throw std::runtime_error(std::string("trace read: ") + cudaGetErrorString(code));
  });
}

int kvb_debug_read_merge_trace(unsigned long long* out, size_t count) {
  return guarded([&] {
    if (out == nullptr) throw std::invalid_argument("output pointer is null");
    bool available = false;
    const cudaError_t code = kvbridge::detail::read_merge_trace(out, count, &available);
    if (!available)
      throw std::invalid_argument("this library was built without the event trace (KVB_TC_TRACE)");
    if (code != cudaSuccess) throw std::runtime_error(std::string("trace read: ") + cudaGetErrorString(code));
  });
}

int kvb_set_decode_kernel(int choice) {
  kvbridge::detail::set_decode_kernel(choice);
  return KVB_OK;
}

int kvb_decode_kernel(void) { return kvbridge::detail::decode_kernel(); }

int kvb_debug_skip_stage(unsigned stage) {
  kvbridge::detail::skip_stage(stage);
  return KVB_OK;
}

int kvb_read_wait_failure(long long* record6) { return int(kvbridge::read_wait_failure(record6)); }

int kvb_launch_attention_noalloc(const kvb_shape* s, const kvb_device_input* in,
                                 unsigned partitions, float* m, float* l, float* n,
                                 void* out_f16, void* stream) {
  return guarded([&] {
    kvbridge::detail::launch_attention_noalloc(to_shape(s), to_input(in), partitions, m, l, n,
                                               out_f16, as_stream(stream));
  });
}

uint32_t kvb_schedule_cta_of(uint64_t stage, uint64_t total, uint32_t ctas) {
  if (total == 0 || ctas == 0 || stage >= total) return 0;
  return kvb::cta_of_stage(stage, total, ctas);
}

}  // extern "C"
