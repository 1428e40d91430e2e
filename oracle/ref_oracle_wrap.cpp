// TEST INFRASTRUCTURE - C wrapper around the reference repository's own FP64
// oracle, compiled from the reference's sources where they lie (see
// oracle/Makefile; output goes to oracle/_ref/ only). Used to pin this
// repository's C oracle (oracle/kvb_oracle.c) to the reference bit for bit
// and as the timed CPU baseline of bench.py. Nothing in the product links it.
//
// Calls kvbridge_example::reference() (reference examples/attention_reference.h:
// 53-89) and the reference's host shape layer (src/attention_shape.cpp). For
// multi-threaded runs the call is split into one sub-fixture per query head
// (q_heads = kv_heads = 1, holding that head's KV); reference() treats every
// (row, head) independently, so the results are the same doubles as one
// whole-fixture call.
#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <thread>
#include <vector>

#include "attention_reference.h"
#include "kvbridge/attention_shape.h"

namespace {

struct Handle {
  kvbridge::Shape whole;
  std::vector<kvbridge_example::Fixture> parts;  // one per query head
  std::vector<kvbridge_example::Oracle> results;
};

kvbridge::Shape make_shape(const uint32_t* dims, float scale, int int8) {
  return kvbridge::Shape{dims[0], dims[1], dims[2], dims[3], dims[4],
                         dims[5], dims[6], dims[7], dims[8], scale, int8 != 0};
}

}  // namespace

extern "C" {

// dims = {rows, q_heads, kv_heads, dim, page_tokens, pages, tokens, begin, end}
const char* kvbref_shape_error(const uint32_t* dims, float scale, int int8) {
  return kvbridge::attention_shape_error(make_shape(dims, scale, int8));
}

// Reference sizing helpers; return 0 and write the value, or 1 if the
// reference throws std::invalid_argument.
int kvbref_sizes(const uint32_t* dims, float scale, int int8, uint64_t* out4) {
  try {
    const auto s = make_shape(dims, scale, int8);
    out4[0] = kvbridge::split_count(s);
    out4[1] = kvbridge::scratch_elements(s);
    out4[2] = kvbridge::output_scalar_elements(s);
    out4[3] = kvbridge::output_numerator_elements(s);
    return 0;
  } catch (const std::invalid_argument&) {
    return 1;
  }
}

int kvbref_mma_supported(const uint32_t* dims, float scale, int int8) {
  return kvbridge::attention_mma_supported(make_shape(dims, scale, int8)) ? 1 : 0;
}

// Copies the inputs into per-KV-head reference fixtures. K/V are int8 in the
// reference layouts. Returns nullptr on invalid metadata.
void* kvbref_prepare(const uint32_t* dims, float scale, const float* q, const int64_t* qpos,
                     const int64_t* kpos, const uint32_t* table, const int8_t* k, const int8_t* v,
                     const float* ks, const float* vs) {
  const kvbridge::Shape s = make_shape(dims, scale, 1);
  if (!kvbridge::attention_shape_valid(s)) return nullptr;
  auto* h = new Handle;
  h->whole = s;
  const uint32_t group = s.q_heads / s.kv_heads, P = s.page_tokens, D = s.dim;
  for (uint32_t head = 0; head < s.q_heads; ++head) {
    const uint32_t kv = head / group;
    kvbridge_example::Fixture f;
    f.shape = s;
    f.shape.q_heads = 1;
    f.shape.kv_heads = 1;
    f.q.resize(size_t(s.rows) * D);
    for (uint32_t r = 0; r < s.rows; ++r)
      std::memcpy(&f.q[size_t(r) * D], q + (size_t(r) * s.q_heads + head) * D, D * sizeof(float));
    f.qpos.assign(qpos, qpos + s.rows);
    f.kpos.assign(kpos, kpos + s.tokens);
    f.table.assign(table, table + s.pages);
    const size_t slots = size_t(s.pages) * P;
    f.k.resize(slots * D);
    f.v.resize(slots * D);
    f.ks.resize(slots);
    f.vs.resize(slots);
    for (uint32_t p = 0; p < s.pages; ++p) {
      const size_t unit = size_t(p) * s.kv_heads + kv;
      std::memcpy(&f.k[size_t(p) * P * D], k + unit * P * D, size_t(P) * D);
      std::memcpy(&f.v[size_t(p) * D * P], v + unit * D * P, size_t(D) * P);
      std::memcpy(&f.ks[size_t(p) * P], ks + unit * P, P * sizeof(float));
      std::memcpy(&f.vs[size_t(p) * P], vs + unit * P, P * sizeof(float));
    }
    h->parts.push_back(std::move(f));
  }
  h->results.resize(h->parts.size());
  return h;
}

// Runs reference() over every query head with up to `threads` threads and
// returns the wall time of the calls in *seconds.
int kvbref_run(void* handle, int threads, double* seconds) {
  auto* h = static_cast<Handle*>(handle);
  if (!h) return 1;
  const size_t n = h->parts.size();
  if (threads < 1) threads = 1;
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<std::thread> pool;
  for (int w = 0; w < threads; ++w)
    pool.emplace_back([h, n, w, threads] {
      for (size_t i = w; i < n; i += threads) h->results[i] = kvbridge_example::reference(h->parts[i]);
    });
  for (auto& t : pool) t.join();
  const auto t1 = std::chrono::steady_clock::now();
  if (seconds) *seconds = std::chrono::duration<double>(t1 - t0).count();
  return 0;
}

// normalized: [rows][q_heads][dim]; visible: [rows][q_heads].
int kvbref_result(void* handle, double* normalized, uint8_t* visible) {
  auto* h = static_cast<Handle*>(handle);
  if (!h) return 1;
  const auto& s = h->whole;
  const uint32_t D = s.dim;
  for (uint32_t head = 0; head < s.q_heads; ++head) {
    const auto& o = h->results[head];
    if (o.normalized.empty()) return 2;
    for (uint32_t r = 0; r < s.rows; ++r) {
      const size_t dst = size_t(r) * s.q_heads + head;
      std::memcpy(normalized + dst * D, &o.normalized[size_t(r) * D], D * sizeof(double));
      visible[dst] = o.visible[r] ? 1 : 0;
    }
  }
  return 0;
}

void kvbref_free(void* handle) { delete static_cast<Handle*>(handle); }

}  // extern "C"
