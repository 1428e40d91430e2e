#pragma once
// General-geometry split kernel (CUDA cores, fp32 math) for every valid Shape
// the tensor-core kernel does not take: fp32 KV, head dims that are not 64,
// 128 or 256, pages that do not divide 64 tokens, query groups wider than the
// MMA tile, or buffers without 16-byte alignment.
//
// It writes the reference scratch layout with 256-token splits
// (reference src/attention_shared.cu:42-293 computes the same partials):
// one CTA per (row, KV head, split) handles the KV head's query heads in
// chunks of 8. Phase 1: warps take tokens round-robin, lanes stride over the
// head dim and reduce the dots with shuffles. Phase 2: one warp per head does
// the masked softmax of the split. Phase 3: threads own dims and accumulate
// the weighted V.
#include "kvb_device.cuh"

namespace kvb {

struct SimtParams {
  const float* q;
  const int64_t* q_positions;
  const int64_t* k_positions;
  const uint32_t* table;
  const void* k;
  const void* v;
  const float* k_scales;
  const float* v_scales;
  float* scratch;
  uint32_t rows, q_heads, kv_heads, dim, page_tokens, pages, begin, end, splits;
  float scale;
};

constexpr int kSimtThreads = 128;
constexpr int kSimtChunk = 8;  // query heads per pass
constexpr int kSimtSplit = 256;
constexpr uint32_t kInvisible = 0xffffffffu;  // vrow marker; real offsets are < 2^32 - 1

template <bool Q8>
__device__ __forceinline__ float kv_value(const void* base, size_t i) {
  if constexpr (Q8)
    return static_cast<float>(static_cast<const int8_t*>(base)[i]);
  else
    return static_cast<const float*>(base)[i];
}

template <bool Q8>
__global__ void __launch_bounds__(kSimtThreads) decode_simt_kernel(SimtParams p) {
  __shared__ float qs[kSimtChunk][256];
  __shared__ float ws[kSimtChunk][kSimtSplit];
  __shared__ float vsc[kSimtSplit];
  __shared__ uint32_t vrow[kSimtSplit];
  __shared__ float mx[kSimtChunk], den[kSimtChunk];
  grid_dependency_wait();

  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t r = blockIdx.x / p.kv_heads, h = blockIdx.x % p.kv_heads;
  const uint32_t split = blockIdx.y;
  const uint32_t group = p.q_heads / p.kv_heads;
  const uint32_t D = p.dim, P = p.page_tokens;
  const uint32_t start = p.begin + split * kSimtSplit;
  const uint32_t count = start < p.end ? min(uint32_t(kSimtSplit), p.end - start) : 0u;
  const int64_t qp = p.q_positions[r];

  // Token metadata shared by every head chunk.
  for (uint32_t t = tid; t < kSimtSplit; t += kSimtThreads) {
    uint32_t row = 0;
    float vs = 0.f;
    if (t < count && p.k_positions[start + t] <= qp) {
      const uint32_t tok = start + t;
      const uint32_t page = p.table[tok / P];
      if (page < p.pages) {
        const size_t unit = size_t(page) * p.kv_heads + h;
        row = static_cast<uint32_t>(unit * D * P + tok % P);
        vs = Q8 ? p.v_scales[unit * P + tok % P] : 1.f;
        vsc[t] = vs;
        vrow[t] = row;
        continue;
      }
      atomicMax(&g_kvb_status, 4);  // page id outside the pool
    }
    vsc[t] = 0.f;
    vrow[t] = kInvisible;
  }

  for (uint32_t hc = 0; hc < group; hc += kSimtChunk) {
    const uint32_t gh = min(uint32_t(kSimtChunk), group - hc);
    __syncthreads();
    for (uint32_t i = tid; i < gh * D; i += kSimtThreads) {
      const uint32_t hh = i / D, d = i % D;
      qs[hh][d] = p.q[(size_t(r) * p.q_heads + size_t(h) * group + hc + hh) * D + d];
    }
    __syncthreads();

    // Phase 1: scores.
    for (uint32_t t = warp; t < kSimtSplit; t += kSimtThreads / 32) {
      const bool vis = vrow[t] != kInvisible;
      float dot[kSimtChunk];
#pragma unroll
      for (int i = 0; i < kSimtChunk; ++i) dot[i] = 0.f;
      if (vis) {
        const uint32_t tok = start + t;
        const size_t unit = size_t(p.table[tok / P]) * p.kv_heads + h;
        const size_t kidx = (unit * P + tok % P) * D;
        const float ks = Q8 ? p.k_scales[unit * P + tok % P] : 1.f;
        for (uint32_t d = lane; d < D; d += 32) {
          const float kv = kv_value<Q8>(p.k, kidx + d);
#pragma unroll
          for (int i = 0; i < kSimtChunk; ++i)
            if (uint32_t(i) < gh) dot[i] = fmaf(qs[i][d], kv, dot[i]);
        }
#pragma unroll
        for (int i = 0; i < kSimtChunk; ++i) dot[i] = warp_sum(dot[i]) * ks * p.scale;
      }
      if (lane == 0)
#pragma unroll
        for (int i = 0; i < kSimtChunk; ++i)
          if (uint32_t(i) < gh) ws[i][t] = vis ? dot[i] : -INFINITY;
    }
    __syncthreads();

    // Phase 2: softmax of the split per head; ws becomes w * vscale.
    for (uint32_t i = warp; i < gh; i += kSimtThreads / 32) {
      float m = -INFINITY;
      for (uint32_t t = lane; t < kSimtSplit; t += 32) m = fmaxf(m, ws[i][t]);
      m = warp_max(m);
      float sum = 0.f;
      for (uint32_t t = lane; t < kSimtSplit; t += 32) {
        const float w = m == -INFINITY || ws[i][t] == -INFINITY ? 0.f : expf(ws[i][t] - m);
        sum += w;
        ws[i][t] = w == 0.f ? 0.f : w * vsc[t];
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        mx[i] = m;
        den[i] = sum;
      }
    }
    __syncthreads();

    // Phase 3: numerators; threads own dims.
    for (uint32_t d = tid; d < D; d += kSimtThreads) {
      float acc[kSimtChunk];
#pragma unroll
      for (int i = 0; i < kSimtChunk; ++i) acc[i] = 0.f;
      for (uint32_t t = 0; t < count; ++t) {
        if (vrow[t] == kInvisible) continue;
        const float v = kv_value<Q8>(p.v, size_t(vrow[t]) + size_t(d) * P);
#pragma unroll
        for (int i = 0; i < kSimtChunk; ++i)
          if (uint32_t(i) < gh) acc[i] = fmaf(ws[i][t], v, acc[i]);
      }
#pragma unroll
      for (int i = 0; i < kSimtChunk; ++i) {
        if (uint32_t(i) >= gh) break;
        const size_t rh = size_t(r) * p.q_heads + size_t(h) * group + hc + i;
        p.scratch[(rh * p.splits + split) * (D + 2) + 2 + d] = acc[i];
      }
    }
    if (tid < gh) {
      const size_t rh = size_t(r) * p.q_heads + size_t(h) * group + hc + tid;
      p.scratch[(rh * p.splits + split) * (D + 2) + 0] = mx[tid];
      p.scratch[(rh * p.splits + split) * (D + 2) + 1] = den[tid];
    }
  }
}

}  // namespace kvb
