#pragma once
// Paged KV append: quantise new K and V rows and write them into the
// reference's pool layout (include/kvbridge/attention_common.h:11-46):
// K codes at ((page * Hkv + h) * P + s) * D + d, V codes at
// ((page * Hkv + h) * D + d) * P + s, scales at (page * Hkv + h) * P + s.
//
// Quantisation is the symmetric per-(token, kv-head) absmax rule the
// benchmark configurations state for the cache contents (the reference's
// fixtures write codes and scales directly and ship no quantiser):
//   scale = max_d |x_d| / 127            (fp32)
//   code_d = clamp(rint(x_d / scale), -127, 127)   (fp32 division, ties to even)
// with scale = 0 and all codes 0 for an all-zero row.
#include "kvb_device.cuh"

namespace kvb {

constexpr int kStatusBadSlot = 6;  // an append slot at or beyond pages * page_tokens

struct AppendParams {
  const float* k_new;    // [tokens][kv_heads][dim]
  const float* v_new;    // [tokens][kv_heads][dim]
  const int64_t* slots;  // [tokens]: page * page_tokens + s; negative = skip
  int8_t* k;
  int8_t* v;
  float* k_scales;
  float* v_scales;
  uint32_t tokens, kv_heads, dim, page_tokens;
  uint64_t slots_total;  // pages * page_tokens
};

constexpr int kAppendWarps = 8;
constexpr int kAppendMaxK = 8;  // dims per lane: d = lane + 32k, dim <= 256

// One warp per (token, kv head, K or V) row: coalesced loads of the row,
// a warp max of |x|, then the codes (K: one contiguous row; V: one byte per
// dim-major row, stride page_tokens) and the scale.
__global__ void __launch_bounds__(32 * kAppendWarps) append_kv_kernel(AppendParams p) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t row = uint64_t(blockIdx.x) * kAppendWarps + (threadIdx.x >> 5);
  if (row >= uint64_t(p.tokens) * p.kv_heads * 2) return;
  const uint32_t kind = uint32_t(row & 1);  // 0: K, 1: V
  const uint64_t th = row >> 1;             // token * kv_heads + h
  const uint32_t token = uint32_t(th / p.kv_heads), h = uint32_t(th % p.kv_heads);
  const int64_t slot = p.slots[token];
  if (slot < 0) return;
  if (uint64_t(slot) >= p.slots_total) {
    if (lane == 0) atomicMax(&g_kvb_status, kStatusBadSlot);
    return;
  }
  const uint32_t D = p.dim, P = p.page_tokens;
  const uint64_t page = uint64_t(slot) / P, s = uint64_t(slot) % P;
  const float* x = (kind == 0 ? p.k_new : p.v_new) + th * D;
  float vals[kAppendMaxK];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kAppendMaxK; ++i) {
    const uint32_t d = lane + 32u * i;
    vals[i] = d < D ? __ldg(x + d) : 0.f;
    amax = fmaxf(amax, fabsf(vals[i]));
  }
  amax = warp_max(amax);
  const float scale = amax / 127.0f;
  const float div = scale > 0.f ? scale : 1.0f;
  const uint64_t unit = page * p.kv_heads + h;  // (page, kv head)
#pragma unroll
  for (int i = 0; i < kAppendMaxK; ++i) {
    const uint32_t d = lane + 32u * i;
    if (d >= D) break;
    const float c = fminf(fmaxf(rintf(vals[i] / div), -127.f), 127.f);
    const int8_t code = static_cast<int8_t>(static_cast<int>(c));
    if (kind == 0)
      p.k[(unit * P + s) * D + d] = code;
    else
      p.v[(unit * D + d) * P + s] = code;
  }
  if (lane == 0) (kind == 0 ? p.k_scales : p.v_scales)[unit * P + s] = scale;
}

}  // namespace kvb
