#pragma once
// Split-K partial kernel for paged fp32 KV (Shape::int8 == false) on sm_100a.
//
// Same partial as the int8 kernels and as reference
// src/attention_shared.cu:42-209 with Q8 = false: for every piece of the
// split-K schedule (kvb_schedule.h), scores s = scale * q.k over the
// piece's visible tokens, m = max s, l = sum exp(s - m),
// n = sum exp(s - m) * v, written as one (m, l, n[dim]) partial per query
// column into the reference scratch layout.
//
// fp32 KV moves 8 * dim bytes per (token, KV head) for 2 * columns * dim
// multiply-adds, ~2 flop/B at one query row of a 32/8-head model: far below
// the CUDA cores' rate, so the kernel is built to keep HBM streaming.
//  * Data movement: a producer warp looks the pages of each 64-token stage
//    up in the page table (two stages ahead) and issues one bulk
//    asynchronous copy per (page, K | V) into a STAGES-deep shared-memory
//    ring guarded by mbarriers (K: the stage's token rows back to back; V:
//    each page's dim x page_tokens block, 16-token pages at a pitch of one
//    block + 64 bytes so the lanes of a PV read hit distinct banks).
//  * Math (8 consumer warps; one CTA of 4 query columns per SM): per stage,
//    QK -- eight lanes per token, lane j holding dims 32 i + 4 j .. + 3 of
//    the 4 columns' queries in registers; the 8-lane dot sums are reduced
//    by a transposed butterfly (4 shuffles for 4 columns) that leaves each
//    lane pair one column's score -- a CTA barrier, the stage max per column
//    and P = exp(s - m) (one value a thread), a second barrier, then PV with
//    each warp owning dim / 8 dims: lane (quad, dim group) reads 16-byte
//    runs of 4 tokens of a V row and the matching P, and accumulates
//    dims x 4 columns. Every thread runs the same online-softmax update,
//    so no state is exchanged except through the two barriers.
//  * At the end: shuffle sums over the token lanes, a fixed-order sum of
//    the warps' l (bitwise reproducible), one partial per column.
// Tokens of pages that were not copied (outside the piece, or a page id
// outside the pool, status 4) are never read: their scores are -inf and
// their V quads are skipped.
#include "decode_tma.cuh"

namespace kvb {

constexpr int kF32ConsumerWarps = 8;
constexpr int kF32ProducerWarp = kF32ConsumerWarps;
constexpr int kF32Threads = 32 * (kF32ConsumerWarps + 1);
constexpr int kF32Cols = 4;  // query columns per CTA
// Floats per column row of the P buffer: 64 tokens + 4, so that the four
// columns' stores of one token land in different banks (16-byte aligned rows).
constexpr int kF32PPitch = kStageTokens + 4;

// a[i] for a lane-dependent i without indexing a register array (which
// would put the array in local memory).
template <typename T>
__device__ __forceinline__ T pick_col(const T (&a)[kF32Cols], uint32_t i) {
  T r = a[0];
#pragma unroll
  for (int c = 1; c < kF32Cols; ++c) r = i == uint32_t(c) ? a[c] : r;
  return r;
}

template <int D>
struct F32Smem {
  // V block pitch of a page inside a stage (bytes).
  static __host__ __device__ constexpr uint32_t v_pitch(uint32_t page_tokens) {
    return D * page_tokens * 4 + (page_tokens == 16 ? 64u : 0u);
  }
  static constexpr uint32_t kK = 0;                                    // K rows, 64 x D fp32
  static constexpr uint32_t kV = kStageTokens * D * 4;                 // V blocks
  static constexpr uint32_t kStage = kV + kStageTokens * D * 4 + 256;  // 16-token pages: 4 x 64 B pad
};

template <int D, int STAGES>
struct F32Layout {
  static constexpr uint32_t kRing = STAGES * F32Smem<D>::kStage;
  static constexpr uint32_t kOffP = kRing;                                 // P[col][kF32PPitch]
  static constexpr uint32_t kOffWmax = kOffP + kF32Cols * kF32PPitch * 4;  // [warp][col]
  static constexpr uint32_t kOffLw = kOffWmax + kF32ConsumerWarps * kF32Cols * 4;
  static constexpr uint32_t kOffOk = kOffLw + kF32ConsumerWarps * kF32Cols * 4;  // [slot] page mask
  static constexpr uint32_t kOffBar = (kOffOk + 4 * STAGES + 7) / 8 * 8;
  static constexpr uint32_t kOffAbort = kOffBar + 2 * STAGES * 8;
  static constexpr uint32_t kBytes = kOffAbort + 16;
};

// Producer: one lane per (page of the stage, K | V) copy.
template <int D, int STAGES>
__device__ void produce_f32(const DecodeParams& p, const Piece& pc, uint8_t* ring, uint32_t* stage_ok,
                            uint64_t* full, uint64_t* empty, volatile int* abort_flag) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t policy = l2_evict_first_policy();
  const uint32_t P = p.page_tokens;
  const uint32_t pps = kStageTokens >> p.log2_page;  // pages per stage: 1, 2 or 4
  const uint32_t page_bytes = P * D * 4;             // of K, and of V
  const uint32_t vpitch = F32Smem<D>::v_pitch(P);
  const uint32_t k_page = lane >> 1, is_v = lane & 1;
  const bool copier = k_page < pps;
  const float* kf = reinterpret_cast<const float*>(p.k);
  const float* vf = reinterpret_cast<const float*>(p.v);
  grid_dependency_wait();
  const uint32_t first_stage = pc.lo / kStageTokens;
  const uint32_t page_lo = max(pc.lo, (first_stage + pc.j0) * kStageTokens) >> p.log2_page;
  const uint32_t page_hi = (min(pc.hi, (first_stage + pc.j1) * kStageTokens) - 1) >> p.log2_page;
  // This lane's logical page of stage j, if the piece reads it.
  auto lane_page = [&](uint32_t j, uint32_t& pg) {
    pg = (first_stage + j) * pps + k_page;
    return copier && j < pc.j1 && pg >= page_lo && pg <= page_hi;
  };
  // Table entries two stages ahead.
  uint32_t pg, t[3];
  bool in[3];
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    in[u] = lane_page(pc.j0 + u, pg);
    t[u] = in[u] ? __ldg(p.table + pg) : 0u;
  }
  uint32_t g = 0;
  bool failed = false;
  for (uint32_t j = pc.j0; j < pc.j1; ++j) {
    const uint32_t phys = t[0];
    const bool mine = in[0];
    const bool ok = mine && phys < p.pages;
    t[0] = t[1];
    in[0] = in[1];
    t[1] = t[2];
    in[1] = in[2];
    in[2] = lane_page(j + 3, pg);
    t[2] = in[2] ? __ldg(p.table + pg) : 0u;
    if (__ballot_sync(0xffffffffu, mine && !ok) != 0u && lane == 0) atomicMax(&g_kvb_status, kStatusBadPage);
    const uint32_t okk = __ballot_sync(0xffffffffu, ok && !is_v);  // bit 2k: page k copied
    uint32_t okpages = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) okpages |= ((okk >> (2 * k)) & 1u) << k;
    const uint32_t slot = g % STAGES;
    if (mbar_wait_bounded(&empty[slot], ((g / STAGES) & 1u) ^ 1u, abort_flag, kStatusEmptyWaitTimeout,
                          int(g), p.wait_limit_ns) != kWaitOk) {
      failed = true;
      break;
    }
    if (lane == 0) {
      stage_ok[slot] = okpages;
      // The page mask is written before the arrive (release); the consumers
      // read it after their wait on the same phase (acquire).
      mbar_arrive_expect_tx(&full[slot], 2u * __popc(okpages) * page_bytes);
    }
    __syncwarp();
    if (ok) {
      uint8_t* st = ring + size_t(slot) * F32Smem<D>::kStage;
      const size_t unit = size_t(phys) * p.kv_heads + pc.h;  // (page, KV head)
      if (is_v)
        bulk_copy_g2s(st + F32Smem<D>::kV + k_page * vpitch, vf + unit * D * P, page_bytes, &full[slot],
                      policy);
      else
        bulk_copy_g2s(st + F32Smem<D>::kK + k_page * page_bytes, kf + unit * P * D, page_bytes, &full[slot],
                      policy);
    }
    ++g;
  }
  if (!failed) mark_empty_splits<D>(p, pc);
  drain_copies<STAGES>(full, g, p.wait_limit_ns);
}

template <int D, int STAGES>
__global__ void __launch_bounds__(kF32Threads, 1) decode_partial_f32_kernel(DecodeParams p) {
  using L = F32Layout<D, STAGES>;
  constexpr int kQv = D / 32;                        // float4 runs of a lane's query dims
  constexpr int kDpl = D / (kF32ConsumerWarps * 4);  // PV dims per lane
  static_assert(kDpl >= 2 && kDpl % 2 == 0 && D % (kF32ConsumerWarps * 4) == 0, "head dim");
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  float* Ps = reinterpret_cast<float*>(smem + L::kOffP);
  float* Wmax = reinterpret_cast<float*>(smem + L::kOffWmax);
  float* Lw = reinterpret_cast<float*>(smem + L::kOffLw);
  uint32_t* stage_ok = reinterpret_cast<uint32_t*>(smem + L::kOffOk);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* empty = full + STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kF32ConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const Piece pc = single_piece(p, blockIdx.x);
  if (warp == kF32ProducerWarp) {
    produce_f32<D, STAGES>(p, pc, ring, stage_ok, full, empty, abort_flag);
    return;
  }
  grid_dependency_wait();

  const uint32_t P = p.page_tokens;
  const uint32_t vpitch_f = F32Smem<D>::v_pitch(P) / 4;  // floats
  const uint32_t first_stage = pc.lo / kStageTokens;
  const uint32_t sub = lane & 7;  // QK: the lane's dims within a token
  const uint32_t tq = lane & 7;   // PV: the lane's token quads (tq, tq + 8)
  const uint32_t dg = lane >> 3;  // PV: the lane's dim group
  // The column whose score this lane keeps after the transposed reduce.
  const uint32_t my_col = ((sub >> 2) & 1u) * 2u + ((sub >> 1) & 1u);

  // Query columns col0 .. col0 + 3 of the piece's KV head, pre-scaled by
  // scale * log2(e) (the softmax runs in base 2; m is written back in
  // natural units).
  float4 qv[kF32Cols][kQv];
  int64_t qpos[kF32Cols];
  bool cvalid[kF32Cols];
  const float qscale = p.score_scale * kLog2e;
#pragma unroll
  for (int c = 0; c < kF32Cols; ++c) {
    const uint32_t col = pc.col0 + c;
    cvalid[c] = col < p.qr;
    const uint32_t r = cvalid[c] ? col / p.group : 0u, gq = cvalid[c] ? col % p.group : 0u;
    const float* qrow = p.q + (size_t(r) * p.q_heads + size_t(pc.h) * p.group + gq) * D;
#pragma unroll
    for (int i = 0; i < kQv; ++i) {
      float4 f = cvalid[c] ? __ldg(reinterpret_cast<const float4*>(qrow + 32 * i + 4 * sub))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      f.x *= qscale;
      f.y *= qscale;
      f.z *= qscale;
      f.w *= qscale;
      qv[c][i] = f;
    }
    qpos[c] = cvalid[c] ? __ldg(p.q_positions + r) : INT64_MIN;
  }
  // Every token of the piece is visible to every valid column when its
  // last token is (k_positions is nondecreasing).
  const uint32_t last = min(pc.hi, (first_stage + pc.j1) * kStageTokens) - 1;
  int64_t qmin = INT64_MAX;
#pragma unroll
  for (int c = 0; c < kF32Cols; ++c)
    if (cvalid[c]) qmin = min(qmin, qpos[c]);
  const bool all_visible = __ldg(p.k_positions + last) <= qmin;
  const int64_t my_qpos = pick_col(qpos, my_col);
  const bool my_valid = pick_col(cvalid, my_col);

  float m_run[kF32Cols], acc[kDpl][kF32Cols], lpart = 0.f;
#pragma unroll
  for (int c = 0; c < kF32Cols; ++c) {
    m_run[c] = -INFINITY;
#pragma unroll
    for (int dd = 0; dd < kDpl; ++dd) acc[dd][c] = 0.f;
  }
  const uint32_t dbase = warp * (D / kF32ConsumerWarps) + dg * kDpl;
  const uint32_t all_pages = (1u << (kStageTokens >> p.log2_page)) - 1u;

  for (uint32_t j = pc.j0, g = 0; j < pc.j1; ++j, ++g) {
    const uint32_t slot = g % STAGES;
    mbar_wait_bounded(&full[slot], (g / STAGES) & 1u, abort_flag, kStatusFullWaitTimeout, int(g),
                      p.wait_limit_ns);
    const uint8_t* st = ring + size_t(slot) * F32Smem<D>::kStage;
    const float* Ks = reinterpret_cast<const float*>(st + F32Smem<D>::kK);
    const float* Vs = reinterpret_cast<const float*>(st + F32Smem<D>::kV);
    const uint32_t okp = stage_ok[slot];
    const uint32_t tb = (first_stage + j) * kStageTokens;
    const bool full_stage = all_visible && okp == all_pages && tb >= pc.lo && tb + kStageTokens <= pc.hi;

    // ---- QK: tokens 8 warp + 4 r + lane / 8.
    float xs[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint32_t tt = 8 * warp + 4 * r + (lane >> 3);
      const float* krow = Ks + tt * D + 4 * sub;
      float4 kk[kQv];
#pragma unroll
      for (int i = 0; i < kQv; ++i) kk[i] = *reinterpret_cast<const float4*>(krow + 32 * i);
      float dot[kF32Cols];
#pragma unroll
      for (int c = 0; c < kF32Cols; ++c) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < kQv; ++i) {
          a = fmaf(qv[c][i].x, kk[i].x, a);
          a = fmaf(qv[c][i].y, kk[i].y, a);
          a = fmaf(qv[c][i].z, kk[i].z, a);
          a = fmaf(qv[c][i].w, kk[i].w, a);
        }
        dot[c] = a;
      }
      // Transposed butterfly over the token's 8 lanes: keep two columns,
      // then one, then finish the sum (lanes sub and sub ^ 1 agree).
      const bool b2 = (sub & 4u) != 0u, b1 = (sub & 2u) != 0u;
      const float keep0 = b2 ? dot[2] : dot[0], keep1 = b2 ? dot[3] : dot[1];
      const float send0 = b2 ? dot[0] : dot[2], send1 = b2 ? dot[1] : dot[3];
      const float a0 = keep0 + __shfl_xor_sync(0xffffffffu, send0, 4);
      const float a1 = keep1 + __shfl_xor_sync(0xffffffffu, send1, 4);
      float x = (b1 ? a1 : a0) + __shfl_xor_sync(0xffffffffu, b1 ? a0 : a1, 2);
      x += __shfl_xor_sync(0xffffffffu, x, 1);
      bool vis = my_valid;
      if (!full_stage) {
        const uint32_t t = tb + tt;
        vis = vis && t >= pc.lo && t < pc.hi && ((okp >> (tt >> p.log2_page)) & 1u);
        if (vis && !all_visible) vis = __ldg(p.k_positions + t) <= my_qpos;
      }
      xs[r] = vis ? x : -INFINITY;
    }
    float wm = fmaxf(xs[0], xs[1]);
    wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, 8));
    wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, 16));
    if (lane < 8 && (lane & 1u) == 0u) Wmax[warp * kF32Cols + my_col] = wm;
    named_barrier(1, 32 * kF32ConsumerWarps);

    // ---- stage max, rescale factors, P (one value per thread).
    float alpha[kF32Cols];
    {
      float smax[kF32Cols];
#pragma unroll
      for (int c = 0; c < kF32Cols; ++c) smax[c] = -INFINITY;
#pragma unroll
      for (int w = 0; w < kF32ConsumerWarps; ++w) {
        const float4 v = *reinterpret_cast<const float4*>(Wmax + w * kF32Cols);
        smax[0] = fmaxf(smax[0], v.x);
        smax[1] = fmaxf(smax[1], v.y);
        smax[2] = fmaxf(smax[2], v.z);
        smax[3] = fmaxf(smax[3], v.w);
      }
#pragma unroll
      for (int c = 0; c < kF32Cols; ++c) {
        const float mn = fmaxf(m_run[c], smax[c]);
        alpha[c] = m_run[c] == -INFINITY ? 0.f : fast_exp2(m_run[c] - mn);
        m_run[c] = mn;
      }
    }
    if ((lane & 1u) == 0u) {
      const float mc = pick_col(m_run, my_col);
      float ps[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        ps[r] = xs[r] == -INFINITY ? 0.f : fast_exp2(xs[r] - mc);
        Ps[my_col * kF32PPitch + 8 * warp + 4 * r + (lane >> 3)] = ps[r];
      }
      lpart = fmaf(lpart, pick_col(alpha, my_col), ps[0] + ps[1]);
    }
    named_barrier(1, 32 * kF32ConsumerWarps);

    // ---- PV: dims dbase .. + kDpl, token quads tq and tq + 8.
#pragma unroll
    for (int dd = 0; dd < kDpl; ++dd)
#pragma unroll
      for (int c = 0; c < kF32Cols; ++c) acc[dd][c] *= alpha[c];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t t0 = 4 * (tq + 8 * h);
      const uint32_t pg = t0 >> p.log2_page, s0 = t0 & (P - 1u);
      if (!full_stage && ((okp >> pg) & 1u) == 0u) continue;
      float4 pv[kF32Cols];
#pragma unroll
      for (int c = 0; c < kF32Cols; ++c) pv[c] = *reinterpret_cast<const float4*>(Ps + c * kF32PPitch + t0);
      const float* vrow = Vs + pg * vpitch_f + s0;
#pragma unroll
      for (int dd = 0; dd < kDpl; ++dd) {
        const float4 v = *reinterpret_cast<const float4*>(vrow + (dbase + dd) * P);
#pragma unroll
        for (int c = 0; c < kF32Cols; ++c) {
          float a = acc[dd][c];
          a = fmaf(pv[c].x, v.x, a);
          a = fmaf(pv[c].y, v.y, a);
          a = fmaf(pv[c].z, v.z, a);
          a = fmaf(pv[c].w, v.w, a);
          acc[dd][c] = a;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  grid_launch_dependents();

  // ---- combine: token lanes, then the warps' l in a fixed order.
#pragma unroll
  for (int dd = 0; dd < kDpl; ++dd)
#pragma unroll
    for (int c = 0; c < kF32Cols; ++c) {
      float a = acc[dd][c];
      a += __shfl_xor_sync(0xffffffffu, a, 1);
      a += __shfl_xor_sync(0xffffffffu, a, 2);
      a += __shfl_xor_sync(0xffffffffu, a, 4);
      acc[dd][c] = a;
    }
  lpart += __shfl_xor_sync(0xffffffffu, lpart, 8);
  lpart += __shfl_xor_sync(0xffffffffu, lpart, 16);
  if (lane < 8 && (lane & 1u) == 0u) Lw[warp * kF32Cols + my_col] = lpart;
  named_barrier(1, 32 * kF32ConsumerWarps);
  if (tq != 0) return;
#pragma unroll
  for (int c = 0; c < kF32Cols; ++c) {
    if (!cvalid[c]) continue;
    const uint32_t col = pc.col0 + c;
    const uint32_t r = col / p.group, gq = col % p.group;
    const size_t rh = size_t(r) * p.q_heads + size_t(pc.h) * p.group + gq;
    float* out = p.part + (rh * p.split_stride + pc.slot) * (D + 2);
    if (warp == 0 && dg == 0) {
      float lsum = 0.f;
#pragma unroll
      for (int w = 0; w < kF32ConsumerWarps; ++w) lsum += Lw[w * kF32Cols + c];
      out[0] = m_run[c] == -INFINITY ? -INFINITY : m_run[c] * kLn2;
      out[1] = lsum;
    }
#pragma unroll
    for (int dd = 0; dd < kDpl; dd += 2)
      *reinterpret_cast<float2*>(out + 2 + dbase + dd) = make_float2(acc[dd][c], acc[dd + 1][c]);
  }
}

}  // namespace kvb
