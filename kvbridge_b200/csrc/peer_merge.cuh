#pragma once
// Cross-GPU merge of sequence-shard partials over NVLink peer memory: the
// exchange and the log-sum-exp merge (reference src/attention_shared.cu:
// 295-335, one split per GPU) in one kernel, in place of an all-gather
// followed by merge_kernel<kMergeShards>.
//
// Every rank owns one peer buffer (device memory it exported by CUDA IPC and
// every other rank mapped): a flag block, then two slots of [m | l | n]
// partials (row_heads, row_heads, row_heads * dim floats). Call number
// `epoch` (1, 2, ...) of a rank writes its decode partials into slot
// epoch % 2 of its own buffer; its merge kernel then
//   1. waits for the decode (programmatic dependent launch),
//   2. stores `epoch` into its flag in every rank's buffer (flag word
//      `rank`) with system-scope release stores,
//   3. waits, bounded by wait_limit_ns, until its own flag block shows
//      `epoch` from every rank,
//   4. reads every rank's slot over NVLink and merges (one warp per
//      row-head, all shards' loads in flight at once).
// Two slots make reuse safe without a second handshake: rank r rewrites
// slot s at call e + 2 only after its merge of call e + 1 saw every rank's
// flag e + 1, which each rank stores after its merge of call e, the last
// reader of slot s.
#include <cuda_bf16.h>

#include "kvb_device.cuh"

namespace kvb {

constexpr int kStatusPeerWaitTimeout = 7;  // a rank's partials were not published within the limit
constexpr uint32_t kMaxPeers = 8;
constexpr uint32_t kPeerFlagBytes = 256;  // flag block at the start of a peer buffer
constexpr int kPeerMergeWarps = 4;

// Floats of one slot.
__host__ __device__ inline size_t peer_slot_floats(uint32_t row_heads, uint32_t dim) {
  return size_t(row_heads) * (dim + 2u);
}

struct PeerMergeParams {
  const float* peers[kMaxPeers];  // every rank's buffer base; [rank] is this rank's own
  uint32_t world, rank, epoch, row_heads, dim;
  float* m;
  float* l;
  float* n;
  __half* out;
  __nv_bfloat16* out_bf16;
  unsigned long long wait_limit_ns;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// KD = dims a lane holds (ceil(dim / 32)).
template <int KD>
__global__ void __launch_bounds__(32 * kPeerMergeWarps) merge_peers_kernel(PeerMergeParams p) {
  __shared__ int ready;
  grid_launch_dependents();
  grid_dependency_wait();  // this rank's slot is written
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t RH = p.row_heads, D = p.dim;

  // 2. Publish this rank's slot to every rank: release stores, ordering the
  //    slot's writes (which the preceding grid completed) before the flag.
  //    Every CTA stores the same value, so that no CTA's wait below depends
  //    on another CTA of this grid.
  if (threadIdx.x < p.world) {
    uint32_t* peer_flags = reinterpret_cast<uint32_t*>(const_cast<float*>(p.peers[threadIdx.x]));
    st_release_sys(peer_flags + p.rank, p.epoch);
  }
  // 3. Wait for every rank's slot of this epoch (acquire loads).
  if (threadIdx.x == 0) {
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(p.peers[p.rank]);
    const unsigned long long start = global_ns();
    const long long start_cycles = clock64();
    int ok = 1;
    for (uint32_t s = 0; s < p.world && ok; ++s) {
      for (uint32_t spin = 1; ld_acquire_sys(flags + s) != p.epoch; ++spin) {
        if ((spin & 63u) == 0) {
          const unsigned long long waited = global_ns() - start;
          if (waited > p.wait_limit_ns) {
            record_wait_failure(kStatusPeerWaitTimeout, int(s), static_cast<long long>(waited),
                                clock64() - start_cycles);
            ok = 0;
            break;
          }
        }
      }
    }
    ready = ok;
  }
  __syncthreads();
  if (!ready) return;

  // 4. One warp per row-head: lane s holds shard s's m and l, every lane the
  //    shards' n at its dims d = lane + 32 k.
  const uint32_t rh = blockIdx.x * kPeerMergeWarps + warp;
  if (rh >= RH) return;
  const size_t slot = kPeerFlagBytes / sizeof(float) + (p.epoch & 1u) * peer_slot_floats(RH, D);
  float ms = -INFINITY, ls = 0.f;
  if (lane < p.world) {
    const float* base = p.peers[lane] + slot;
    ms = base[rh];
    ls = base[RH + rh];
  }
  float nv[kMaxPeers][KD];
#pragma unroll
  for (int s = 0; s < int(kMaxPeers); ++s) {
    const float* nb = p.peers[s] + slot + 2u * RH + size_t(rh) * D;
#pragma unroll
    for (int k = 0; k < KD; ++k) {
      const uint32_t d = lane + 32u * k;
      nv[s][k] = (uint32_t(s) < p.world && d < D) ? nb[d] : 0.f;
    }
  }
  // A shard with l = 0 contributes nothing (its n is not used).
  const bool live = lane < p.world && ls > 0.f;
  const float M = warp_max(live ? ms : -INFINITY);
  const float e = live ? expf(ms - M) : 0.f;
  const float L = warp_sum(e * ls);
  const uint32_t livemask = __ballot_sync(0xffffffffu, live);
  float acc[KD];
#pragma unroll
  for (int k = 0; k < KD; ++k) acc[k] = 0.f;
#pragma unroll
  for (int s = 0; s < int(kMaxPeers); ++s) {
    const float es = __shfl_sync(0xffffffffu, e, s);
#pragma unroll
    for (int k = 0; k < KD; ++k) acc[k] = ((livemask >> s) & 1u) != 0u ? fmaf(es, nv[s][k], acc[k]) : acc[k];
  }
  if (lane == 0) {
    p.m[rh] = L > 0.f ? M : -INFINITY;
    p.l[rh] = L;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int k = 0; k < KD; ++k) {
    const uint32_t d = lane + 32u * k;
    if (d >= D) continue;
    const float v = L > 0.f ? acc[k] : 0.f;
    p.n[size_t(rh) * D + d] = v;
    if (p.out != nullptr) p.out[size_t(rh) * D + d] = __float2half_rn(v * inv);
    if (p.out_bf16 != nullptr) p.out_bf16[size_t(rh) * D + d] = __float2bfloat16_rn(v * inv);
  }
}

}  // namespace kvb
