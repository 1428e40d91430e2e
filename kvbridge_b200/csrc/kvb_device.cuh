#pragma once
// sm_100a device helpers for the decode-attention kernels: mbarrier
// pipelines, bulk (TMA) global->shared copies, the warp-level int8 tensor-core
// MMA, L2 prefetch and bounded waits. Everything is inline PTX of documented
// instructions; nothing here restates a CUDA math-library routine.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace kvb {

// Status codes written to the library's device status word.
enum : int {
  kStatusOk = 0,
  kStatusFullWaitTimeout = 1,   // consumer gave up waiting for a stage
  kStatusEmptyWaitTimeout = 2,  // producer gave up waiting for a free stage
  kStatusDrainTimeout = 3,      // copies still in flight at exit
};

// Device status word of this module (0 = ok; otherwise the largest code any
// kernel reported since the host last read it). All kernels live in one
// translation unit, so this is the module's single definition.
__device__ int g_kvb_status;

// The first bounded wait that gave up since the host last read it:
// {code, block, warp, stage, waited ns (globaltimer), waited SM cycles}.
__device__ long long g_kvb_first_failure[6];

__device__ __forceinline__ void record_wait_failure(int code, int stage, long long ns,
                                                    long long cycles) {
  if (atomicCAS(reinterpret_cast<unsigned long long*>(&g_kvb_first_failure[0]), 0ull,
                static_cast<unsigned long long>(code)) == 0ull) {
    g_kvb_first_failure[1] = blockIdx.x;
    g_kvb_first_failure[2] = threadIdx.x >> 5;
    g_kvb_first_failure[3] = stage;
    g_kvb_first_failure[4] = ns;
    g_kvb_first_failure[5] = cycles;
  }
  atomicMax(&g_kvb_status, code);
}

// Default upper bound of any single pipeline wait (the kernels take the bound
// as a launch parameter). A correct pipeline never waits more than a few
// microseconds; the bound only keeps a broken one from holding the GPU.
constexpr unsigned long long kDefaultWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

enum WaitResult : int { kWaitOk = 0, kWaitTimeout = 1, kWaitAborted = 2 };

// Wait for phase `parity` of `bar` to complete, giving up after `limit_ns`.
// `abort_flag` (shared memory) ends every later wait of the CTA once one wait
// has timed out. A timeout is recorded (first failure wins) with `code` and
// `stage`; an abort is not, so the record names the wait that gave up first.
__device__ __forceinline__ int mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                 volatile int* abort_flag, int code, int stage,
                                                 unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return kWaitOk;
  const unsigned long long start = global_ns();
  const long long start_cycles = clock64();
  for (unsigned spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return kWaitOk;
    if ((spin & 255u) == 0) {
      if (*abort_flag) return kWaitAborted;
      const unsigned long long waited = global_ns() - start;
      if (waited > limit_ns) {
        *abort_flag = 1;
        record_wait_failure(code, stage, static_cast<long long>(waited), clock64() - start_cycles);
        return kWaitTimeout;
      }
    }
  }
}

// Wait until the shared word `*tag` equals `value` (bounded like
// mbar_wait_bounded; same codes and abort behaviour).
__device__ __forceinline__ int wait_tag_bounded(const volatile uint32_t* tag, uint32_t value,
                                                volatile int* abort_flag, int code, int stage,
                                                unsigned long long limit_ns) {
  if (*tag == value) return kWaitOk;
  const unsigned long long start = global_ns();
  const long long start_cycles = clock64();
  for (unsigned spin = 1;; ++spin) {
    if (*tag == value) return kWaitOk;
    if ((spin & 255u) == 0) {
      if (*abort_flag) return kWaitAborted;
      const unsigned long long waited = global_ns() - start;
      if (waited > limit_ns) {
        *abort_flag = 1;
        record_wait_failure(code, stage, static_cast<long long>(waited), clock64() - start_cycles);
        return kWaitTimeout;
      }
    }
  }
}

// One bulk asynchronous copy global -> shared, completing `bytes` of
// transaction count on `bar`. Source, destination and size must be multiples
// of 16 bytes. The L2 policy marks the streamed KV bytes evict-first.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Four-row gather (TMA tile::gather4) from a 2-D tensor map whose box is one
// row high: rows r0..r3 of the map, from column 0, land back to back at
// `dst` (128-byte aligned), completing their bytes on `bar`. The map lives
// in kernel parameter space (a __grid_constant__ parameter).
__device__ __forceinline__ void tma_gather4(void* dst, const void* tmap, int32_t r0, int32_t r1,
                                            int32_t r2, int32_t r3, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(0), "r"(r0), "r"(r1), "r"(r2), "r"(r3),
      "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Prefetch the cache line holding `p` into L2.
__device__ __forceinline__ void prefetch_line_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p) : "memory");
}

// Prefetch `bytes` (multiple of 16, 16-byte aligned address) into L2.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// Programmatic dependent launch: wait for the preceding grid's memory, and
// allow the following grid to start its prologue.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Named barrier over `threads` threads (multiple of 32), id 1..15.
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// D += A * B for one m16n8k32 tile, s8 operands, exact s32 accumulators.
__device__ __forceinline__ void imma_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                           uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2^x on the MUFU unit (ex2.approx, denormal results flushed to zero).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

}  // namespace kvb
