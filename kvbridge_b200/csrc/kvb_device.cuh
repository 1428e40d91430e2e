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

// Non-blocking test of phase `parity` of `bar`.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
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

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core) and tiled TMA helpers, used by the
// TMEM-accumulator partial kernel (decode_tc.cuh). All inline PTX of
// documented sm_100a instructions.
namespace tc {

// Tiled 2-D TMA load global -> shared (no multicast), completing its bytes on
// `bar`. x is the innermost coordinate (a multiple of 16 bytes here).
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int32_t x, int32_t y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// TMEM allocation by one full warp: `cols` columns (a power of two >= 32);
// the TMEM address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst)),
               "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes become visible to the async proxy
// (tensor core operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> s32, one CTA.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}

// The mbarrier receives one arrival once every tcgen05 operation this
// thread issued before has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

// Instruction descriptor, kind::i8: s32 accumulator, signed A and B, both
// K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t m, uint32_t n) {
  return (2u << 4)            // D format: s32
         | (1u << 7)          // A: signed 8-bit
         | (1u << 10)         // B: signed 8-bit
         | ((n >> 3) << 17)   // N / 8
         | ((m >> 4) << 24);  // M / 16
}

// Shared-memory matrix descriptor (tcgen05): start address, leading and
// stride byte offsets (16-byte units), descriptor version 1, layout type
// (0 none, 2 = 128B swizzle, 4 = 64B, 6 = 32B).
enum : uint32_t { kSwizzleNone = 0, kSwizzle128 = 2, kSwizzle64 = 4, kSwizzle32 = 6 };
__device__ __forceinline__ uint64_t smem_desc(const void* start, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  const uint32_t a = smem_addr(start);
  return uint64_t((a & 0x3FFFFu) >> 4) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(layout) << 61);
}

// TMEM -> registers: 32 lanes x 32 bits, `N` consecutive columns per thread
// (thread i of the warp reads lane base + i).
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]);

#define KVB_TMEM_LD_REGS8(o) "=r"(r[o + 0]), "=r"(r[o + 1]), "=r"(r[o + 2]), "=r"(r[o + 3]), \
                             "=r"(r[o + 4]), "=r"(r[o + 5]), "=r"(r[o + 6]), "=r"(r[o + 7])
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : KVB_TMEM_LD_REGS8(0)
               : "r"(taddr)
               : "memory");
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : KVB_TMEM_LD_REGS8(0), KVB_TMEM_LD_REGS8(8)
      : "r"(taddr)
      : "memory");
}
template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : KVB_TMEM_LD_REGS8(0), KVB_TMEM_LD_REGS8(8), KVB_TMEM_LD_REGS8(16), KVB_TMEM_LD_REGS8(24)
      : "r"(taddr)
      : "memory");
}
#undef KVB_TMEM_LD_REGS8

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace tc

}  // namespace kvb
