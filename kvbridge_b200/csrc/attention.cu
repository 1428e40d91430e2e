// Host launchers of the kvbridge-b200 decode-attention path: the reference's
// C++ entry points (include/kvbridge/attention_common.h) and the B200
// extensions (include/kvbridge/attention_b200.h). Every kernel of the library
// is instantiated in this one translation unit.
#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <cstring>
#include <limits>
#include <map>
#include <mutex>
#include <stdexcept>
#include <utility>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "kvbridge/attention_b200.h"
#include "kvbridge/attention_common.h"
#include "launch_checks.h"
#include "decode_simt.cuh"
#include "decode_tma.cuh"
#include "decode_tc.cuh"
#include "decode_f32.cuh"
#include "merge.cuh"
#include "peer_merge.cuh"
#include "append_kv.cuh"

namespace kvbridge {
namespace {

using detail::aligned_to;
using detail::cuda_ok;

// ---------------------------------------------------------------------------
// Device facts, cached per device ordinal (they never change for a device).

struct DeviceFacts {
  int sms = 0;
  int major = 0;
};

DeviceFacts current_device_facts() {
  static std::mutex mu;
  static std::map<int, DeviceFacts> cache;
  int dev = 0;
  cuda_ok(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  DeviceFacts f;
  cuda_ok(cudaDeviceGetAttribute(&f.sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
  cuda_ok(cudaDeviceGetAttribute(&f.major, cudaDevAttrComputeCapabilityMajor, dev),
          "compute capability");
  cache.emplace(dev, f);
  return f;
}

// ---------------------------------------------------------------------------
// Tensor-core kernel variants: (head dim, n-tiles of 8 query rows, stages).

struct FastVariant {
  const void* fn = nullptr;
  uint32_t smem = 0;
  void (*launch)(const kvb::DecodeParamsGather&, cudaStream_t) = nullptr;
};

// Failure-path test hooks (attention_b200.h, detail::fail_launch and
// detail::skip_stage): thread-local, one-shot, off unless armed.
thread_local unsigned t_fail_countdown = 0;
thread_local cudaError_t t_fail_code = cudaSuccess;
thread_local uint32_t t_skip_stage = 0xffffffffu;

// The armed launch-failure hook's error for this launch (cudaSuccess when the
// launch is to be made).
cudaError_t injected_launch_failure() {
  if (t_fail_countdown == 0 || --t_fail_countdown != 0) return cudaSuccess;
  return t_fail_code;
}

// The skipped stage for the next partial launch (0xffffffff = none); reading
// disarms the hook.
uint32_t take_skip_stage() {
  const uint32_t stage = t_skip_stage;
  t_skip_stage = 0xffffffffu;
  return stage;
}

std::atomic<unsigned long long> g_wait_limit_ns{kvb::kDefaultWaitLimitNs};

void launch_pdl(const void* fn, dim3 grid, dim3 block, uint32_t smem, cudaStream_t stream,
                void** args, const char* what) {
  if (const cudaError_t injected = injected_launch_failure()) cuda_ok(injected, what);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cuda_ok(cudaLaunchKernelExC(&cfg, fn, args), what);
}

// The merge kernels use 4 KB of shared memory, and left to itself the driver
// gives an SM running one a small shared-memory carveout. A partial-kernel CTA
// (two per SM at ~100 KB each) cannot start on that SM until the merge CTA
// has left and the SM has been reconfigured, which held back the next call's
// CTAs on every SM that ran a merge CTA (~3.5 us late at 64K tokens). Asking
// for the largest carveout keeps both kernels on one configuration.
cudaError_t prefer_max_shared(const void* fn) {
  return cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                              int(cudaSharedmemCarveoutMaxShared));
}

template <int D, int NT, int STAGES, bool SMALL, bool BATCHED>
const void* kernel_fn() {
  if constexpr (SMALL)
    return reinterpret_cast<const void*>(&kvb::decode_partial_kernel_gather<D, NT, STAGES, BATCHED>);
  else
    return reinterpret_cast<const void*>(&kvb::decode_partial_kernel<D, NT, STAGES, false, BATCHED>);
}

template <int D, int NT, int STAGES, bool SMALL, bool BATCHED>
void launch_fast_variant(const kvb::DecodeParamsGather& prm, cudaStream_t stream) {
  const void* fn =
      kernel_fn<D, NT, STAGES, SMALL, BATCHED>();
  constexpr uint32_t smem = kvb::DecodeSmem<D, NT, STAGES, !BATCHED>::kBytes;
  cuda_ok(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
          "decode kernel shared-memory opt-in");
  cuda_ok(prefer_max_shared(fn), "decode kernel carveout");
  // 64-token-page kernels take the parameters without the gather maps.
  kvb::KernelParams<SMALL> copy = prm;
  void* args[] = {&copy};
  launch_pdl(fn, dim3(prm.ctas), dim3(kvb::kDecodeThreads), smem, stream, args,
             "decode partial launch");
}

template <int D, int NT, int STAGES, bool SMALL, bool BATCHED>
FastVariant make_variant() {
  FastVariant v;
  v.fn = kernel_fn<D, NT, STAGES, SMALL, BATCHED>();
  v.smem = kvb::DecodeSmem<D, NT, STAGES, !BATCHED>::kBytes;
  v.launch = &launch_fast_variant<D, NT, STAGES, SMALL, BATCHED>;
  return v;
}

// Page size (small pages have their own producer) and mode (single
// sequence or batched) are template parameters, so that each kernel carries
// only the code it runs; compiling the other paths in cost the 64-token
// single-sequence call ~1.6 us at cfg2.
template <int D, int NT, int STAGES, bool BATCHED>
FastVariant make_variant(bool small_pages) {
  return small_pages ? make_variant<D, NT, STAGES, true, BATCHED>()
                     : make_variant<D, NT, STAGES, false, BATCHED>();
}

// Stage counts keep two CTAs per SM resident (<= ~110 KB each) except at
// dim 256, where one CTA per SM holds 33 KB stages. Single-sequence kernels
// keep their combine buffer in the ring, which makes room for a sixth stage
// at dim 128 (and at dim 256 leaves six stages room beside a merge CTA).
FastVariant fast_variant(uint32_t dim, uint32_t nt, uint32_t page_tokens, bool batched) {
  const bool small = page_tokens < kvb::kStageTokens;
  if (batched) {
    if (dim == 128 && nt == 0) return make_variant<128, 0, 5, true>(small);
    if (dim == 128 && nt == 1) return make_variant<128, 1, 5, true>(small);
    if (dim == 128 && nt == 2) return make_variant<128, 2, 4, true>(small);
    if (dim == 64 && nt == 0) return make_variant<64, 0, 8, true>(small);
    if (dim == 64 && nt == 1) return make_variant<64, 1, 8, true>(small);
    if (dim == 64 && nt == 2) return make_variant<64, 2, 7, true>(small);
    if (dim == 256 && nt == 0) return make_variant<256, 0, 4, true>(small);
    if (dim == 256 && nt == 1) return make_variant<256, 1, 4, true>(small);
    return FastVariant{};
  }
  if (dim == 128 && nt == 0) return make_variant<128, 0, 6, false>(small);
  if (dim == 128 && nt == 1) return make_variant<128, 1, 6, false>(small);
  if (dim == 64 && nt == 0) return make_variant<64, 0, 8, false>(small);
  if (dim == 64 && nt == 1) return make_variant<64, 1, 8, false>(small);
  if (dim == 256 && nt == 0) return make_variant<256, 0, 6, false>(small);
  if (dim == 256 && nt == 1) return make_variant<256, 1, 6, false>(small);
  return FastVariant{};
}

// Resident CTAs of a kernel per SM on the current device (cached).
int resident_ctas(const void* fn, int threads, uint32_t smem) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> cache;
  int dev = 0;
  cuda_ok(cudaGetDevice(&dev), "cudaGetDevice");
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find({dev, fn});
    if (it != cache.end()) return it->second;
  }
  cuda_ok(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
          "decode kernel shared-memory opt-in");
  int blocks = 0;
  cuda_ok(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, threads, smem),
          "occupancy query");
  blocks = std::max(blocks, 1);
  std::lock_guard<std::mutex> lock(mu);
  cache[{dev, fn}] = blocks;
  return blocks;
}

int resident_ctas(const FastVariant& v) { return resident_ctas(v.fn, kvb::kDecodeThreads, v.smem); }

// ---------------------------------------------------------------------------
// tcgen05 (TMEM accumulator) variants of the single-sequence partial kernel:
// (head dim, page tokens, query columns per KV head, ring slots, column
// halves per thread group).

struct TcVariant {
  const void* fn = nullptr;
  uint32_t smem = 0;
  int threads = 0;
  uint32_t columns = 0;  // query columns per KV head it holds
  void (*launch)(const kvb::DecodeParamsTc&, cudaStream_t) = nullptr;
};

template <int D, int P, int NC, int SLOTS, int NH>
const void* tc_kernel_fn() {
  return reinterpret_cast<const void*>(&kvb::decode_partial_tc_kernel<D, P, NC, SLOTS, NH>);
}

template <int D, int P, int NC, int SLOTS, int NH>
void launch_tc_variant(const kvb::DecodeParamsTc& prm, cudaStream_t stream) {
  using L = kvb::TcSmem<D, P, NC, SLOTS, NH>;
  const void* fn = tc_kernel_fn<D, P, NC, SLOTS, NH>();
  constexpr uint32_t smem = L::kDynamicBytes;
  cuda_ok(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
          "decode kernel shared-memory opt-in");
  cuda_ok(prefer_max_shared(fn), "decode kernel carveout");
  kvb::DecodeParamsTc copy = prm;
  void* args[] = {&copy};
  launch_pdl(fn, dim3(prm.ctas), dim3(L::kThreads), smem, stream, args, "decode partial launch");
}

template <int D, int P, int NC, int SLOTS, int NH>
TcVariant make_tc_variant() {
  using L = kvb::TcSmem<D, P, NC, SLOTS, NH>;
  TcVariant v;
  v.fn = tc_kernel_fn<D, P, NC, SLOTS, NH>();
  v.smem = L::kDynamicBytes;
  v.threads = int(L::kThreads);
  v.columns = NC;
  v.launch = &launch_tc_variant<D, P, NC, SLOTS, NH>;
  return v;
}

TcVariant tc_variant(uint32_t dim, uint32_t page_tokens, uint32_t qrows) {
  if (dim == 256 && page_tokens == 32 && qrows <= 48) return make_tc_variant<256, 32, 48, 4, 3>();
  if (dim == 128 && page_tokens == 64 && qrows <= 8) return make_tc_variant<128, 64, 8, 6, 1>();
  return TcVariant{};
}

// Which single-sequence partial kernel runs: 0 = by shape (tcgen05 where it
// was measured to win), 1 = the warp-level MMA kernel, 2 = tcgen05 wherever
// a variant exists, 3 = the general CUDA-core kernel (decode_simt.cuh) for
// every launch_attention call, int8 or fp32 KV. Process-wide
// (detail::set_decode_kernel).
std::atomic<int> g_decode_kernel{0};

uint32_t query_rows(const Shape& s) { return s.rows * (s.q_heads / s.kv_heads); }

// Eager load of the fp32-KV partial kernels (defined with their launcher).
cudaError_t preload_f32_kernels();

// Single sequence: a CTA takes 8 query columns of one KV head (nt = 1), or at
// most 4 in the four-column layout (nt = 0: one query row of a 32/8-head
// model, as at BASELINE cfg1/cfg2); more columns (rows x group up to 64,
// e.g. the reference's native 8 rows x group 6) are cut into column groups,
// one CTA per group and KV range, whose repeated page reads hit L2. Measured
// at 64K tokens with 16 columns, two 8-column groups (51.8 us) beat one
// 16-column CTA (69.3 us), whose PV accumulators spill. (The batched path,
// without column groups, still takes up to 16 columns in one CTA.)
struct ColumnPlan {
  uint32_t nt, groups;
};
constexpr uint32_t kMaxQueryColumns = 64;

ColumnPlan column_plan(uint32_t /*dim*/, uint32_t qrows) {
  return qrows <= 4 ? ColumnPlan{0, 1} : ColumnPlan{1, (qrows + 7) / 8};
}

// Query columns of a CTA for `nt` (decode_tma.cuh, cta_cols).
uint32_t columns_of(uint32_t nt) { return nt == 0 ? 4u : 8u * nt; }

// Batched: one CTA takes a sequence's whole query group (at most 16).
uint32_t batched_nt(uint32_t group) { return group <= 4 ? 0u : (group + 7) / 8; }

// Tensor-core geometry. `max_rows`: query columns per KV head the caller can
// cut into column groups (single sequence), or one group's worth (batched).
bool fast_geometry(uint32_t dim, uint32_t page_tokens, uint32_t qrows, uint32_t max_rows) {
  const bool dim_ok = dim == 64 || dim == 128 || dim == 256;
  const bool page_ok = page_tokens == 16 || page_tokens == 32 || page_tokens == 64;
  return dim_ok && page_ok && qrows >= 1 && qrows <= max_rows;
}

uint32_t log2_exact(uint32_t x) {
  uint32_t r = 0;
  while ((1u << r) < x) ++r;
  return r;
}

// ---------------------------------------------------------------------------
// Merge launches.

// The merge kernel for a layout and a head dim (dims per lane 2, 4 or 8).
template <int KD>
const void* merge_fn_kd(int mode) {
  if (mode == kvb::kMergeScratch)
    return reinterpret_cast<const void*>(&kvb::merge_kernel<kvb::kMergeScratch, KD>);
  if (mode == kvb::kMergeBatched)
    return reinterpret_cast<const void*>(&kvb::merge_kernel<kvb::kMergeBatched, KD>);
  return reinterpret_cast<const void*>(&kvb::merge_kernel<kvb::kMergeShards, KD>);
}

const void* merge_fn(int mode, uint32_t dim) {
  return dim <= 64 ? merge_fn_kd<2>(mode) : dim <= 128 ? merge_fn_kd<4>(mode) : merge_fn_kd<8>(mode);
}

// Merges of more than kMergeWideAbove partials per row-head (reference
// scratch or shard layout): one CTA per 32 dims of a row-head.
const void* merge_wide_fn(int mode) {
  return mode == kvb::kMergeScratch ? reinterpret_cast<const void*>(&kvb::merge_wide_kernel<kvb::kMergeScratch>)
                                    : reinterpret_cast<const void*>(&kvb::merge_wide_kernel<kvb::kMergeShards>);
}

void launch_merge(int mode, const kvb::MergeParams& prm, cudaStream_t stream) {
  if (prm.row_heads == 0) return;
  const bool wide = mode != kvb::kMergeBatched && prm.np > kvb::kMergeWideAbove;
  // One CTA per row-head, or per 32 dims of one.
  const uint32_t blocks = wide ? prm.row_heads * ((prm.dim + 31) / 32) : prm.row_heads;
  kvb::MergeParams copy = prm;
  void* args[] = {&copy};
  const void* fn = wide ? merge_wide_fn(mode) : merge_fn(mode, prm.dim);
  cuda_ok(prefer_max_shared(fn), "merge kernel carveout");
  launch_pdl(fn, dim3(blocks), dim3(32 * (wide ? kvb::kMergeWideWarps : kvb::kMergeWarps)), 0, stream, args,
             "attention merge launch");
}

kvb::MergeParams scratch_merge_params(const Shape& s, float* scratch, uint32_t np, uint32_t stride,
                                      bool fill_empty, float* m, float* l, float* n, void* out,
                                      void* out_bf16 = nullptr) {
  kvb::MergeParams mp{};
  mp.part = scratch;
  mp.m = m;
  mp.l = l;
  mp.n = n;
  mp.out = static_cast<__half*>(out);
  mp.out_bf16 = static_cast<__nv_bfloat16*>(out_bf16);
  mp.row_heads = s.rows * s.q_heads;
  mp.dim = s.dim;
  mp.np = np;
  mp.split_stride = stride;
  mp.fill_empty = fill_empty ? 1u : 0u;
  return mp;
}

void launch_simt(const Shape& s, const DeviceInput& in, float* scratch, uint32_t splits,
                 cudaStream_t stream) {
  kvb::SimtParams sp{};
  sp.q = in.q;
  sp.q_positions = in.q_positions;
  sp.k_positions = in.k_positions;
  sp.table = in.page_table;
  sp.k = in.k;
  sp.v = in.v;
  sp.k_scales = in.k_scales;
  sp.v_scales = in.v_scales;
  sp.scratch = scratch;
  sp.rows = s.rows;
  sp.q_heads = s.q_heads;
  sp.kv_heads = s.kv_heads;
  sp.dim = s.dim;
  sp.page_tokens = s.page_tokens;
  sp.pages = s.pages;
  sp.begin = s.begin;
  sp.end = s.end;
  sp.splits = splits;
  sp.scale = s.scale;
  void* args[] = {&sp};
  const void* fn = s.int8 ? reinterpret_cast<const void*>(&kvb::decode_simt_kernel<true>)
                          : reinterpret_cast<const void*>(&kvb::decode_simt_kernel<false>);
  launch_pdl(fn, dim3(s.rows * s.kv_heads, splits), dim3(kvb::kSimtThreads), 0, stream, args,
             "attention split launch");
}

uint32_t batched_ctas(const FastVariant& v) {
  return uint32_t(current_device_facts().sms) * uint32_t(resident_ctas(v));
}

// The tcgen05 variant a single-sequence call on the tensor-core path uses,
// or none (the warp-level MMA kernel).
TcVariant chosen_tc_variant(const Shape& s) {
  const int choice = g_decode_kernel.load();
  if (choice == 1) return TcVariant{};
  const TcVariant v = tc_variant(s.dim, s.page_tokens, query_rows(s));
  if (v.fn == nullptr) return v;
  if (choice == 2) return v;
  // By shape: many query columns per KV head at dim 256, where the warp-level
  // kernel splits the columns over CTAs that each re-read the pages.
  return (s.dim == 256 && query_rows(s) > 8) ? v : TcVariant{};
}

}  // namespace

// ---------------------------------------------------------------------------
// B200 predicates and planning.

// Granularity of automatic partition counts above it (attention_partitions).
constexpr uint32_t kPartitionQuantum = 128;

bool attention_b200_supported(const Shape& s, const DeviceInput& in) noexcept {
  if (!attention_shape_valid(s) || !s.int8) return false;
  if (!fast_geometry(s.dim, s.page_tokens, query_rows(s), kMaxQueryColumns)) return false;
  return aligned_to(in.q, 16) && aligned_to(in.k, 16) && aligned_to(in.v, 16) &&
         aligned_to(in.k_scales, 16) && aligned_to(in.v_scales, 16);
}

unsigned attention_partitions(const Shape& s, unsigned requested) {
  validate_shape(s);
  const uint32_t stages = kvb::stages_of_range(s.begin, s.end);
  if (stages == 0) return 0;
  uint32_t parts = requested;
  if (parts == 0) {
    const TcVariant tcv = chosen_tc_variant(s);
    if (tcv.fn != nullptr) {
      const uint32_t wave = uint32_t(current_device_facts().sms) *
                            uint32_t(resident_ctas(tcv.fn, tcv.threads, tcv.smem));
      parts = std::max(1u, wave / s.kv_heads);
    } else {
      const ColumnPlan plan = column_plan(s.dim, query_rows(s));
      const FastVariant v = fast_variant(s.dim, plan.nt, s.page_tokens, false);
      const uint32_t sms = uint32_t(current_device_facts().sms);
      const uint32_t wave = v.fn ? sms * uint32_t(resident_ctas(v)) : 1u;
      // One wave of CTAs; above kPartitionQuantum partitions per KV head
      // (few KV heads per GPU, where the many-partials merge runs) a
      // multiple of it, which leaves some SMs' second slot free, so the
      // merge's CTAs are resident before the partial grid ends. Measured
      // on cfg2's share of one rank (65,536 tokens; 4-warp merge): one KV
      // head, 296 slots -> 256 partitions 8.81 us a call (224: 9.01, 192:
      // 9.35, 148: 9.33, 128: 9.14); two KV heads, 148 slots -> 128
      // partitions 10.34 us (148: 11.11). With the 8-warp merge (one round
      // of 256 partials): one KV head 256 -> 8.37 us (192: 8.90, 128:
      // 9.10); two KV heads 128 -> 10.42 us, 148 -> 11.72 us.
      parts = std::max(1u, wave / (s.kv_heads * plan.groups));
      if (parts > kPartitionQuantum) parts -= parts % kPartitionQuantum;
    }
  }
  parts = std::min(parts, stages);
  parts = std::min(parts, split_count(s));
  return std::max(parts, 1u);
}

// ---------------------------------------------------------------------------
// Reference entry points.

cudaError_t preload_attention_reference_kernels() {
  cudaFuncAttributes a{};
  const void* fns[] = {
      reinterpret_cast<const void*>(&kvb::decode_simt_kernel<true>),
      reinterpret_cast<const void*>(&kvb::decode_simt_kernel<false>),
      merge_fn(kvb::kMergeScratch, 64),  merge_fn(kvb::kMergeScratch, 128),
      merge_fn(kvb::kMergeScratch, 256), merge_fn(kvb::kMergeBatched, 64),
      merge_fn(kvb::kMergeBatched, 128), merge_fn(kvb::kMergeBatched, 256),
      merge_fn(kvb::kMergeShards, 64),   merge_fn(kvb::kMergeShards, 128),
      merge_fn(kvb::kMergeShards, 256),  merge_wide_fn(kvb::kMergeScratch),
      merge_wide_fn(kvb::kMergeShards),
  };
  for (const void* fn : fns) {
    cudaError_t code = cudaFuncGetAttributes(&a, fn);
    // The merges (every entry after the two SIMT kernels) share the partial
    // kernels' shared-memory configuration.
    if (code == cudaSuccess && fn != fns[0] && fn != fns[1]) code = prefer_max_shared(fn);
    if (code != cudaSuccess) return code;
  }
  return cudaSuccess;
}

cudaError_t preload_attention_mma_kernels() {
  int dev = 0, major = 0;
  cudaError_t code = cudaGetDevice(&dev);
  if (code != cudaSuccess) return code;
  code = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (code != cudaSuccess) return code;
  if (major != 10) return cudaErrorNotSupported;
  const std::pair<uint32_t, uint32_t> variants[] = {{128, 1}, {128, 2}, {64, 1}, {64, 2}, {256, 1}};
  for (int mode = 0; mode < 4; ++mode) {
    for (const auto& dv : variants) {
      const FastVariant v = fast_variant(dv.first, dv.second, mode & 1 ? 16u : 64u, mode >= 2);
      if (v.fn == nullptr) continue;
      cudaFuncAttributes a{};
      code = cudaFuncGetAttributes(&a, v.fn);
      if (code != cudaSuccess) return code;
      code = cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(v.smem));
      if (code != cudaSuccess) return code;
    }
  }
  return cudaSuccess;
}

cudaError_t preload_attention_kernels() {
  cudaError_t code = preload_attention_reference_kernels();
  if (code == cudaSuccess) code = preload_attention_mma_kernels();
  return code == cudaSuccess ? preload_f32_kernels() : code;
}

namespace {

// Stages per CTA prefetched into L2 while the preceding grid finishes. At
// cfg2 (28 stages a CTA) 0, 2, 4, 5 and 6 stages gave 26.7, 24.9, 23.7,
// 23.6 and 23.7 us a call: the prefetch fills the HBM time the previous
// call's drain and merge leave idle; more of it competes with that call.
constexpr uint32_t kPrefetchStages = 5;

// cuTensorMapEncodeTiled through the runtime's driver entry point (the
// library does not link libcuda); null when the driver does not offer it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult found{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &found) !=
            cudaSuccess ||
        found != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

// 16-token pages at dim <= 128: tensor maps of the K and V pools with one
// row of page_tokens * dim bytes (read as 8-byte elements, <= 256 a row) per
// (page, KV head), for the producer's four-row gathers. Anything that does
// not fit a map (or a missing encoder) leaves gather_kv = 0: per-page copies.
void set_gather_maps(kvb::DecodeParamsGather& prm, uint32_t dim, uint64_t pages) {
  prm.gather_kv = 0;
  if (prm.page_tokens != 16) return;
  const uint64_t row_bytes = uint64_t(prm.page_tokens) * dim;
  const uint64_t row_elems = row_bytes / 8;
  const uint64_t rows = pages * prm.kv_heads;
  if (row_bytes % 16 != 0 || row_elems == 0 || row_elems > 256 || rows == 0 ||
      rows > 0x7fffffffull)
    return;
  if (!aligned_to(prm.k, 16) || !aligned_to(prm.v, 16)) return;
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr) return;
  auto make = [&](CUtensorMap* map, const void* base) {
    const cuuint64_t dims[2] = {row_elems, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {cuuint32_t(row_elems), 1};
    const cuuint32_t elem_strides[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides,
                  box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
  };
  if (make(&prm.tm_k, prm.k) && make(&prm.tm_v, prm.v)) prm.gather_kv = 1;
}

// Kernel parameters of a single-sequence partial kernel (the tensor-core
// kernels, or with tensor_core = false the fp32-KV kernel); partials go to
// `scratch` with `split_stride` slots per row-head.
kvb::DecodeParamsGather single_params(const Shape& s, const DeviceInput& in, uint32_t parts,
                                float* scratch, uint32_t split_stride, bool tensor_core = true) {
  kvb::DecodeParamsGather prm{};
  prm.q = in.q;
  prm.q_positions = in.q_positions;
  prm.k_positions = in.k_positions;
  prm.table = in.page_table;
  prm.k = static_cast<const int8_t*>(in.k);
  prm.v = static_cast<const int8_t*>(in.v);
  prm.k_scales = in.k_scales;
  prm.v_scales = in.v_scales;
  prm.seq_lens = nullptr;
  prm.part = scratch;
  prm.batch = 1;
  prm.rows = s.rows;
  prm.q_heads = s.q_heads;
  prm.kv_heads = s.kv_heads;
  prm.group = s.q_heads / s.kv_heads;
  prm.qr = query_rows(s);
  prm.page_tokens = s.page_tokens;
  prm.log2_page = log2_exact(s.page_tokens);
  prm.pages = s.pages;
  prm.table_stride = 0;
  prm.begin = s.begin;
  prm.end = s.end;
  prm.seg_stages = kvb::stages_of_range(s.begin, s.end);
  prm.split_stride = split_stride;
  prm.max_tokens = s.tokens;
  const ColumnPlan plan = column_plan(s.dim, query_rows(s));
  prm.col_groups = plan.groups;
  prm.group_cols = columns_of(plan.nt);
  prm.ctas = parts * s.kv_heads * plan.groups;
  prm.total_stages = uint64_t(prm.seg_stages) * s.kv_heads;
  prm.score_scale = s.scale;
  prm.wait_limit_ns = wait_limit_ns();
  // The stage-skip test hook and the gather maps belong to the tensor-core
  // kernels; the fp32-KV kernel neither reads them nor consumes the hook.
  prm.fault_stage = tensor_core ? take_skip_stage() : 0xffffffffu;
  if (tensor_core) set_gather_maps(prm, s.dim, s.pages);
  return prm;
}

// Tensor maps of the tcgen05 kernel: K rows of `dim` bytes per (page, KV
// head, slot) in boxes of 128 bytes x page_tokens rows, 128-byte swizzle;
// V as 64-byte rows (one dim of a 64-token page, two of a 32-token page) in
// boxes of one page's rows, 64-byte swizzle (the K-major operand layouts of
// tcgen05.mma). False when they cannot be encoded.
bool set_tc_maps(kvb::DecodeParamsTc& prm, uint32_t dim) {
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  const uint64_t P = prm.page_tokens;
  const uint64_t units = uint64_t(prm.pages) * prm.kv_heads;
  const cuuint32_t elem_strides[2] = {1, 1};
  const cuuint64_t k_dims[2] = {dim, units * P};
  const cuuint64_t k_strides[1] = {dim};
  const cuuint32_t k_box[2] = {128, cuuint32_t(P)};
  // 64-byte V rows: one dim of a 64-token page, or two dims of a 32-token page.
  const uint64_t v_rows_per_page = dim * P / 64;
  const cuuint64_t v_dims[2] = {64, units * v_rows_per_page};
  const cuuint64_t v_strides[1] = {64};
  const cuuint32_t v_box[2] = {64, cuuint32_t(v_rows_per_page)};
  if (k_dims[1] > 0x7fffffffull || v_dims[1] > 0x7fffffffull) return false;
  return encode(&prm.tm_k, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(prm.k), k_dims, k_strides,
                k_box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS &&
         encode(&prm.tm_v, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(prm.v), v_dims, v_strides,
                v_box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The single-sequence partial kernel (tcgen05 or warp-level MMA, as chosen
// for the shape) over `parts` partitions; partials go to `scratch` with
// `split_stride` slots per row-head.
void launch_single_partials(const Shape& s, const DeviceInput& in, uint32_t parts, float* scratch,
                            uint32_t split_stride, cudaStream_t stream) {
  kvb::DecodeParamsGather prm = single_params(s, in, parts, scratch, split_stride);
  prm.prefetch_stages = kPrefetchStages;
  const TcVariant tcv = chosen_tc_variant(s);
  if (tcv.fn != nullptr) {
    kvb::DecodeParamsTc tp{};
    static_cast<kvb::DecodeParams&>(tp) = static_cast<const kvb::DecodeParams&>(prm);
    tp.col_groups = 1;
    tp.group_cols = tcv.columns;
    tp.ctas = parts * s.kv_heads;
    if (set_tc_maps(tp, s.dim)) {
      tcv.launch(tp, stream);
      return;
    }
  }
  fast_variant(s.dim, prm.group_cols == 4 ? 0 : prm.group_cols / 8, s.page_tokens, false).launch(prm, stream);
}

// ---------------------------------------------------------------------------
// fp32 KV (Shape::int8 == false): the streaming kernel of decode_f32.cuh for
// head dims 64 and 128, 16/32/64-token pages and up to 16 query columns per
// KV head (4 a CTA; more columns run as column groups whose CTAs share the
// pages in L2), with 16-byte aligned q, k and v. Every other fp32 shape runs
// the general kernel. One CTA per SM (a ring of 3 stages of 64 KB at dim
// 128, 6 of 32 KB at dim 64).

constexpr uint32_t kF32MaxColumns = 16;

struct F32Variant {
  const void* fn = nullptr;
  uint32_t smem = 0;
};

template <int D, int STAGES>
F32Variant make_f32_variant() {
  return F32Variant{reinterpret_cast<const void*>(&kvb::decode_partial_f32_kernel<D, STAGES>),
                    kvb::F32Layout<D, STAGES>::kBytes};
}

F32Variant f32_variant(uint32_t dim) {
  return dim == 64 ? make_f32_variant<64, 6>() : make_f32_variant<128, 3>();
}

bool f32_geometry(const Shape& s, const DeviceInput& in, const float* scratch) {
  return !s.int8 && (s.dim == 64 || s.dim == 128) &&
         (s.page_tokens == 16 || s.page_tokens == 32 || s.page_tokens == 64) &&
         query_rows(s) >= 1 && query_rows(s) <= kF32MaxColumns && aligned_to(in.q, 16) &&
         aligned_to(in.k, 16) && aligned_to(in.v, 16) && aligned_to(scratch, 8);
}

uint32_t f32_column_groups(const Shape& s) {
  return (query_rows(s) + kvb::kF32Cols - 1) / kvb::kF32Cols;
}

// Partitions per KV head: one CTA per SM over all heads and column groups
// unless the caller asked for a count; at most one per stage and split.
uint32_t f32_partitions(const Shape& s, uint32_t requested) {
  const uint32_t stages = kvb::stages_of_range(s.begin, s.end);
  if (stages == 0) return 0;
  const uint32_t sms = uint32_t(current_device_facts().sms);
  uint32_t parts = requested != 0 ? requested : sms / (s.kv_heads * f32_column_groups(s));
  parts = std::min(std::max(parts, 1u), std::min(stages, split_count(s)));
  return parts;
}

void launch_f32_partials(const Shape& s, const DeviceInput& in, uint32_t parts, float* scratch,
                         uint32_t split_stride, cudaStream_t stream) {
  kvb::DecodeParams prm = single_params(s, in, parts, scratch, split_stride, false);
  prm.group_cols = kvb::kF32Cols;
  prm.col_groups = f32_column_groups(s);
  prm.ctas = parts * s.kv_heads * prm.col_groups;
  const F32Variant v = f32_variant(s.dim);
  cuda_ok(cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(v.smem)),
          "fp32 decode kernel shared-memory opt-in");
  void* args[] = {&prm};
  launch_pdl(v.fn, dim3(prm.ctas), dim3(kvb::kF32Threads), v.smem, stream, args,
             "fp32 decode partial launch");
}

cudaError_t preload_f32_kernels() {
  for (uint32_t dim : {64u, 128u}) {
    const F32Variant v = f32_variant(dim);
    cudaFuncAttributes a{};
    cudaError_t code = cudaFuncGetAttributes(&a, v.fn);
    if (code == cudaSuccess)
      code = cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(v.smem));
    if (code != cudaSuccess) return code;
  }
  return cudaSuccess;
}

}  // namespace

namespace detail {
void set_decode_kernel(int choice) noexcept { g_decode_kernel.store(choice < 0 || choice > 3 ? 0 : choice); }
int decode_kernel() noexcept { return g_decode_kernel.load(); }
}  // namespace detail

unsigned launch_attention_partials(const Shape& s, const DeviceInput& in, unsigned partitions,
                                   float* scratch, cudaStream_t stream) {
  if (scratch == nullptr) throw std::invalid_argument("scratch must be a non-null device buffer");
  detail::check_inputs(s, in, scratch, scratch, scratch, scratch);
  if (!attention_b200_supported(s, in))
    throw std::invalid_argument("launch_attention_partials needs the tensor-core geometry "
                                "(attention_b200_supported)");
  const uint32_t splits = split_count(s);
  const uint32_t parts = attention_partitions(s, partitions);
  if (parts == 0) return 0;
  launch_single_partials(s, in, parts, scratch, splits, stream);
  return parts;
}

void merge_attention_ex(const Shape& s, const float* scratch, unsigned partitions, float* m,
                        float* l, float* n, void* out_f16, void* out_bf16, cudaStream_t stream) {
  detail::check_outputs(s, scratch, m, l, n);
  const uint32_t splits = split_count(s);
  if (partitions > splits)
    throw std::invalid_argument("merge partitions exceed split_count(shape)");
  launch_merge(kvb::kMergeScratch,
               scratch_merge_params(s, const_cast<float*>(scratch), partitions, splits,
                                    partitions < splits, m, l, n, out_f16, out_bf16),
               stream);
}

void merge_attention_ex(const Shape& s, const float* scratch, unsigned partitions, float* m,
                        float* l, float* n, void* out_f16, cudaStream_t stream) {
  merge_attention_ex(s, scratch, partitions, m, l, n, out_f16, nullptr, stream);
}

void launch_attention_ex(const Shape& s, const DeviceInput& in, const LaunchOptions& opt,
                         float* scratch, float* m, float* l, float* n, cudaStream_t stream) {
  detail::check_inputs(s, in, scratch, m, l, n);
  const uint32_t splits = split_count(s);
  const bool general = g_decode_kernel.load() == 3;
  if (!attention_b200_supported(s, in) || general) {
    const uint32_t parts = !general && f32_geometry(s, in, scratch) ? f32_partitions(s, opt.partitions) : 0u;
    if (parts != 0) {
      launch_f32_partials(s, in, parts, scratch, splits, stream);
      // The partial kernel has already marked splits [parts, splits) empty.
      launch_merge(kvb::kMergeScratch,
                   scratch_merge_params(s, scratch, parts, splits, false, m, l, n, opt.out_f16,
                                        opt.out_bf16),
                   stream);
      return;
    }
    launch_simt(s, in, scratch, splits, stream);
    launch_merge(kvb::kMergeScratch,
                 scratch_merge_params(s, scratch, splits, splits, false, m, l, n, opt.out_f16,
                                      opt.out_bf16),
                 stream);
    return;
  }
  const uint32_t parts = launch_attention_partials(s, in, opt.partitions, scratch, stream);
  // The partial kernel has already marked splits [parts, splits) empty.
  launch_merge(kvb::kMergeScratch,
               scratch_merge_params(s, scratch, parts, splits, false, m, l, n, opt.out_f16,
                                    opt.out_bf16),
               stream);
}

void launch_attention(const Shape& s, const DeviceInput& in, float* scratch, float* m, float* l,
                      float* n, cudaStream_t stream) {
  launch_attention_ex(s, in, LaunchOptions{0, nullptr}, scratch, m, l, n, stream);
}

void launch_attention_mma(const Shape& s, const DeviceInput& in, float* scratch, float* m,
                          float* l, float* n, cudaStream_t stream) {
  detail::check_inputs(s, in, scratch, m, l, n);
  if (!attention_mma_supported(s))
    throw std::invalid_argument(
        "launch_attention_mma requires int8 KV, rows8/group6/dim256/page32 and a page-aligned "
        "begin");
  cuda_ok(preload_attention_mma_kernels(), "MMA current-context preparation");
  launch_attention_ex(s, in, LaunchOptions{0, nullptr}, scratch, m, l, n, stream);
}

void merge_attention(const Shape& s, const float* scratch, unsigned splits, float* m, float* l,
                     float* n, cudaStream_t stream) {
  detail::check_outputs(s, scratch, m, l, n);
  if (splits != split_count(s))
    throw std::invalid_argument("merge split count does not match shape");
  launch_merge(kvb::kMergeScratch,
               scratch_merge_params(s, const_cast<float*>(scratch), splits, splits, false, m, l,
                                    n, nullptr),
               stream);
}

// ---------------------------------------------------------------------------
// Batched ragged decode.

const char* batch_shape_error(const BatchShape& s) noexcept {
  if (s.batch == 0 || s.q_heads == 0 || s.kv_heads == 0)
    return "batch and head counts must be positive";
  if (s.q_heads % s.kv_heads) return "q_heads must be divisible by kv_heads";
  if (!fast_geometry(s.dim, s.page_tokens, s.q_heads / s.kv_heads, s.dim == 256 ? 8u : 16u))
    return "batched decode needs dim 64/128/256, page_tokens 16/32/64 and a query group of at "
           "most 16 (8 at dim 256)";
  if (s.pages == 0 || s.table_stride == 0) return "pages and table_stride must be positive";
  if (uint64_t(s.max_tokens) > uint64_t(s.table_stride) * s.page_tokens)
    return "max_tokens exceeds the block-table row capacity";
  if (!std::isfinite(s.scale)) return "score scale must be finite";
  if (uint64_t(s.batch) * s.q_heads > 0x7fffffffull) return "batch/head product too large";
  // The batched kernel addresses the pool with 64-bit offsets; a pool is
  // bounded only by device memory (kept below 2^48 bytes here).
  const uint64_t extent = uint64_t(s.pages) * s.kv_heads * s.page_tokens * s.dim;
  if (extent >= (uint64_t(1) << 48)) return "physical KV pool exceeds 2^48 bytes";
  if (uint64_t(s.batch) * s.table_stride > std::numeric_limits<uint32_t>::max())
    return "block table exceeds 32-bit indexing";
  return nullptr;
}

size_t batch_workspace_bytes(const BatchShape& s) {
  if (const char* e = batch_shape_error(s)) throw std::invalid_argument(e);
  const uint32_t group = s.q_heads / s.kv_heads;
  const FastVariant v = fast_variant(s.dim, batched_nt(group), s.page_tokens, true);
  const uint64_t slots = uint64_t(batched_ctas(v)) + uint64_t(s.batch) * s.kv_heads;
  return size_t(slots * group * (s.dim + 2) * sizeof(float));
}

void launch_attention_batched(const BatchShape& s, const BatchInput& in, void* workspace,
                              size_t workspace_bytes, float* m, float* l, float* n, void* out_f16,
                              cudaStream_t stream) {
  launch_attention_batched(s, in, workspace, workspace_bytes, m, l, n, out_f16, nullptr, stream);
}

void launch_attention_batched(const BatchShape& s, const BatchInput& in, void* workspace,
                              size_t workspace_bytes, float* m, float* l, float* n, void* out_f16,
                              void* out_bf16, cudaStream_t stream) {
  if (const char* e = batch_shape_error(s)) throw std::invalid_argument(e);
  if (!in.q || !in.seq_lens || !in.block_table || !in.k || !in.v || !in.k_scales ||
      !in.v_scales || !workspace || !m || !l || !n)
    throw std::invalid_argument("batched decode buffers must be non-null");
  if (!aligned_to(in.q, 16) || !aligned_to(in.k, 16) || !aligned_to(in.v, 16) ||
      !aligned_to(in.k_scales, 16) || !aligned_to(in.v_scales, 16) || !aligned_to(workspace, 16))
    throw std::invalid_argument("batched decode buffers must be 16-byte aligned");
  if (workspace_bytes < batch_workspace_bytes(s))
    throw std::invalid_argument("workspace smaller than batch_workspace_bytes(shape)");
  const uint32_t group = s.q_heads / s.kv_heads;
  const FastVariant v = fast_variant(s.dim, batched_nt(group), s.page_tokens, true);
  kvb::DecodeParamsGather prm{};
  prm.q = in.q;
  prm.table = in.block_table;
  prm.k = in.k;
  prm.v = in.v;
  prm.k_scales = in.k_scales;
  prm.v_scales = in.v_scales;
  prm.seq_lens = in.seq_lens;
  prm.part = static_cast<float*>(workspace);
  prm.batch = s.batch;
  prm.rows = 1;
  prm.q_heads = s.q_heads;
  prm.kv_heads = s.kv_heads;
  prm.group = group;
  prm.qr = group;
  prm.page_tokens = s.page_tokens;
  prm.log2_page = log2_exact(s.page_tokens);
  prm.pages = s.pages;
  prm.table_stride = s.table_stride;
  prm.max_tokens = s.max_tokens;
  prm.ctas = batched_ctas(v);
  prm.col_groups = 1;
  prm.group_cols = columns_of(batched_nt(group));
  prm.score_scale = s.scale;
  prm.prefetch_stages = kPrefetchStages;
  prm.wait_limit_ns = wait_limit_ns();
  prm.fault_stage = take_skip_stage();
  set_gather_maps(prm, s.dim, s.pages);
  v.launch(prm, stream);

  kvb::MergeParams mp{};
  mp.part = static_cast<float*>(workspace);
  mp.m = m;
  mp.l = l;
  mp.n = n;
  mp.out = static_cast<__half*>(out_f16);
  mp.out_bf16 = static_cast<__nv_bfloat16*>(out_bf16);
  mp.row_heads = s.batch * s.q_heads;
  mp.dim = s.dim;
  mp.seq_lens = in.seq_lens;
  mp.batch = s.batch;
  mp.q_heads = s.q_heads;
  mp.kv_heads = s.kv_heads;
  mp.group = group;
  mp.max_tokens = s.max_tokens;
  mp.ctas = prm.ctas;
  launch_merge(kvb::kMergeBatched, mp, stream);
}

void merge_attention_shards_ex(unsigned shards, unsigned row_heads, unsigned dim,
                               const float* m_parts, const float* l_parts, const float* n_parts,
                               size_t shard_stride, float* m, float* l, float* n, void* out_f16,
                               void* out_bf16, cudaStream_t stream) {
  if (shards == 0 || row_heads == 0 || dim == 0 || dim > 256)
    throw std::invalid_argument("shards, row_heads must be positive and dim in [1,256]");
  if (!m_parts || !l_parts || !n_parts || !m || !l || !n)
    throw std::invalid_argument("shard merge buffers must be non-null");
  if (shard_stride != 0 && shard_stride < row_heads)
    throw std::invalid_argument("shard_stride must be 0 or at least row_heads");
  kvb::MergeParams mp{};
  mp.m_parts = m_parts;
  mp.l_parts = l_parts;
  mp.n_parts = n_parts;
  mp.m = m;
  mp.l = l;
  mp.n = n;
  mp.out = static_cast<__half*>(out_f16);
  mp.out_bf16 = static_cast<__nv_bfloat16*>(out_bf16);
  mp.row_heads = row_heads;
  mp.dim = dim;
  mp.np = shards;
  mp.shard_stride = shard_stride;
  launch_merge(kvb::kMergeShards, mp, stream);
}

void merge_attention_shards(unsigned shards, unsigned row_heads, unsigned dim,
                            const float* m_parts, const float* l_parts, const float* n_parts,
                            float* m, float* l, float* n, void* out_f16, cudaStream_t stream) {
  merge_attention_shards_ex(shards, row_heads, dim, m_parts, l_parts, n_parts, 0, m, l, n, out_f16,
                            nullptr, stream);
}

// ---------------------------------------------------------------------------
// Cross-GPU merge over NVLink peer memory (peer_merge.cuh).

size_t peer_buffer_bytes(unsigned row_heads, unsigned dim) {
  if (row_heads == 0 || dim == 0 || dim > 256)
    throw std::invalid_argument("row_heads must be positive and dim in [1,256]");
  return kvb::kPeerFlagBytes + 2 * kvb::peer_slot_floats(row_heads, dim) * sizeof(float);
}

float* peer_slot(void* buffer, unsigned epoch, unsigned row_heads, unsigned dim) {
  if (buffer == nullptr) throw std::invalid_argument("peer buffer is null");
  return reinterpret_cast<float*>(static_cast<char*>(buffer) + kvb::kPeerFlagBytes) +
         (epoch & 1u) * kvb::peer_slot_floats(row_heads, dim);
}

void peer_buffer_alloc(size_t bytes, void** buffer, unsigned char handle[64]) {
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  if (buffer == nullptr || handle == nullptr) throw std::invalid_argument("output pointers are null");
  if (bytes < kvb::kPeerFlagBytes) throw std::invalid_argument("peer buffer smaller than its flag block");
  void* p = nullptr;
  cuda_ok(cudaMalloc(&p, bytes), "peer buffer cudaMalloc");
  // Flags start at 0 (epochs count from 1).
  cudaError_t code = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h{};
  if (code == cudaSuccess) code = cudaIpcGetMemHandle(&h, p);
  if (code != cudaSuccess) {
    cudaFree(p);
    cuda_ok(code, "peer buffer export");
  }
  std::memcpy(handle, &h, sizeof(h));
  *buffer = p;
}

void peer_buffer_open(const unsigned char handle[64], void** peer_buffer) {
  if (handle == nullptr || peer_buffer == nullptr) throw std::invalid_argument("handle or output is null");
  cudaIpcMemHandle_t h{};
  std::memcpy(&h, handle, sizeof(h));
  cuda_ok(cudaIpcOpenMemHandle(peer_buffer, h, cudaIpcMemLazyEnablePeerAccess), "peer buffer open");
}

void peer_buffer_close(void* peer_buffer) {
  if (peer_buffer != nullptr) cuda_ok(cudaIpcCloseMemHandle(peer_buffer), "peer buffer close");
}

void peer_buffer_free(void* buffer) {
  if (buffer != nullptr) cuda_ok(cudaFree(buffer), "peer buffer free");
}

void merge_attention_peers(const void* const* buffers, unsigned world, unsigned rank, unsigned epoch,
                           unsigned row_heads, unsigned dim, float* m, float* l, float* n, void* out_f16,
                           void* out_bf16, cudaStream_t stream) {
  if (world == 0 || world > kvb::kMaxPeers || rank >= world)
    throw std::invalid_argument("world must be in [1, 8] and rank below it");
  if (epoch == 0) throw std::invalid_argument("epochs count from 1");
  if (row_heads == 0 || dim == 0 || dim > 256)
    throw std::invalid_argument("row_heads must be positive and dim in [1,256]");
  if (buffers == nullptr || !m || !l || !n) throw std::invalid_argument("peer merge buffers must be non-null");
  kvb::PeerMergeParams pp{};
  for (unsigned i = 0; i < world; ++i) {
    if (buffers[i] == nullptr || !aligned_to(buffers[i], 16))
      throw std::invalid_argument("peer buffers must be non-null and 16-byte aligned");
    pp.peers[i] = static_cast<const float*>(buffers[i]);
  }
  pp.world = world;
  pp.rank = rank;
  pp.epoch = epoch;
  pp.row_heads = row_heads;
  pp.dim = dim;
  pp.m = m;
  pp.l = l;
  pp.n = n;
  pp.out = static_cast<__half*>(out_f16);
  pp.out_bf16 = static_cast<__nv_bfloat16*>(out_bf16);
  pp.wait_limit_ns = wait_limit_ns();
  const uint32_t kd = (dim + 31) / 32;
  const void* fn = kd <= 1   ? reinterpret_cast<const void*>(&kvb::merge_peers_kernel<1>)
                   : kd <= 2 ? reinterpret_cast<const void*>(&kvb::merge_peers_kernel<2>)
                   : kd <= 4 ? reinterpret_cast<const void*>(&kvb::merge_peers_kernel<4>)
                             : reinterpret_cast<const void*>(&kvb::merge_peers_kernel<8>);
  void* args[] = {&pp};
  launch_pdl(fn, dim3((row_heads + kvb::kPeerMergeWarps - 1) / kvb::kPeerMergeWarps),
             dim3(32 * kvb::kPeerMergeWarps), 0, stream, args, "peer merge launch");
}

// ---------------------------------------------------------------------------
// Paged KV append.

const char* append_shape_error(const AppendShape& s) noexcept {
  if (s.kv_heads == 0) return "kv_heads must be positive";
  if (s.dim == 0 || s.dim > 256) return "dim must be in [1, 256]";
  if (s.page_tokens == 0) return "page_tokens must be positive";
  if (s.pages == 0) return "pages must be positive";
  // Pool extent pages * kv_heads * page_tokens * dim must stay below 2^48.
  const uint64_t per_page = uint64_t(s.kv_heads) * s.page_tokens * s.dim;
  if (uint64_t(s.pages) > ((uint64_t(1) << 48) - 1) / per_page) return "pool extent exceeds 2^48";
  return nullptr;
}

void append_kv(const AppendShape& s, const AppendInput& in, cudaStream_t stream) {
  if (const char* e = append_shape_error(s)) throw std::invalid_argument(e);
  if (s.tokens == 0) return;
  if (in.k_new == nullptr || in.v_new == nullptr || in.slots == nullptr || in.k == nullptr ||
      in.v == nullptr || in.k_scales == nullptr || in.v_scales == nullptr)
    throw std::invalid_argument("append rows, slots and the pool must be non-null device buffers");
  if (!aligned_to(in.k_new, 4) || !aligned_to(in.v_new, 4) || !aligned_to(in.k_scales, 4) ||
      !aligned_to(in.v_scales, 4) || !aligned_to(in.slots, 8))
    throw std::invalid_argument("append float buffers must be 4-byte and slots 8-byte aligned");
  const uint64_t rows = uint64_t(s.tokens) * s.kv_heads * 2;
  const uint64_t blocks = (rows + kvb::kAppendWarps - 1) / kvb::kAppendWarps;
  if (blocks > 0x7fffffffull) throw std::invalid_argument("append call too large for one grid");
  kvb::AppendParams prm{};
  prm.k_new = in.k_new;
  prm.v_new = in.v_new;
  prm.slots = in.slots;
  prm.k = in.k;
  prm.v = in.v;
  prm.k_scales = in.k_scales;
  prm.v_scales = in.v_scales;
  prm.tokens = s.tokens;
  prm.kv_heads = s.kv_heads;
  prm.dim = s.dim;
  prm.page_tokens = s.page_tokens;
  prm.slots_total = uint64_t(s.pages) * s.page_tokens;
  if (const cudaError_t injected = injected_launch_failure()) cuda_ok(injected, "append launch");
  kvb::append_kv_kernel<<<dim3(uint32_t(blocks)), dim3(32 * kvb::kAppendWarps), 0, stream>>>(prm);
  cuda_ok(cudaGetLastError(), "append launch");
}

cudaError_t read_device_status(int* status) {
  if (status == nullptr) return cudaErrorInvalidValue;
  int value = 0;
  cudaError_t code = cudaMemcpyFromSymbol(&value, kvb::g_kvb_status, sizeof(int));
  if (code != cudaSuccess) return code;
  const int zero = 0;
  code = cudaMemcpyToSymbol(kvb::g_kvb_status, &zero, sizeof(int));
  *status = value;
  return code;
}

cudaError_t read_wait_failure(long long* record6) {
  if (record6 == nullptr) return cudaErrorInvalidValue;
  cudaError_t code = cudaMemcpyFromSymbol(record6, kvb::g_kvb_first_failure, 6 * sizeof(long long));
  if (code != cudaSuccess) return code;
  const long long zeros[6] = {0, 0, 0, 0, 0, 0};
  return cudaMemcpyToSymbol(kvb::g_kvb_first_failure, zeros, sizeof(zeros));
}

void set_wait_limit_ns(unsigned long long ns) noexcept {
  g_wait_limit_ns.store(ns == 0 ? kvb::kDefaultWaitLimitNs : ns);
}

unsigned long long wait_limit_ns() noexcept { return g_wait_limit_ns.load(); }

namespace detail {

cudaError_t read_tc_trace(unsigned long long* out, size_t count, bool* available) noexcept {
#ifdef KVB_TC_TRACE
  *available = true;
  const size_t all = size_t(kvb::kTraceCtas) * kvb::kTraceTiles * kvb::kTraceEvents;
  cudaError_t code = cudaMemcpyFromSymbol(out, kvb::g_tc_trace, std::min(count, all) * sizeof(unsigned long long));
  if (code != cudaSuccess) return code;
  static const unsigned long long zeros[kvb::kTraceCtas][kvb::kTraceTiles][kvb::kTraceEvents] = {};
  return cudaMemcpyToSymbol(kvb::g_tc_trace, zeros, sizeof(zeros));
#else
  (void)out;
  (void)count;
  *available = false;
  return cudaSuccess;
#endif
}

cudaError_t read_cta_trace(unsigned long long* out, size_t count, bool* available) noexcept {
#ifdef KVB_TC_TRACE
  *available = true;
  const size_t all = size_t(kvb::kCtaTraceCtas) * kvb::kCtaTraceEvents;
  cudaError_t code = cudaMemcpyFromSymbol(out, kvb::g_cta_trace, std::min(count, all) * sizeof(unsigned long long));
  if (code != cudaSuccess) return code;
  static const unsigned long long zeros[kvb::kCtaTraceCtas][kvb::kCtaTraceEvents] = {};
  return cudaMemcpyToSymbol(kvb::g_cta_trace, zeros, sizeof(zeros));
#else
  (void)out;
  (void)count;
  *available = false;
  return cudaSuccess;
#endif
}

cudaError_t read_merge_trace(unsigned long long* out, size_t count, bool* available) noexcept {
#ifdef KVB_TC_TRACE
  *available = true;
  const size_t all = size_t(kvb::kMergeTraceCtas) * kvb::kMergeTraceEvents;
  cudaError_t code =
      cudaMemcpyFromSymbol(out, kvb::g_merge_trace, std::min(count, all) * sizeof(unsigned long long));
  if (code != cudaSuccess) return code;
  static const unsigned long long zeros[kvb::kMergeTraceCtas][kvb::kMergeTraceEvents] = {};
  return cudaMemcpyToSymbol(kvb::g_merge_trace, zeros, sizeof(zeros));
#else
  (void)out;
  (void)count;
  *available = false;
  return cudaSuccess;
#endif
}

void fail_launch(unsigned nth, cudaError_t code) noexcept {
  t_fail_countdown = nth;
  t_fail_code = code == cudaSuccess ? cudaErrorLaunchFailure : code;
}

void skip_stage(unsigned stage) noexcept { t_skip_stage = stage; }

}  // namespace detail

// ---------------------------------------------------------------------------
// Decode call that allocates nothing (kvb_launch_attention_noalloc in
// include/kvbridge_c.h). Some callers cannot call cudaMalloc when they
// decode: an inference server whose memory pool reserved every byte of HBM
// up front for its KV cache, or a host whose decode path must not allocate.
// For them the split-K partials live in this file-scope device array instead
// of a caller-provided scratch buffer.
//
// Every GPU that loads the library holds the array (2 MiB) until process
// exit. All calls share it and it keeps the last call's contents; nothing in
// it needs to start at zero, because the partial kernel of a call writes
// every slot that call's merge reads. Calls that may run concurrently on the
// GPU (different streams) race on the array and must be serialised by the
// caller.

namespace {

constexpr size_t kNoAllocScratchFloats = size_t(1) << 19;  // 2 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Unique ID of the calling thread's current CUDA context (0 when there is
// none, or when the driver does not offer cuCtxGetId). IDs are never reused
// in a process, so the context that replaces a destroyed one (after
// cudaDeviceReset) has a new ID even if its handle value is reused.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static const std::pair<GetCurrent, GetId> fns = [] {
    void* cur = nullptr;
    void* id = nullptr;
    cudaDriverEntryPointQueryResult found{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &cur, cudaEnableDefault, &found) != cudaSuccess ||
        found != cudaDriverEntryPointSuccess)
      cur = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &id, cudaEnableDefault, &found) != cudaSuccess ||
        found != cudaDriverEntryPointSuccess)
      id = nullptr;
    return std::make_pair(reinterpret_cast<GetCurrent>(cur), reinterpret_cast<GetId>(id));
  }();
  if (fns.first == nullptr || fns.second == nullptr) return 0;
  CUcontext ctx = nullptr;
  if (fns.first(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (fns.second(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_noalloc_scratch in the current context. In host code
// the array's name is only a host-side stand-in, so the address is looked up
// with cudaGetSymbolAddress (with the device current) once per CUDA context
// and cached under the context's unique ID; a context created after
// cudaDeviceReset gets a fresh lookup. The first call in a context does the
// lookup, so it should come before any stream capture.
float* noalloc_scratch_in_current_context() {
  static std::mutex mu;
  static std::map<unsigned long long, float*> cache;
  std::lock_guard<std::mutex> lock(mu);
  const unsigned long long before = current_context_id();
  if (before != 0) {
    auto it = cache.find(before);
    if (it != cache.end()) return it->second;
  }
  void* ptr = nullptr;
  cuda_ok(cudaGetSymbolAddress(&ptr, g_noalloc_scratch), "cudaGetSymbolAddress(static scratch)");
  // The lookup makes the device's primary context current if none was.
  const unsigned long long id = current_context_id();
  if (id != 0) cache[id] = static_cast<float*>(ptr);
  return static_cast<float*>(ptr);
}

}  // namespace

namespace detail {

void launch_attention_noalloc(const Shape& s, const DeviceInput& in, unsigned partitions,
                              float* m, float* l, float* n, void* out_f16, cudaStream_t stream) {
  validate_shape(s);
  if (m == nullptr || l == nullptr || n == nullptr)
    throw std::invalid_argument("m, l and n must be non-null device buffers");
  check_inputs(s, in, m, m, l, n);  // input buffers; the scratch is internal
  if (!attention_b200_supported(s, in))
    throw std::invalid_argument(
        "the no-allocation call needs the tensor-core geometry (attention_b200_supported)");
  const size_t per_partition = size_t(s.rows) * s.q_heads * (size_t(s.dim) + 2);
  const size_t fit = kNoAllocScratchFloats / per_partition;
  if (fit == 0)
    throw std::invalid_argument(
        "rows * q_heads * (dim + 2) exceeds the 524288-float static scratch of the "
        "no-allocation call");
  uint32_t parts = attention_partitions(s, partitions);
  parts = uint32_t(std::min<size_t>(parts, fit));
  float* scratch = noalloc_scratch_in_current_context();
  if (parts > 0) {
    // Partials packed [row-head][partition]: split stride = parts. Same
    // kernel and launch as launch_attention_partials.
    launch_single_partials(s, in, parts, scratch, parts, stream);
  }
  launch_merge(kvb::kMergeScratch,
               scratch_merge_params(s, scratch, parts, parts, false, m, l, n, out_f16), stream);
}

}  // namespace detail

}  // namespace kvbridge
