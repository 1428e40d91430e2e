#pragma once
// Split-K partial kernel on the 5th-generation tensor cores (tcgen05, TMEM
// accumulators) for paged INT8 KV on sm_100a: single-sequence calls whose
// query columns per KV head (rows x group) are many (the reference's native
// 8 rows x group 6 = 48 columns), so that one CTA covers all of them and
// every K/V page crosses HBM and L2 once.
//
// Computes the partial (m, l, n[dim]) of each piece of the single-sequence
// split-K schedule (kvb_schedule.h) - the quantities of reference
// src/attention_shared.cu:42-209 and include/kvbridge/partial_attention_mma.
// cuh:153-477: s = scale * kscale * q.k over the visible tokens of the piece,
// m = max s, l = sum exp(s - m), n = sum exp(s - m) * vscale * v.
//
// Tiles of 128 tokens (two 64-token stages of the copy ring), per tile:
//   QK  S^T[token][n] = K[token][d] . Qd[n][d]        (tcgen05.mma kind::i8)
//       A = the K codes exactly as stored, 128 token rows, loaded by TMA in
//       the 128-byte-swizzled K-major layout; B = the query side as signed
//       int8 digits, row n = 3 c + k holding digit k of query column c
//       (q = d0 + 256 d1 + 65536 d2, a 22-bit fixed-point value per column
//       with a power-of-two scale). The s32 accumulator S^T lives in TMEM
//       with one lane per token, so all digits of a column land in one
//       thread.
//   softmax (4 NH warps; warp w takes the 32 tokens of TMEM lane quadrant
//       w % 4 and the query columns of half w / 4): scores in log2 units,
//       the tile's per-column max (warp shuffles + shared memory), online
//       rescale, and P = w * vscale as a signed 15-bit fixed-point value per
//       (tile, column) - the power-of-two scale is added to the exp2
//       argument - written as two signed int8 digits into P^T[n][token], the
//       B operand of PV.
//   PV  O^T[d][n] = V[d][token] . P^T[n][token]       (tcgen05.mma kind::i8)
//       A = the V codes exactly as stored (dim-major pages, loaded by TMA
//       as 64-byte rows in the 64-byte-swizzled K-major layout), 128 rows per
//       MMA; the s32 accumulator has one TMEM lane per dim (or dim pair).
//   fold (4 NH warps, one thread per dim and column half): O[d][c] =
//       O[d][c] * alpha_c + (lo + 256 hi) / pscale_c in fp32 registers.
// One warp issues the TMA copies into the ring, one owns TMEM and issues the
// MMAs from a single thread, taking QK and PV in whichever order their
// inputs become ready. Every hand-off is an mbarrier and every wait is
// bounded (kvb_device.cuh), so a broken pipeline reports a status instead of
// holding the GPU.
//
// Precision: QK is exact up to the 2^-22 (relative to the column's largest
// |q|) rounding of q; P is exact up to 2^-14 of the tile's bound on |P| per
// column; all digit products are exact s32 sums.
#include <cuda.h>

#include "decode_tma.cuh"
#include "kvb_device.cuh"

namespace kvb {

// Parameters: the single-sequence block of DecodeParams plus the tensor
// maps of the K pool (rows of `dim` bytes per (page, KV head, slot), boxes of
// 128 bytes x page_tokens rows, 128-byte swizzle) and of the V pool (rows of
// 64 bytes - one dim of a 64-token page or two dims of a 32-token page -
// boxes of 64 bytes x one page's rows, 64-byte swizzle).
struct DecodeParamsTc : DecodeParams {
  CUtensorMap tm_k, tm_v;
};

// Event timeline (trace builds only, -DKVB_TC_TRACE): SM clock stamps
// (clock64; one CTA runs on one SM, so differences within a CTA are exact) of
// the first kTraceCtas CTAs and kTraceTiles tiles of the last launch, read by
// the host with kvb_debug_read_tc_trace. Events per tile: see kTrace*.
constexpr uint32_t kTraceCtas = 16, kTraceTiles = 16, kTraceEvents = 18;
enum : uint32_t {
  kTraceStart = 0,       // tile 0 only: the CTA passed its setup barrier
  kTraceQkIssued = 1,    // MMA thread issued QK(t) (its stages had landed)
  kTraceSoftmaxIn = 2,   // softmax warp 0 saw S(t) ready
  kTraceSoftmaxOut = 3,  // softmax warp 0 published P(t)
  kTracePvIssued = 4,    // MMA thread issued PV(t)
  kTraceFoldIn = 5,      // fold warp 0 saw O(t) ready
  kTraceFoldOut = 6,     // fold warp 0 released O(t)
  kTraceCopyIssued = 7,  // producer armed the tile's first stage
  kTraceSmLoaded = 8,    // softmax warp 0 has S(t) in registers
  kTraceSmReduced = 9,   // softmax warp 0 passed the column-max barrier
  kTraceSmParams = 10,   // softmax warp 0 passed the column-parameter barrier
  kTracePReadySeen = 11,  // MMA thread first saw P(t) published by every softmax warp
  kTraceOFreeSeen = 12,   // MMA thread first saw O^T released for PV(t)
  kTraceVSeen = 13,       // MMA thread first saw V(t) landed
  kTraceSmStored = 14,    // softmax warp 0 finished its P digit stores (before the proxy fence)
  kTracePGroup = 15,      // + g (g < 3): softmax warp 0 finished the P digits of column group g (4 columns)
};
#ifdef KVB_TC_TRACE
__device__ unsigned long long g_tc_trace[kTraceCtas][kTraceTiles][kTraceEvents];
#define KVB_TC_MARK(tile, event)                                                    \
  do {                                                                              \
    if (blockIdx.x < kTraceCtas && (tile) < kTraceTiles)                            \
      g_tc_trace[blockIdx.x][(tile)][(event)] = clock64();                          \
  } while (0)
#else
#define KVB_TC_MARK(tile, event) \
  do {                           \
  } while (0)
#endif

// Shared-memory layout (byte offsets; the dynamic shared memory base is
// rounded up to 1024 bytes first) and warp roles. NC query columns per KV
// head, split into NH halves between the softmax (and fold) warp groups; the
// QK MMA has N = 3 NC (query digits), the PV MMA N = 2 NC (P digits), each
// rounded up to a multiple of 16. K and V stages have rings of their own
// (SLOTS 64-token slots each; a K slot is free once QK has read it, a V slot
// once PV has), and the K/V scales a ring twice as deep, freed once the
// softmax warps have read them.
template <int D, int P, int NC, int SLOTS, int NH>
struct TcSmem {
  static constexpr uint32_t kCH = NC / NH;  // columns per softmax / fold thread
  static constexpr uint32_t kSoftmaxWarps = 4 * NH;
  static constexpr uint32_t kFoldWarps = 4 * NH;
  static constexpr uint32_t kProducerKWarp = 8 * NH;
  static constexpr uint32_t kMmaWarp = 8 * NH + 1;
  static constexpr uint32_t kProducerVWarp = 8 * NH + 2;
  static constexpr uint32_t kWarps = 8 * NH + 3;
  static constexpr uint32_t kThreads = 32 * kWarps;
  // Registers are split between the SM's four sub-partitions (16K each) and
  // the warps are spread over them round-robin.
  static constexpr uint32_t kWarpsPerSubpartition = (kWarps + 3) / 4;
  static constexpr uint32_t kMaxRegs = (16384 / (32 * kWarpsPerSubpartition)) / 8 * 8;
  static constexpr uint32_t kNQK = (3 * NC + 15) / 16 * 16;
  static constexpr uint32_t kNPV = (2 * NC + 15) / 16 * 16;
  static constexpr uint32_t kScaleSlots = 2 * SLOTS;
  static constexpr uint32_t kChunks = D / 128;             // 128-byte K chunks of a K row
  static constexpr uint32_t kKChunkBytes = SLOTS * 8192u;  // one chunk of every slot (64 rows)
  static constexpr uint32_t kOffK = 0;
  static constexpr uint32_t kOffV = kOffK + kChunks * kKChunkBytes;
  static constexpr uint32_t kVSlotBytes = 64u * D;
  // V pages are loaded as rows of 64 bytes (64-byte swizzle): with 32-token
  // pages a row holds two dims (2i: bytes 0-31, 2i + 1: bytes 32-63), which
  // halves the TMA rows per page; the PV MMA reads the even dims at K offset
  // 0 and the odd dims at K offset 32 into two accumulator regions.
  static constexpr bool kVPair = P == 32;
  static constexpr uint32_t kVRows = kVPair ? D / 2 : D;  // 64-byte rows per page
  static constexpr uint32_t kOffScales = kOffV + SLOTS * kVSlotBytes;  // [scale slot][k|v][64] floats
  static constexpr uint32_t kOffQ = (kOffScales + kScaleSlots * 512u + 1023u) / 1024u * 1024u;
  static constexpr uint32_t kQBytes = kChunks * kNQK * 128u;
  static constexpr uint32_t kPBufBytes = kNPV * 128u;  // [8 token chunks][kNPV rows][16 B]
  static constexpr uint32_t kOffP = kOffQ + kQBytes;
  static constexpr uint32_t kOffStats = kOffP + 2 * kPBufBytes;  // [2][NC][alpha, 1/pscale] (fold)
  static constexpr uint32_t kOffColP = kOffStats + 2 * NC * 8;   // [2][NC] float4 {cf, off, inv, alpha}
  static constexpr uint32_t kOffRed = kOffColP + 2 * NC * 16;    // [2][softmax warps][32]
  // qpos[NC] (int64), then cf[NC] and the running max m[2][NC] (float)
  static constexpr uint32_t kOffCol = kOffRed + 2 * kSoftmaxWarps * 32 * 4;
  static constexpr uint32_t kOffBar = (kOffCol + NC * 8 + NC * 4 + 2 * NC * 4 + 7) / 8 * 8;
  // barriers: full_k[SLOTS], empty_k[SLOTS], full_v[SLOTS], empty_v[SLOTS],
  // empty_s[2 SLOTS], s_ready[2], s_free[2], p_ready[2], p_free[2],
  // stats_free[2], o_ready, o_free, mma_done
  static constexpr uint32_t kBars = 6 * SLOTS + 10 + 3;
  static constexpr uint32_t kOffMisc = kOffBar + kBars * 8;  // tmem address, abort flag
  static constexpr uint32_t kBytes = kOffMisc + 64;
  static constexpr uint32_t kDynamicBytes = kBytes + 1024;  // room to align the base
  // TMEM columns: S^T[2] (kNQK each) and O^T[D / 128] (kNPV each), regions
  // rounded to 32 columns.
  static constexpr uint32_t kRegionS = (kNQK + 31) / 32 * 32;
  static constexpr uint32_t kRegionO = (kNPV + 31) / 32 * 32;
  static constexpr uint32_t kTmemUsed = 2 * kRegionS + (D / 128) * kRegionO;
  static constexpr uint32_t kTmemCols = kTmemUsed <= 32 ? 32 : kTmemUsed <= 64 ? 64 : kTmemUsed <= 128 ? 128
                                        : kTmemUsed <= 256 ? 256 : 512;
  static_assert(kTmemUsed <= 512, "TMEM columns");
  static_assert(NC % (8 * NH) == 0 && kCH < 32 && kNQK <= 256, "columns: whole 8-column chunks per half");
  static_assert(SLOTS % 2 == 0, "tiles are slot pairs");
  static_assert((P == 32 && D == 256) || P == 64, "V view: dim-paired 32-token pages at dim 256, or 64-token pages");
};

template <int D, int P, int NC, int SLOTS, int NH>
__global__ void __maxnreg__((TcSmem<D, P, NC, SLOTS, NH>::kMaxRegs))
    decode_partial_tc_kernel(const __grid_constant__ DecodeParamsTc p) {
  using L = TcSmem<D, P, NC, SLOTS, NH>;
  constexpr uint32_t NQK = L::kNQK, NPV = L::kNPV, CH = L::kCH, SS = L::kScaleSlots;
  constexpr uint32_t kPps = 64 / P;  // pages per 64-token stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* full_k = bars;
  uint64_t* empty_k = bars + SLOTS;
  uint64_t* full_v = bars + 2 * SLOTS;
  uint64_t* empty_v = bars + 3 * SLOTS;
  uint64_t* empty_s = bars + 4 * SLOTS;  // SS of them
  uint64_t* s_ready = bars + 6 * SLOTS;
  uint64_t* s_free = s_ready + 2;
  uint64_t* p_ready = s_ready + 4;
  uint64_t* p_free = s_ready + 6;
  uint64_t* stats_free = s_ready + 8;
  uint64_t* o_ready = s_ready + 10;
  uint64_t* o_free = s_ready + 11;
  uint64_t* mma_done = s_ready + 12;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile uint32_t* tmem_holder = misc;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  int64_t* col_qpos = reinterpret_cast<int64_t*>(smem + L::kOffCol);
  float* col_cf = reinterpret_cast<float*>(smem + L::kOffCol + NC * 8);
  // Running max per column (log2 units), double-buffered by tile parity: tile
  // t reads buffer (t + 1) & 1 and writes buffer t & 1.
  float* col_m = col_cf + NC;
  float* stats = reinterpret_cast<float*>(smem + L::kOffStats);
  float4* colp = reinterpret_cast<float4*>(smem + L::kOffColP);
  float* red = reinterpret_cast<float*>(smem + L::kOffRed);

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned long long limit_ns = p.wait_limit_ns;
  auto wait = [&](uint64_t* bar, uint32_t parity, int code, int stage) {
    return mbar_wait_bounded(bar, parity, abort_flag, code, stage, limit_ns) == kWaitOk;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < SLOTS; ++s) {
      mbar_init(&full_k[s], 1);
      mbar_init(&empty_k[s], 1);
      mbar_init(&full_v[s], 1);
      mbar_init(&empty_v[s], 1);
    }
    for (int s = 0; s < int(SS); ++s) mbar_init(&empty_s[s], L::kSoftmaxWarps);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_ready[b], 1);
      mbar_init(&s_free[b], L::kSoftmaxWarps);
      mbar_init(&p_ready[b], L::kSoftmaxWarps);
      mbar_init(&p_free[b], 1);
      mbar_init(&stats_free[b], L::kFoldWarps);
    }
    mbar_init(o_ready, 1);
    mbar_init(o_free, L::kFoldWarps);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == L::kProducerKWarp && lane == 0) tc::prefetch_tmap(&p.tm_k);
  if (warp == L::kProducerVWarp && lane == 0) tc::prefetch_tmap(&p.tm_v);
  if (warp == L::kMmaWarp) {
    tc::tmem_alloc(const_cast<uint32_t*>(tmem_holder), L::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const uint32_t tm_s[2] = {tmem, tmem + L::kRegionS};
  const uint32_t tm_o = tmem + 2 * L::kRegionS;

  const Piece pc = single_piece(p, blockIdx.x);
  const uint32_t first_stage = pc.lo / kStageTokens;
  const uint32_t nstages = pc.j1 - pc.j0;
  const uint32_t ntiles = (nstages + 1) / 2;
  const uint32_t cols = p.qr;  // <= NC
  grid_dependency_wait();
  if (threadIdx.x == 0) KVB_TC_MARK(0u, kTraceStart);

  if (warp == L::kProducerKWarp || warp == L::kProducerVWarp) {
    // ---- TMA producers: stage g of the piece goes to K (or V) slot
    // g % SLOTS and, with its scales, to scale slot g % (2 SLOTS).
    const bool kside = warp == L::kProducerKWarp;
    const uint64_t policy = l2_evict_first_policy();
    const uint32_t page_lo = max(pc.lo, (first_stage + pc.j0) * kStageTokens) / P;
    const uint32_t page_hi = (min(pc.hi, (first_stage + pc.j1) * kStageTokens) - 1) / P;
    uint64_t* full = kside ? full_k : full_v;
    uint64_t* empty = kside ? empty_k : empty_v;
    uint32_t g = 0;
    bool failed = false;
    for (; g < nstages && !failed; ++g) {
      const uint32_t slot = g % SLOTS, use = g / SLOTS;
      if (!wait(&empty[slot], (use & 1u) ^ 1u, kStatusEmptyWaitTimeout, int(g)) ||
          (kside && !wait(&empty_s[g % SS], ((g / SS) & 1u) ^ 1u, kStatusEmptyWaitTimeout, int(g)))) {
        failed = true;
        break;
      }
      // Lane q < kPps handles page q of the stage.
      const uint32_t pg = (first_stage + pc.j0 + g) * kPps + lane;
      const bool mine = lane < kPps && pg >= page_lo && pg <= page_hi;
      const uint32_t phys = mine ? __ldg(p.table + pg) : 0u;
      const bool ok = mine && phys < p.pages;
      if (kside && __ballot_sync(0xffffffffu, mine && !ok) && lane == 0) atomicMax(&g_kvb_status, kStatusBadPage);
      const uint32_t nok = __popc(__ballot_sync(0xffffffffu, ok));
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[slot], nok * (kside ? P * D + 8u * P : P * D));
        if (kside && (g & 1u) == 0) KVB_TC_MARK(g / 2, kTraceCopyIssued);
      }
      __syncwarp();
      if (ok) {
        const uint32_t unit = phys * p.kv_heads + pc.h;  // < 2^32 / (P * D): 32-bit extent
        if (kside) {
          for (uint32_t c = 0; c < L::kChunks; ++c)
            tc::tma_load_2d(smem + L::kOffK + c * L::kKChunkBytes + slot * 8192u + lane * P * 128u, &p.tm_k,
                            int32_t(c * 128u), int32_t(unit * P), &full[slot], policy);
          float* sc = reinterpret_cast<float*>(smem + L::kOffScales + (g % SS) * 512u);
          bulk_copy_g2s(sc + lane * P, p.k_scales + size_t(unit) * P, 4 * P, &full[slot], policy);
          bulk_copy_g2s(sc + 64 + lane * P, p.v_scales + size_t(unit) * P, 4 * P, &full[slot], policy);
        } else {
          tc::tma_load_2d(smem + L::kOffV + slot * L::kVSlotBytes + lane * P * D, &p.tm_v, 0,
                          int32_t(unit * L::kVRows), &full[slot], policy);
        }
      }
    }
    if (kside && !failed) mark_empty_splits<D>(p, pc);
    // Drain: copies of the last SLOTS stages may still be in flight.
    for (uint32_t s = g > SLOTS ? g - SLOTS : 0u; s < g; ++s) {
      volatile int no_abort = 0;
      if (mbar_wait_bounded(&full[s % SLOTS], (s / SLOTS) & 1u, &no_abort, kStatusDrainTimeout, int(s),
                            limit_ns) != kWaitOk)
        break;
    }
  } else if (warp == L::kMmaWarp) {
    // ---- MMA issuer (one thread): QK of tile qk once its stages have landed
    // and its S buffer is free, PV of tile pv once its P digits are written
    // and O^T has been read - in whichever order they become ready, so that
    // a tile's PV never waits behind the next tile's copies. Waits first for
    // the query digits.
    named_barrier(1, 32 * (L::kSoftmaxWarps + L::kFoldWarps + 1));
    if (lane == 0) {
      tc::fence_after_sync();
      constexpr uint32_t kIdescQk = tc::idesc_i8(128, NQK);
      constexpr uint32_t kIdescPv = tc::idesc_i8(128, NPV);
      uint32_t qk = 0, pv = 0, spins = 0;
#ifdef KVB_TC_TRACE
      uint32_t seen = 0;  // which PV inputs of tile pv were seen ready (trace only)
#endif
      unsigned long long idle_since = 0;
      while (pv < ntiles) {
        bool progressed = false;
        if (qk < ntiles) {
          const uint32_t b = qk & 1u, s0 = 2 * qk, nst = min(2u, nstages - s0);
          bool ready = mbar_test(&s_free[b], ((qk >> 1) & 1u) ^ 1u);
          for (uint32_t si = 0; si < nst && ready; ++si)
            ready = mbar_test(&full_k[(s0 + si) % SLOTS], ((s0 + si) / SLOTS) & 1u);
          if (ready) {
            tc::fence_after_sync();
            // 128 token rows: slots s0 and s0 + 1 are adjacent in every K
            // chunk (s0 and SLOTS are even, so a pair never wraps).
            const uint32_t slot0 = s0 % SLOTS;
            for (uint32_t c = 0; c < L::kChunks; ++c)
              for (uint32_t kk = 0; kk < 4; ++kk) {
                const uint64_t a = tc::smem_desc(smem + L::kOffK + c * L::kKChunkBytes + slot0 * 8192u + kk * 32u,
                                                 16u, 1024u, tc::kSwizzle128);
                const uint64_t bq = tc::smem_desc(smem + L::kOffQ + c * NQK * 128u + kk * 32u, 16u, 1024u,
                                                  tc::kSwizzle128);
                tc::mma_i8(tm_s[b], a, bq, kIdescQk, c != 0 || kk != 0);
              }
            tc::commit(&s_ready[b]);
            for (uint32_t si = 0; si < nst; ++si) tc::commit(&empty_k[(s0 + si) % SLOTS]);
            KVB_TC_MARK(qk, kTraceQkIssued);
            ++qk;
            progressed = true;
          }
        }
        if (pv < qk) {
          const uint32_t b = pv & 1u;
          const uint32_t s0 = 2 * pv, nst = min(2u, nstages - s0);
          const bool p_in = mbar_test(&p_ready[b], (pv >> 1) & 1u);
          const bool o_in = mbar_test(o_free, (pv & 1u) ^ 1u);
          bool v_in = true;
          for (uint32_t si = 0; si < nst && v_in; ++si)
            v_in = mbar_test(&full_v[(s0 + si) % SLOTS], ((s0 + si) / SLOTS) & 1u);
#ifdef KVB_TC_TRACE
          if (p_in && !(seen & 1u)) KVB_TC_MARK(pv, kTracePReadySeen);
          if (o_in && !(seen & 2u)) KVB_TC_MARK(pv, kTraceOFreeSeen);
          if (v_in && !(seen & 4u)) KVB_TC_MARK(pv, kTraceVSeen);
          seen |= (p_in ? 1u : 0u) | (o_in ? 2u : 0u) | (v_in ? 4u : 0u);
#endif
          const bool ready = p_in && o_in && v_in;
          if (ready) {
            tc::fence_after_sync();
            const uint8_t* pbuf = smem + L::kOffP + b * L::kPBufBytes;
            for (uint32_t h = 0; h < D / 128; ++h) {
              bool acc = false;
              for (uint32_t si = 0; si < nst; ++si) {
                const uint8_t* vslot = smem + L::kOffV + ((s0 + si) % SLOTS) * L::kVSlotBytes;
                for (uint32_t pg = 0; pg < kPps; ++pg)
                  for (uint32_t kk = 0; kk < P / 32; ++kk) {
                    // Region h: dims 2i + h (dim-paired pages) or 128 h + i.
                    const uint32_t off = L::kVPair ? h * 32u : h * 128u * 64u + kk * 32u;
                    const uint64_t a = tc::smem_desc(vslot + pg * P * D + off, 16u, 512u, tc::kSwizzle64);
                    const uint32_t tok = si * 64u + pg * P + kk * 32u;  // token offset in the tile
                    const uint64_t bd = tc::smem_desc(pbuf + (tok / 16u) * (NPV * 16u), NPV * 16u, 128u,
                                                      tc::kSwizzleNone);
                    tc::mma_i8(tm_o + h * L::kRegionO, a, bd, kIdescPv, acc);
                    acc = true;
                  }
              }
            }
            tc::commit(o_ready);
            tc::commit(&p_free[b]);
            for (uint32_t si = 0; si < nst; ++si) tc::commit(&empty_v[(s0 + si) % SLOTS]);
            KVB_TC_MARK(pv, kTracePvIssued);
#ifdef KVB_TC_TRACE
            seen = 0;
#endif
            ++pv;
            progressed = true;
          }
        }
        if (progressed) {
          spins = 0;
          idle_since = 0;
          continue;
        }
        // Idle: back off briefly, so that the poll does not take issue slots
        // from the softmax and fold warps of this SM sub-partition.
        __nanosleep(64);
        if ((++spins & 63u) == 0) {
          if (*abort_flag) break;
          const unsigned long long now = global_ns();
          if (idle_since == 0) {
            idle_since = now;
          } else if (now - idle_since > limit_ns) {
            *abort_flag = 1;
            record_wait_failure(kStatusFullWaitTimeout, int(2 * pv), static_cast<long long>(now - idle_since), 0);
            break;
          }
        }
      }
      tc::commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait_bounded(mma_done, 0, &no_abort, kStatusDrainTimeout, -1, limit_ns);
    }
    __syncwarp();
  } else {
    // ---- query digits (softmax and fold warps): rows n = 3c + k of the QK B
    // operand in the 128-byte-swizzled K-major layout [chunk][NQK rows][128 B].
    // Rows past 3 NC only feed TMEM columns that nothing reads.
    uint8_t* qt = smem + L::kOffQ;
    constexpr uint32_t kComputeWarps = L::kSoftmaxWarps + L::kFoldWarps;
    constexpr uint32_t kColsPerWarp = (NC + kComputeWarps - 1) / kComputeWarps;
    constexpr uint32_t kPer = D / 32;  // dims per lane, contiguous
    // Every load of the warp's query rows is issued before any is used.
    float4 qv[kColsPerWarp][kPer / 4];
#pragma unroll
    for (uint32_t k = 0; k < kColsPerWarp; ++k) {
      const uint32_t c = warp + k * kComputeWarps;
      const bool valid = c < cols;
      const uint32_t r = valid ? c / p.group : 0, gq = valid ? c % p.group : 0;
      const float* qrow = p.q + (size_t(r) * p.q_heads + size_t(pc.h) * p.group + gq) * D + lane * kPer;
#pragma unroll
      for (uint32_t i = 0; i < kPer / 4; ++i)
        qv[k][i] = valid ? __ldg(reinterpret_cast<const float4*>(qrow) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (uint32_t k = 0; k < kColsPerWarp; ++k) {
      const uint32_t c = warp + k * kComputeWarps;
      if (c >= NC) break;
      const bool valid = c < cols;
      const uint32_t r = valid ? c / p.group : 0;
      float v[kPer];
#pragma unroll
      for (uint32_t i = 0; i < kPer / 4; ++i) {
        v[4 * i] = qv[k][i].x;
        v[4 * i + 1] = qv[k][i].y;
        v[4 * i + 2] = qv[k][i].z;
        v[4 * i + 3] = qv[k][i].w;
      }
      float amax = 0.f;
#pragma unroll
      for (uint32_t i = 0; i < kPer; ++i) amax = fmaxf(amax, fabsf(v[i]));
      amax = warp_max(amax);
      // 2^e > max|q|; q * 2^(22-e) rounds to an integer of magnitude < 2^22,
      // split into signed base-256 digits d0, d1 in [-128, 127], |d2| <= 64.
      int e = 0;
      if (amax > 0.f) e = int((__float_as_uint(amax) >> 23) & 0xffu) - 126;
      e = max(-100, min(100, e));
      const float up = __uint_as_float(uint32_t(127 + 22 - e) << 23);
      uint32_t dg[3][kPer / 4];
#pragma unroll
      for (uint32_t i = 0; i < kPer; i += 4) {
        uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          const int qi = __float2int_rn(v[i + j] * up);
          const int l0 = ((qi + 128) & 255) - 128;
          const int t1 = (qi - l0) >> 8;
          const int l1 = ((t1 + 128) & 255) - 128;
          const int l2 = (t1 - l1) >> 8;
          w0 |= (uint32_t(l0) & 0xffu) << (8 * j);
          w1 |= (uint32_t(l1) & 0xffu) << (8 * j);
          w2 |= (uint32_t(l2) & 0xffu) << (8 * j);
        }
        dg[0][i / 4] = w0;
        dg[1][i / 4] = w1;
        dg[2][i / 4] = w2;
      }
      // Dims lane*kPer .. +kPer-1 sit in one 16-byte unit of one chunk.
      const uint32_t d = lane * kPer;
      const uint32_t chunk = d / 128, b = d % 128, unit = b / 16;
#pragma unroll
      for (uint32_t k = 0; k < 3; ++k) {
        const uint32_t n = 3 * c + k;
        uint8_t* dst = qt + chunk * NQK * 128u + n * 128u + (((unit ^ (n & 7u)) << 4) | (b & 15u));
        if (kPer == 8)
          *reinterpret_cast<uint2*>(dst) = make_uint2(dg[k][0], dg[k][kPer / 4 - 1]);
        else
          *reinterpret_cast<uint32_t*>(dst) = dg[k][0];
      }
      if (lane == 0) {
        col_cf[c] = p.score_scale * kLog2e * __uint_as_float(uint32_t(127 + e - 22) << 23);
        col_qpos[c] = valid ? __ldg(p.q_positions + r) : INT64_MAX;
        col_m[c] = -INFINITY;
        col_m[NC + c] = -INFINITY;
      }
    }
    tc::fence_proxy_async_smem();
    named_barrier(1, 32 * (L::kSoftmaxWarps + L::kFoldWarps + 1));

    if (warp < L::kSoftmaxWarps) {
      // ---- softmax: warp w = lane quadrant w % 4 (tokens r = 32 (w % 4) +
      // lane of the tile) x column half w / 4 (columns cbase .. cbase + CH).
      const uint32_t qd = warp & 3u, hh = warp >> 2;
      const uint32_t r = 32 * qd + lane;
      const uint32_t cbase = hh * CH;
      const uint32_t lane_base = (32 * qd) << 16;
      // Whole-piece visibility: k_positions is nondecreasing, so the piece's
      // last token decides.
      int64_t qmin = INT64_MAX;
      for (uint32_t c = 0; c < cols; ++c) qmin = min(qmin, col_qpos[c]);
      const uint32_t last = min(pc.hi, (first_stage + pc.j1) * kStageTokens) - 1;
      const bool all_visible = nstages == 0 || __ldg(p.k_positions + last) <= qmin;
      float lp[CH];  // this thread's share of l per column
#pragma unroll
      for (uint32_t j = 0; j < CH; ++j) lp[j] = 0.f;
      // Every warp runs every tile and every named barrier, also after a
      // failed wait (the waits then return at once and the data is unused),
      // so that no warp is left alone at a barrier.
      for (uint32_t t = 0; t < ntiles; ++t) {
        const uint32_t b = t & 1u;
        const bool got = wait(&s_ready[b], (t >> 1) & 1u, kStatusFullWaitTimeout, int(2 * t));
        if (threadIdx.x == 0) KVB_TC_MARK(t, kTraceSoftmaxIn);
        tc::fence_after_sync();
        // Columns 3c + k of S^T hold digit k's dot of query column c (exact
        // s32, each below 2^22 in magnitude): x = dot0 + 256 dot1 + 65536
        // dot2, then scaled by the token's K scale. Each dot becomes a float
        // exactly without the conversion pipe: the bits of 1.5 * 2^23 + i
        // are 0x4B400000 + i for |i| < 2^22, and subtracting 1.5 * 2^23 is
        // exact.
        float x[CH];
#pragma unroll
        for (uint32_t c8 = 0; c8 < CH; c8 += 8) {
          uint32_t r0[8], r1[8], r2[8];
          const uint32_t col = tm_s[b] + lane_base + 3 * (cbase + c8);
          tc::tmem_ld<8>(col, r0);
          tc::tmem_ld<8>(col + 8, r1);
          tc::tmem_ld<8>(col + 16, r2);
          tc::tmem_ld_wait();
          const uint32_t* raw[3] = {r0, r1, r2};
#pragma unroll
          for (uint32_t j = 0; j < 8; ++j) {
            constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
            const float f0 = __uint_as_float(raw[(3 * j) / 8][(3 * j) % 8] + 0x4B400000u) - kRound;
            const float f1 = __uint_as_float(raw[(3 * j + 1) / 8][(3 * j + 1) % 8] + 0x4B400000u) - kRound;
            const float f2 = __uint_as_float(raw[(3 * j + 2) / 8][(3 * j + 2) % 8] + 0x4B400000u) - kRound;
            x[c8 + j] = fmaf(f2, 65536.f, fmaf(f1, 256.f, f0));
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[b]);
        if (threadIdx.x == 0) KVB_TC_MARK(t, kTraceSmLoaded);
        // This thread's token, its scales (then the scale slots are released).
        const uint32_t s0 = 2 * t, nst = min(2u, nstages - s0);
        const uint32_t tok = (first_stage + pc.j0 + s0) * kStageTokens + r;
        const float* sc = reinterpret_cast<const float*>(smem + L::kOffScales + ((s0 + (r >> 6)) % SS) * 512u);
        const bool in_piece = got && (s0 + (r >> 6)) < nstages && tok >= pc.lo && tok < pc.hi;
        const float ks = in_piece ? sc[r & 63] : 0.f;
        const float vs = in_piece ? sc[64 + (r & 63)] : 0.f;
        __syncwarp();
        if (lane == 0)
          for (uint32_t si = 0; si < nst; ++si) mbar_arrive(&empty_s[(s0 + si) % SS]);
        if (all_visible) {
#pragma unroll
          for (uint32_t j = 0; j < CH; ++j) x[j] = in_piece ? x[j] * ks : -INFINITY;
        } else {
          const int64_t kp = in_piece ? __ldg(p.k_positions + tok) : INT64_MAX;
#pragma unroll
          for (uint32_t j = 0; j < CH; ++j)
            x[j] = (in_piece && kp <= col_qpos[cbase + j]) ? x[j] * ks : -INFINITY;
        }
        // Warp max of every column (and of |vscale|) by reduce-scatter: after
        // the five exchange steps lane j holds column j's max over the
        // warp's 32 tokens (j = CH: the max |vscale|).
        float v[16];
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) {
          const float lo_v = i < CH ? x[i] : (i == CH ? fabsf(vs) : -INFINITY);
          const float hi_v = i + 16 < CH ? x[i + 16] : (i + 16 == CH ? fabsf(vs) : -INFINITY);
          const bool up = lane & 16u;
          const float send = up ? lo_v : hi_v, keep = up ? hi_v : lo_v;
          v[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 16));
        }
#pragma unroll
        for (uint32_t w = 8; w >= 1; w >>= 1) {
          const bool up = lane & w;
#pragma unroll
          for (uint32_t i = 0; i < w; ++i) {
            const float send = up ? v[i] : v[i + w], keep = up ? v[i + w] : v[i];
            v[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, w));
          }
        }
        float* rw = red + b * (L::kSoftmaxWarps * 32);
        rw[warp * 32 + lane] = v[0];
        named_barrier(2, 32 * L::kSoftmaxWarps);
        if (threadIdx.x == 0) KVB_TC_MARK(t, kTraceSmReduced);
        // Per-column scalars, once per column (lane j of the half's first
        // quadrant warp): the tile max score tm, the new running max, alpha,
        // and the power of two 2^sh that puts |P| <= exp2(tm - mnew) * vsmax
        // in [2^13, 2^14) (kept a normal float); published as {cf, sh - msub,
        // 2^-sh, alpha} for every thread, and {alpha, 1/pscale} for the fold.
        if (qd == 0 && lane < CH) {
          const uint32_t c = cbase + lane;
          float tx = rw[(4 * hh) * 32 + lane], vsmax = rw[(4 * hh) * 32 + CH];
#pragma unroll
          for (uint32_t w = 1; w < 4; ++w) {
            tx = fmaxf(tx, rw[(4 * hh + w) * 32 + lane]);
            vsmax = fmaxf(vsmax, rw[(4 * hh + w) * 32 + CH]);
          }
          const float cf = col_cf[c];
          const float tm = tx * cf;  // -inf when no token of the tile is visible
          const float mo = col_m[((t + 1) & 1u) * NC + c];
          const float mnew = fmaxf(mo, tm);
          const float msub = mnew == -INFINITY ? 0.f : mnew;
          const float alpha = mnew == -INFINITY ? 1.f : fast_exp2(mo - msub);
          const float bound = (tm == -INFINITY ? 0.f : fast_exp2(tm - msub)) * vsmax;
          const int xb = int((__float_as_uint(bound) >> 23) & 0xffu);
          const int sh = max(-126, min(126, 140 - xb));
          const float inv = __uint_as_float(uint32_t(127 - sh) << 23);  // 2^-sh
          colp[b * NC + c] = make_float4(cf, float(sh) - msub, inv, alpha);
          col_m[b * NC + c] = mnew;
          if (wait(&stats_free[b], ((t >> 1) & 1u) ^ 1u, kStatusFullWaitTimeout, int(2 * t))) {
            stats[(b * NC + c) * 2] = alpha;
            stats[(b * NC + c) * 2 + 1] = bound > 0.f ? inv : 1.f;
          }
        }
        const bool room = wait(&p_free[b], ((t >> 1) & 1u) ^ 1u, kStatusFullWaitTimeout, int(2 * t));
        named_barrier(2, 32 * L::kSoftmaxWarps);
        if (threadIdx.x == 0) KVB_TC_MARK(t, kTraceSmParams);
        // P digits of this token: row 2c = low digit, 2c + 1 = high digit of
        // u = rint(w vscale 2^sh), |u| < 2^14: the low byte of u, and
        // (u + 128) >> 8. fma(wp, vs, 1.5 * 2^23) rounds the product to the
        // nearest integer (ties to even) in the low mantissa bits, whose bits
        // are 0x4B400000 + u.
        // Groups of four columns: their parameters are loaded before any of
        // the group's digit stores, so that the loads are not held behind
        // stores the compiler cannot prove disjoint.
        uint8_t* pt = smem + L::kOffP + b * L::kPBufBytes + (r / 16u) * (NPV * 16u) + (r & 15u);
#pragma unroll
        for (uint32_t j4 = 0; j4 < CH; j4 += 4) {
          float4 cp[4];
#pragma unroll
          for (uint32_t i = 0; i < 4; ++i) cp[i] = colp[b * NC + cbase + j4 + i];
          int ub[4];
#pragma unroll
          for (uint32_t i = 0; i < 4; ++i) {
            const float wp = fast_exp2(fmaf(x[j4 + i], cp[i].x, cp[i].y));  // w * 2^sh; 0 where x = -inf
            lp[j4 + i] = fmaf(wp, cp[i].z, lp[j4 + i] * cp[i].w);
            ub[i] = int(__float_as_uint(fmaf(wp, vs, 12582912.0f)));  // 0x4B400000 + u
          }
          if (room) {
#pragma unroll
            for (uint32_t i = 0; i < 4; ++i) {
              const uint32_t c = cbase + j4 + i;
              pt[(2 * c) * 16u] = uint8_t(ub[i]);
              pt[(2 * c + 1) * 16u] = uint8_t((ub[i] - int(0x4B400000u) + 128) >> 8);
            }
          }
          if (threadIdx.x == 0 && j4 / 4 < 3) KVB_TC_MARK(t, kTracePGroup + j4 / 4);
        }
        if (threadIdx.x == 0) KVB_TC_MARK(t, kTraceSmStored);
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_ready[b]);
        if (threadIdx.x == 0) KVB_TC_MARK(t, kTraceSoftmaxOut);
      }
      // l over the 128 tokens (the four quadrant warps of the half), then one
      // (m, l) per query column.
      named_barrier(2, 32 * L::kSoftmaxWarps);
      float* rw = red;
#pragma unroll
      for (uint32_t j = 0; j < CH; ++j) {
        const float sum = warp_sum(lp[j]);
        if (lane == 0) rw[warp * 32 + j] = sum;
      }
      named_barrier(2, 32 * L::kSoftmaxWarps);
      if (qd == 0 && lane < CH && cbase + lane < cols) {
        const uint32_t j = lane, c = cbase + lane;
        float lsum = 0.f;
#pragma unroll
        for (uint32_t w = 0; w < 4; ++w) lsum += rw[(4 * hh + w) * 32 + j];
        const float mr = col_m[((ntiles + 1) & 1u) * NC + c];  // written in the last tile
        const uint32_t row = c / p.group, gq = c % p.group;
        const size_t rh = size_t(row) * p.q_heads + size_t(pc.h) * p.group + gq;
        float* out = p.part + (rh * p.split_stride + pc.slot) * (D + 2);
        out[0] = (mr == -INFINITY || lsum == 0.f) ? -INFINITY : mr * kLn2;
        out[1] = lsum;
      }
    } else {
      // ---- fold: warp 4 NH + w = lane quadrant w % 4 (TMEM lane dl = 32
      // (w % 4) + lane: dims 2 dl + h with dim-paired pages, else 128 h + dl)
      // x column half w / 4.
      const uint32_t fw = warp - L::kSoftmaxWarps;
      const uint32_t qd = fw & 3u, hh = fw >> 2;
      const uint32_t dl = 32 * qd + lane;
      const uint32_t cbase = hh * CH;
      const uint32_t lane_base = (32 * qd) << 16;
      float acc[D / 128][CH];
#pragma unroll
      for (uint32_t h = 0; h < D / 128; ++h)
#pragma unroll
        for (uint32_t j = 0; j < CH; ++j) acc[h][j] = 0.f;
      for (uint32_t t = 0; t < ntiles; ++t) {
        const uint32_t b = t & 1u;
        if (!wait(o_ready, t & 1u, kStatusFullWaitTimeout, int(2 * t)) ||
            !wait(&p_ready[b], (t >> 1) & 1u, kStatusFullWaitTimeout, int(2 * t)))
          break;
        if (fw == 0 && lane == 0) KVB_TC_MARK(t, kTraceFoldIn);
        tc::fence_after_sync();
        const float* st = stats + b * NC * 2;
#pragma unroll
        for (uint32_t h = 0; h < D / 128; ++h) {
#pragma unroll
          for (uint32_t c8 = 0; c8 < CH; c8 += 8) {
            uint32_t raw[16];
            tc::tmem_ld<16>(tm_o + h * L::kRegionO + lane_base + 2 * (cbase + c8), raw);
            tc::tmem_ld_wait();
#pragma unroll
            for (uint32_t j = 0; j < 8; ++j) {
              const uint32_t c = cbase + c8 + j;
              const float sum = float(int(raw[2 * j + 1]) * 256 + int(raw[2 * j]));
              acc[h][c8 + j] = fmaf(sum, st[2 * c + 1], acc[h][c8 + j] * st[2 * c]);
            }
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(o_free);
          mbar_arrive(&stats_free[b]);
          if (fw == 0) KVB_TC_MARK(t, kTraceFoldOut);
        }
      }
#pragma unroll
      for (uint32_t j = 0; j < CH; ++j) {
        const uint32_t c = cbase + j;
        if (c < cols) {
          const uint32_t row = c / p.group, gq = c % p.group;
          const size_t rh = size_t(row) * p.q_heads + size_t(pc.h) * p.group + gq;
          float* out = p.part + (rh * p.split_stride + pc.slot) * (D + 2) + 2;
#pragma unroll
          for (uint32_t h = 0; h < D / 128; ++h) out[L::kVPair ? 2 * dl + h : h * 128 + dl] = acc[h][j];
        }
      }
    }
  }
  if (threadIdx.x == 0) grid_launch_dependents();
  tc::fence_before_sync();
  __syncthreads();
  if (warp == L::kMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, L::kTmemCols);
  }
}

}  // namespace kvb
