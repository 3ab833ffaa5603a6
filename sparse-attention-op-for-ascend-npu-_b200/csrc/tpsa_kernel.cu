// TriangleMix paged sparse prefill attention for B200 (sm_100a).
//
// One persistent launch computes, for every query row, the dense causal
// prefix / sink+local-window middle / dense causal tail key set of the
// reference operator (operator/op_kernel/triangle_paged_fia_fast_path.h:
// 209-438) under one online softmax, reading K/V pages straight from the
// BSND paged cache through the block table and writing bf16 output into the
// caller's buffer.
//
// CTA pairs.  The kernel runs as clusters of two CTAs on two SMs that share
// every tensor-core instruction (tcgen05 cta_group::2, M = 256):
//   * a work item is (64-token query block, kv head, key-tile range); its
//     256 rows (64 tokens x 4 GQA heads) are split between the pair: CTA r
//     owns query heads {4h + 2r, 4h + 2r + 1} (128 rows, one M half);
//   * each key tile [k0, k0 + w) is split between the pair as the MMA wants
//     its B operand split along N: CTA r loads keys [k0 + r*w/2, +w/2) of K
//     (for S = Q K^T) and d-half r of V (for O = P V), so every K/V byte is
//     loaded once per pair and serves 4 query heads.
// Roles (384 threads per CTA):
//   warp 0      K producer (Q of each item, K half-tiles; stores finished
//               output boxes)
//   warp 1      CTA 0: tcgen05 MMA issuer; both: TMEM owner
//   warp 2      CTA 0: work scheduler (global counter, longest items first;
//               item records into both CTAs' item rings)
//   warp 3      V producer (V half-tiles)
//   warps 4-11  two softmax warpgroups.  Key tile gt of the pair's tile
//               stream belongs to warpgroup gt % 2; both work on the same
//               rows and pass each row's lazy reference max from tile to
//               tile, so P of every tile is relative to the reference O is
//               kept in.  The owner of an item's last tile finishes the item.
// Tensor memory per CTA (fp32 columns): three S buffers [0,384) and the O
// accumulator [384,512).  Tile gt uses S buffer gt % 3; its P (bf16 pairs)
// overwrites columns 64-127 of that buffer and PV(gt) reads it there.  The
// issuer runs QK up to three tiles ahead of PV across item boundaries.
//
// Softmax arithmetic: scores are scaled into the log2 domain with one fused
// multiply-add, exponentiated with ex2.approx (MUFU), summed in fp32, and
// rounded to bf16 (round-to-nearest-even) for the PV product, as the
// reference does (vendor block_epilogue_online_softmax.hpp:886-906).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>

#include "sm100_ptx.cuh"
#include "tpsa_schedule.h"

namespace tpsa {

__device__ uint32_t g_device_status = 0;

// Optional event trace of one CTA pair (build with -DTPSA_TRACE, pair chosen by
// TPSA_TRACE_CLUSTER; compiled out of
// the library otherwise).  Each tracing thread owns one buffer and a register
// counter, so a trace point is two plain stores and a clock read.
#ifdef TPSA_TRACE
#ifndef TPSA_TRACE_CLUSTER
#define TPSA_TRACE_CLUSTER 0  // CTA pair whose events are recorded
#endif
// Roles: 0 K producer, 1 MMA issuer, 2-3 softmax warpgroups of CTA 0,
// 4 V producer, 5-6 softmax warpgroups of CTA 1.
constexpr uint32_t kTraceRoles = 7;
constexpr uint32_t kTraceCap = 1u << 14;
__device__ unsigned long long g_trace[kTraceRoles][kTraceCap][2];
__device__ uint32_t g_trace_n[kTraceRoles];
#define TPSA_TRACE_STATE uint32_t tr_n_ = 0
#ifndef TPSA_TRACE_EVMASK
#define TPSA_TRACE_EVMASK ~0ull  // events recorded (bit ev)
#endif
#define TPSA_TR(role, ev, arg)                                                    \
  do {                                                                            \
    if (((TPSA_TRACE_EVMASK >> (ev)) & 1ull) &&                                   \
        (blockIdx.x >> 1) == TPSA_TRACE_CLUSTER && tr_n_ < kTraceCap) {           \
      g_trace[role][tr_n_][0] = (static_cast<unsigned long long>(ev) << 32) |     \
                                static_cast<uint32_t>(arg);                        \
      g_trace[role][tr_n_][1] = clock64();                                        \
      ++tr_n_;                                                                    \
      g_trace_n[role] = tr_n_;                                                    \
    }                                                                             \
  } while (0)
#else
#define TPSA_TRACE_STATE \
  do {                   \
  } while (0)
#define TPSA_TR(role, ev, arg) \
  do {                         \
  } while (0)
#endif

namespace {

constexpr int kNumThreads = 384;
constexpr int kSoftmaxWarps = 8;  // two warpgroups, alternate key tiles
constexpr int kFirstSoftmaxWarp = 4;
// Register split (setmaxnreg): the control warpgroup (warps 0-3) keeps 56
// registers a thread, the two softmax warpgroups 224, within the launch's
// 384 x 168: 128 x 56 + 256 x 224 = 64512.
constexpr uint32_t kControlRegs = 56;
constexpr uint32_t kSoftmaxRegs = 224;
static_assert(128 * kControlRegs + 256 * kSoftmaxRegs <= 384 * 168, "register split");
// Tensor memory (512 columns, lane = row): three S buffers (P, as bf16
// pairs, over columns 64-127 of each) and the O accumulator shared by both
// softmax warpgroups.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kNumSBufs = 3;
constexpr uint32_t kTmemO = 384;
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;  // 1 s per wait
constexpr uint64_t kAbortSettleNs = 200000ull;      // let in-flight TMA land
constexpr float kRescaleLog2 = 8.0f;  // lazy O rescale threshold (log2 units)
// Column pairs c (of 16 per 32-column chunk) whose exponentials use the FMA
// pipe polynomial rather than MUFU ex2: bit c set.  None by default: with
// two softmax warps per SM sub-partition the MUFU pipe is not the limit
// (measured: every nonzero mask tried was slower).
#ifndef TPSA_POLY_MASK
#define TPSA_POLY_MASK 0u
#endif
constexpr uint16_t kPairMask = 0x3;

// Shared memory per CTA (offsets from a 1024-byte aligned base).
constexpr uint32_t kQHalfBytes = 128 * 128;        // 128 rows x 64 bf16
constexpr uint32_t kQBytes = 2 * kQHalfBytes;      // one Q buffer (2 d-halves)
constexpr uint32_t kRingSlotBytes = 16384;         // one key tile's K half, or its V half
constexpr uint32_t kKHalfBytes = 8192;             // d-half of a K half-tile
constexpr int kRing = 4;                           // key-tile slots (power of two)
constexpr uint32_t kOffQ = 0;                      // 2 Q buffers
constexpr uint32_t kOffK = kOffQ + 2 * kQBytes;     // K ring
constexpr uint32_t kOffV = kOffK + kRing * kRingSlotBytes;  // V ring
constexpr uint32_t kOffBar = kOffV + kRing * kRingSlotBytes;

enum BarId : uint32_t {
  kBarQFull = 0,                          // [2] CTA 0: both Q halves landed
  kBarQEmpty = kBarQFull + 2,             // [2] both CTAs: Q buffer free
  kBarKFull = kBarQEmpty + 2,             // [kRing] CTA 0: K of both CTAs landed
  kBarKEmpty = kBarKFull + kRing,         // [kRing] both: K slot free (its QK done)
  kBarVFull = kBarKEmpty + kRing,         // [kRing] CTA 0: V of both CTAs landed
  kBarVEmpty = kBarVFull + kRing,         // [kRing] both: V slot free (its PV done)
  kBarSFull = kBarVEmpty + kRing,         // [3] both: S buffer computed
  kBarPFull = kBarSFull + kNumSBufs,      // [3] CTA 0: P of the tile in the S buffer written
  kBarPvDone = kBarPFull + kNumSBufs,     // [3] both: PV from the S buffer completed
  kBarOEmpty = kBarPvDone + kNumSBufs,    // CTA 0: O read by the item's epilogue
  kBarItemFull = kBarOEmpty + 1,          // [2] both: item index written
  kBarItemEmpty = kBarItemFull + 2,       // [2] CTA 0: item index consumed
  kBarTail = kBarItemEmpty + 2,           // per CTA: V tail tile landed
  kBarDrain = kBarTail + 1,               // CTA 0: all MMAs complete
  kNumBars
};
// Arrivals: p_full takes one per warp of the tile's softmax warpgroup in
// both CTAs, o_empty one per warp of the item's finishing warpgroup in both
// CTAs; item_empty takes the two producers, the MMA issuer and the 8
// softmax warps of CTA 0 plus the two producers and the 8 softmax warps of
// CTA 1.
constexpr uint32_t kPairWgArrivals = kSoftmaxWarps;  // 4 warps x 2 CTAs
constexpr uint32_t kItemConsumers = 2 * (2 + kSoftmaxWarps) + 1;
// q_empty: the MMA issuer's commit after the item's last QK.  (The finished
// item's Q buffer then stages its output rows; the K producer stores them
// and waits for the store to read the buffer before it loads the next Q.)
constexpr uint32_t kQEmptyArrivals = 1;

constexpr uint32_t kOffItemSlots = (kOffBar + kNumBars * 8 + 15) & ~15u;  // 2 x ItemRec
constexpr uint32_t kOffTmemSlot = kOffItemSlots + 2 * 64;
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
constexpr uint32_t kOffSplitLast = kOffAbort + 4;  // int32 [2] (by split-item parity)
// Monotonic uint32 counters in shared memory, one count per warp and event
// (see softmax_role).
enum CounterId : uint32_t {
  kCntPub = 0,                  // [8] row values published by softmax warp (wg * 4 + quad)
  kCntCon = kCntPub + 8,        // [8] partner values read by softmax warp (wg * 4 + quad)
  kCntStaged = kCntCon + 8,     // [2] output rows of warpgroup wg staged for its TMA store
  kCntSplitW = kCntStaged + 2,  // split partial written
  kCntSplitD,                   // split merge decided (one count per split item)
  kNumCounters
};
constexpr uint32_t kOffCounters = kOffSplitLast + 8;
// Row values passed between the two warps that hold the same rows in the
// two softmax warpgroups: float [2 publishers][kChanSlots][128 rows].
constexpr uint32_t kChanSlots = 4;
constexpr uint32_t kOffXchg = (kOffCounters + 4 * kNumCounters + 15) & ~15u;
// Output staging: 2 KB per softmax warp (32 rows x 64 bytes), used to turn
// row-per-thread results into coalesced global stores.
constexpr uint32_t kStageBytesPerWarp = 32 * 64;
constexpr uint32_t kOffStage = (kOffXchg + 2 * kChanSlots * 128 * 4 + 127) & ~127u;
constexpr uint32_t kSmemUsed = kOffStage + 8 * kStageBytesPerWarp;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // alignment slack
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

// Workspace control words (first kControlBytes of the workspace, zeroed by
// the launcher): [0] next work item, [64..] one split counter per
// (tail block, kv head, pair rank).
constexpr int kCtlNextItem = 0;
constexpr int kCtlSplitBase = 64;

// One request of a launch (a batch-one call is a launch of one request).
// Its rows are packed at [q_row0, q_row0 + plan.query_tokens) of query and
// out, and its items at [item_base, item_base + plan.total_items) of the
// launch's item order.
struct ReqDesc {
  tpsa_plan plan;     // the request's own plan: its blocks, items and splits
  int32_t item_base;  // first launch item of the request
  int32_t q_row0;     // first packed query / output row
  int32_t table_off;  // its block-table row (int32 elements from block_table)
  int32_t slot_base;  // its first split-KV partial slot
  int32_t ctr_base;   // its first split counter
  int32_t tail_base;  // dispatch position of its first dense-tail item
  int32_t rest_base;  // dispatch position of its first other item, after all tail items
};
constexpr int kMaxReqs = 16;  // requests per launch (varlen batches are cut into launches)

struct KernelArgs {
  tpsa_plan plan;  // launch totals: total_items, kv_heads, scale, grid
  int32_t num_reqs;
  int32_t tail_total;  // dense-tail items of all requests (dispatched first)
  ReqDesc reqs[kMaxReqs];
  const int32_t* block_table;
  __nv_bfloat16* out;
  float* scratch;      // split partials (tail_items slots)
  int32_t* ctl;        // control words
  int32_t num_pages;
  int32_t words_per_row;       // visit mode
  uint32_t* visited;           // visit mode
  unsigned long long* tiles;   // visit mode: [tiles, keys]
};

struct Shared {
  uint8_t* base;
  uint32_t base_u32;
  uint32_t rank;  // CTA rank in the pair
  __device__ uint32_t bar(uint32_t id) const { return base_u32 + kOffBar + 8 * id; }
  // The same barrier in CTA 0 (shared::cluster address).
  __device__ uint32_t bar0(uint32_t id) const { return ptx::mapa(bar(id), 0); }
  __device__ volatile int* abort_flag() const {
    return reinterpret_cast<volatile int*>(base + kOffAbort);
  }
  __device__ uint32_t counter(uint32_t id) const { return base_u32 + kOffCounters + 4 * id; }
  __device__ uint4* item_slot(uint32_t i) const {
    return reinterpret_cast<uint4*>(base + kOffItemSlots + 64 * i);
  }
  __device__ uint32_t item_slot_addr(uint32_t i) const { return base_u32 + kOffItemSlots + 64 * i; }
};

__device__ __forceinline__ void raise_status(uint32_t bits) {
  atomicOr(&g_device_status, bits);
}

#ifdef TPSA_TRACE
// Start and end (globaltimer ns) and items run of every CTA of the last launch.
__device__ unsigned long long g_cta_span[1024][3];
// First wait that gave up: {set, block, thread, shared offset, parity or target}.
__device__ uint32_t g_timeout_site[5];
extern __shared__ uint8_t smem_raw[];
__device__ __forceinline__ void note_timeout(uint32_t addr, uint32_t arg) {
  if (atomicCAS(&g_timeout_site[0], 0u, 1u) == 0u) {
    g_timeout_site[1] = blockIdx.x;
    g_timeout_site[2] = threadIdx.x;
    g_timeout_site[3] = addr - ((ptx::smem_u32(smem_raw) + 1023u) & ~1023u);
    g_timeout_site[4] = arg;
  }
}
#define TPSA_NOTE_TIMEOUT(addr, arg) note_timeout(addr, arg)
#else
#define TPSA_NOTE_TIMEOUT(addr, arg) \
  do {                               \
  } while (0)
#endif

// Bounded wait: gives up after kWaitTimeoutNs or as soon as another role of
// this CTA has aborted; on timeout records TPSA_DEVICE_WAIT_TIMEOUT.
// kCluster selects a cluster-scope acquire (only needed where the signal
// carries the peer's st.shared::cluster stores: the item ring).
template <bool kCluster>
__device__ __forceinline__ bool try_wait_sel(uint32_t bar, uint32_t parity) {
  return kCluster ? ptx::mbar_try_wait_cluster(bar, parity) : ptx::mbar_try_wait(bar, parity);
}

template <bool kCluster>
__device__ __forceinline__ bool wait_bar_slow(uint32_t bar, uint32_t parity,
                                           volatile int* abort_flag) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (true) {
    if (try_wait_sel<kCluster>(bar, parity)) return true;
    if (*abort_flag) return false;
    if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1;
      raise_status(TPSA_DEVICE_WAIT_TIMEOUT);
      TPSA_NOTE_TIMEOUT(bar, parity);
      return false;
    }
  }
}

template <bool kCluster = false>
__device__ __forceinline__ bool wait_bar(const Shared& sh, uint32_t bar, uint32_t parity) {
  if (try_wait_sel<kCluster>(bar, parity)) return true;
  return wait_bar_slow<kCluster>(bar, parity, sh.abort_flag());
}

// Bounded wait used while draining (ignores the abort flag).
__device__ __forceinline__ void drain_bar(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
      raise_status(TPSA_DEVICE_WAIT_TIMEOUT);
      return;
    }
  }
}

// Bounded wait until the monotonic shared counter `id` reaches `target`
// (wrap-safe comparison); gives up like wait_bar.
__device__ __forceinline__ bool wait_count_slow(volatile int* abort_flag, uint32_t addr,
                                            uint32_t target) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (static_cast<int32_t>(ptx::ld_acquire_shared(addr) - target) < 0) {
    if (*abort_flag) return false;
    if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1;
      raise_status(TPSA_DEVICE_WAIT_TIMEOUT);
      TPSA_NOTE_TIMEOUT(addr, target | 0x80000000u);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ bool wait_count_at(const Shared& sh, uint32_t addr, uint32_t target) {
  if (static_cast<int32_t>(ptx::ld_acquire_shared(addr) - target) >= 0) return true;
  return wait_count_slow(sh.abort_flag(), addr, target);
}
__device__ __forceinline__ bool wait_count(const Shared& sh, uint32_t id, uint32_t target) {
  return wait_count_at(sh, sh.counter(id), target);
}

__device__ __forceinline__ uint32_t ring_slot(uint32_t r) { return r % kRing; }
__device__ __forceinline__ uint32_t ring_parity(uint32_t r) { return (r / kRing) & 1; }

__device__ __forceinline__ float mufu_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// (a0, a1) * (b, b) + (c, c) as one packed f32x2 FMA.
__device__ __forceinline__ void fma2(float a0, float a1, float b, float c, float& r0,
                                     float& r1) {
  uint64_t av, bv, cv, rv;
  asm("mov.b64 %0, {%1, %2};" : "=l"(av) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(bv) : "f"(b));
  asm("mov.b64 %0, {%1, %1};" : "=l"(cv) : "f"(c));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rv) : "l"(av), "l"(bv), "l"(cv));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r0), "=f"(r1) : "l"(rv));
}

// (s0, s1) += (a0, a1) as one packed f32x2 add.
__device__ __forceinline__ void add2(float& s0, float& s1, float a0, float a1) {
  uint64_t sv, av;
  asm("mov.b64 %0, {%1, %2};" : "=l"(sv) : "f"(s0), "f"(s1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(av) : "f"(a0), "f"(a1));
  asm("add.rn.f32x2 %0, %0, %1;" : "+l"(sv) : "l"(av));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(s0), "=f"(s1) : "l"(sv));
}

// Packed f32x2 helpers on 64-bit register pairs.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(a), "f"(b));
  return v;
}
__device__ __forceinline__ void unpk2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t add2v(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t sub2v(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2v(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// (2^x0, 2^x1) on the FMA and ALU pipes, the floating-point steps two lanes
// per packed f32x2 instruction: x = n + f with n = round(x) (magic-number
// rounding) and f in [-1/2, 1/2]; 2^f by a degree-3 minimax polynomial (Remez
// fit, max relative error 7.5e-5, coefficients from csrc/fit_exp2_poly.py);
// 2^n added to the exponent field.  x is clamped at -127.5 so that 2^n
// underflows the exponent for any x <= -127.5 (and -inf), and the integer
// max returns +0 there.
__device__ __forceinline__ void poly_exp2_x2(float x0, float x1, float& e0, float& e1) {
  const uint64_t xv = pk2(fmaxf(x0, -127.5f), fmaxf(x1, -127.5f));
  const uint64_t magic = pk2(12582912.0f, 12582912.0f);  // 1.5 * 2^23
  const uint64_t t = add2v(xv, magic);
  const uint64_t f = sub2v(xv, sub2v(t, magic));
  uint64_t q = fma2v(pk2(0.0551716685f, 0.0551716685f), f, pk2(0.2426111251f, 0.2426111251f));
  q = fma2v(q, f, pk2(0.6932609677f, 0.6932609677f));
  q = fma2v(q, f, pk2(0.9999280572f, 0.9999280572f));
  float q0, q1, t0, t1;
  unpk2(q, q0, q1);
  unpk2(t, t0, t1);
  e0 = __int_as_float(max(__float_as_int(q0) + (__float_as_int(t0) << 23), 0));
  e1 = __int_as_float(max(__float_as_int(q1) + (__float_as_int(t1) << 23), 0));
}

// ------------------------------------------------------------ scheduler ring
// Work items flow from CTA 0's producer to every consumer through a 2-slot
// ring in each CTA's shared memory.  A slot holds an item record: the item
// index (total_items or above ends the kernel), the decoded item and its
// block's tile geometry, decoded once by the scheduler so that no consumer
// repeats that integer arithmetic.  Consumers in CTA 0 release on their own
// item_empty, consumers in CTA 1 on CTA 0's (remote arrive).
struct alignas(16) ItemRec {
  int32_t idx;
  tpsa_item it;
  BlockTiles bt;
  // Item tiles only 64 keys wide (all others are 128): bit 0 the item's
  // tile 0, bit 1 its tile 1, bit 2 its last tile (the sink tile and a band
  // or key range that starts or ends half-way through a page).  Bits 8 and
  // up: the item's request within the launch.
  uint32_t narrow;
  __device__ __forceinline__ int32_t req() const { return static_cast<int32_t>(narrow >> 8); }
};
static_assert(sizeof(ItemRec) == 64, "an item record is four 16-byte words");

__device__ __forceinline__ ItemRec make_item_rec(const tpsa_plan& p, int32_t idx) {
  ItemRec rec;
  memset(&rec, 0, sizeof(rec));
  rec.idx = idx;
  if (idx < p.total_items) {
    rec.it = decode_item(p, idx);
    rec.bt = block_tiles(p, rec.it.block);
    const int32_t last = rec.it.tile_end - rec.it.tile_begin - 1;
    int32_t k0, w;
    tile_keys(rec.bt, rec.it.tile_begin, &k0, &w);
    rec.narrow |= w < kTileKeys ? 1u : 0u;
    if (last >= 1) {
      tile_keys(rec.bt, rec.it.tile_begin + 1, &k0, &w);
      rec.narrow |= w < kTileKeys ? 2u : 0u;
    }
    tile_keys(rec.bt, rec.it.tile_begin + last, &k0, &w);
    rec.narrow |= w < kTileKeys ? 4u : 0u;
  }
  return rec;
}

__device__ __forceinline__ bool take_item(const Shared& sh, uint32_t n, ItemRec* rec) {
  const uint32_t slot = n % 2;
  if (!wait_bar<true>(sh, sh.bar(kBarItemFull + slot), (n / 2) & 1)) return false;
  const uint4* src = sh.item_slot(slot);
  uint4* dst = reinterpret_cast<uint4*>(rec);
#pragma unroll
  for (int j = 0; j < 4; ++j) dst[j] = src[j];
  return true;
}

// The fields of item record n the MMA issuer uses: its index, tile count
// and narrow-tile bits.
struct ItemBrief {
  int32_t idx, ntiles;
  uint32_t narrow;
};
__device__ __forceinline__ bool take_item_brief(const Shared& sh, uint32_t n, ItemBrief* b) {
  const uint32_t slot = n % 2;
  if (!wait_bar<true>(sh, sh.bar(kBarItemFull + slot), (n / 2) & 1)) return false;
  const int32_t* w = reinterpret_cast<const int32_t*>(sh.item_slot(slot));
  b->idx = w[offsetof(ItemRec, idx) / 4];
  b->ntiles = w[(offsetof(ItemRec, it) + offsetof(tpsa_item, tile_end)) / 4] -
              w[(offsetof(ItemRec, it) + offsetof(tpsa_item, tile_begin)) / 4];
  b->narrow = static_cast<uint32_t>(w[offsetof(ItemRec, narrow) / 4]);
  return true;
}

__device__ __forceinline__ void release_item(const Shared& sh, uint32_t n) {
  ptx::mbar_arrive_cluster(sh.bar0(kBarItemEmpty + n % 2));
}

// ------------------------------------------------------------ scheduler
// One thread of CTA 0: takes work items from the grid-wide counter
// (longest first), decodes each into an item record and publishes it into
// the pair's two-slot item ring (both CTAs' copies), running up to two items
// ahead of the slowest consumer.  The index past the last item tells every
// consumer to stop.
template <bool kVarlen>
__device__ void scheduler_role(const KernelArgs& a, const Shared& sh) {
  const tpsa_plan& p = a.plan;
  int32_t next = atomicAdd(a.ctl + kCtlNextItem, 1);
  for (uint32_t n = 0;; ++n) {
    const uint32_t slot = n % 2;
    ItemRec rec;
    if (kVarlen) {
      // Dispatch order across the launch's requests: first every request's
      // dense-tail items (the longest), then every request's other items,
      // so that a later request's long items do not start last.  The record
      // carries the request-major index (item_base + item within request),
      // which the consumers use; the terminator carries total_items.
      int32_t q = 0, ridx = 0;
      if (next < p.total_items) {
        if (next < a.tail_total) {
          while (q + 1 < a.num_reqs && next >= a.reqs[q + 1].tail_base) ++q;
          ridx = next - a.reqs[q].tail_base;
        } else {
          const int32_t j = next - a.tail_total;
          while (q + 1 < a.num_reqs && j >= a.reqs[q + 1].rest_base) ++q;
          ridx = a.reqs[q].plan.tail_items + (j - a.reqs[q].rest_base);
        }
        rec = make_item_rec(a.reqs[q].plan, ridx);
        rec.idx = a.reqs[q].item_base + ridx;
      } else {
        rec = make_item_rec(a.reqs[0].plan, a.reqs[0].plan.total_items);
        rec.idx = p.total_items;
      }
      rec.narrow |= static_cast<uint32_t>(q) << 8;
    } else {
      rec = make_item_rec(p, next);
    }
    if (rec.idx < p.total_items) next = atomicAdd(a.ctl + kCtlNextItem, 1);
    if (!wait_bar(sh, sh.bar(kBarItemEmpty + slot), ((n / 2) & 1) ^ 1)) break;
    const uint4* words = reinterpret_cast<const uint4*>(&rec);
    const uint32_t peer = ptx::mapa(sh.item_slot_addr(slot), 1);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sh.item_slot(slot)[j] = words[j];
      ptx::st_cluster_v4(peer + 16 * j, words[j]);
    }
    ptx::mbar_arrive(sh.bar(kBarItemFull + slot));
    ptx::mbar_arrive_cluster_release(ptx::mapa(sh.bar(kBarItemFull + slot), 1));
    if (rec.idx >= p.total_items) break;
  }
}

// ------------------------------------------------------------ producers
// Two single-thread producers per CTA, each following the item ring: the K
// producer loads Q and the K half-tiles into the K ring (a slot frees when
// its QK completes), the V producer the V half-tiles into the V ring (a
// slot frees when its PV completes), so K can run ahead of V by the QK
// lookahead.  Both CTAs of the pair load their halves with pair TMA loads
// that complete on CTA 0's full barrier: of K, keys [r*half, (r+1)*half)
// of the tile, all 128 d; of V, all keys of the tile, d-half r.
// An item's output box staged in its Q buffer, to be stored by the K producer.
struct PendingStore {
  bool stages;          // a full, unsplit block: its epilogue stages the box
  uint32_t staged;      // staged items up to and including this one
  int32_t head, token;  // box coordinates in `out` (d is 0 and 64)
};

// Waits until item `ps` is staged (the finishing warpgroup counts four warps
// on each d-half counter), TMA-stores its two d-half boxes from Q buffer qb,
// and waits until the stores have read it.
__device__ __forceinline__ void flush_store(const Shared& sh, const CUtensorMap* tout,
                                            PendingStore& ps, uint32_t qb) {
  if (!ps.stages) return;
  ps.stages = false;
  if (!wait_count(sh, kCntStaged + 0, 4 * ps.staged)) return;
  if (!wait_count(sh, kCntStaged + 1, 4 * ps.staged)) return;
  const uint32_t src = sh.base_u32 + kOffQ + qb * kQBytes;
  ptx::tma_store_3d(tout, 0, ps.head, ps.token, src);
  ptx::tma_store_3d(tout, 64, ps.head, ps.token, src + kQHalfBytes);
  ptx::bulk_commit_group();
  ptx::bulk_wait_group_read<0>();
}

template <bool kVarlen>
__device__ void producer_role(const KernelArgs& a, const Shared& sh, const CUtensorMap* tq,
                              const CUtensorMap* tk64, const CUtensorMap* tk32,
                              const CUtensorMap* tv, const CUtensorMap* tout, bool v_side) {
  const tpsa_plan& p = a.plan;
  const uint32_t r = sh.rank;
  if (v_side) {
    ptx::prefetch_tmap(tv);
  } else {
    ptx::prefetch_tmap(tq);
    ptx::prefetch_tmap(tk64);
    ptx::prefetch_tmap(tk32);
  }
  const uint32_t bar_full = sh.bar0(v_side ? kBarVFull : kBarKFull);
  const uint32_t bar_empty = sh.bar(v_side ? kBarVEmpty : kBarKEmpty);
  const uint32_t ring_base = sh.base_u32 + (v_side ? kOffV : kOffK);
  uint32_t ring = 0, q_iter = 0, tail_iter = 0;
  // K side: the output boxes staged in the two Q buffers, and staged items so far.
  PendingStore pend0{false, 0, 0, 0}, pend1{false, 0, 0, 0};  // Q buffers 0 and 1
  uint32_t staged = 0;
  bool ok = true;
  TPSA_TRACE_STATE;
  for (uint32_t n = 0; ok; ++n) {
    ItemRec rec;
    if (!take_item(sh, n, &rec)) break;
    release_item(sh, n);
    if (rec.idx >= p.total_items) break;
    if (r == 0 && !v_side) TPSA_TR(0, 20, rec.idx);
    const tpsa_item& it = rec.it;
    const BlockTiles& bt = rec.bt;
    // The item's request (a batch-one launch has one, at row and table 0).
    const ReqDesc& rq = a.reqs[kVarlen ? rec.req() : 0];
    const int32_t* table = kVarlen ? a.block_table + rq.table_off : a.block_table;
    const int32_t req_seq_len = kVarlen ? rq.plan.seq_len : p.seq_len;
    const int32_t q_row0 = kVarlen ? rq.q_row0 : 0;

    if (!v_side) {
      // Q: this CTA's 128 rows (64 tokens x query heads 4h + 2r, 4h + 2r + 1).
      // The buffer last held item n - 2: its QKs completed (q_empty) and its
      // output, if staged there, is stored first.
      const uint32_t qb = q_iter % 2;
      if (q_iter >= 2) {
        if (qb == 0) {
          flush_store(sh, tout, pend0, 0);
        } else {
          flush_store(sh, tout, pend1, 1);
        }
        if (!wait_bar(sh, sh.bar(kBarQEmpty + qb), ((q_iter / 2) - 1) & 1)) break;
      }
      const bool full_block = !kVarlen || bt.q_end - bt.q_begin == kBlockQ;
      PendingStore cur;
      cur.stages = it.num_splits == 1 && full_block;
      staged += cur.stages ? 1u : 0u;
      cur.staged = staged;
      cur.head = it.kv_head * kGroupSize + 2 * static_cast<int32_t>(r);
      cur.token = q_row0 + it.block * kBlockQ;
      if (qb == 0) {
        pend0 = cur;
      } else {
        pend1 = cur;
      }
      ptx::mbar_arrive_expect_tx_cluster(sh.bar0(kBarQFull + qb), kQBytes);
      for (int dh = 0; dh < 2; ++dh) {
        ptx::tma_load_3d_pair(sh.base_u32 + kOffQ + qb * kQBytes + dh * kQHalfBytes, tq, dh * 64,
                              it.kv_head * kGroupSize + 2 * r, q_row0 + it.block * kBlockQ,
                              sh.bar0(kBarQFull + qb));
      }
      ++q_iter;
      if (r == 0) TPSA_TR(0, 21, rec.idx);
    }

    for (int32_t t = it.tile_begin; t < it.tile_end && ok; ++t) {
      int32_t k0, w;
      tile_keys(bt, t, &k0, &w);
      const int32_t page = __ldg(table + k0 / kPageSize);
      int32_t tok;
      if (page < 0 || page >= a.num_pages) {
        raise_status(TPSA_DEVICE_BAD_PAGE);
        tok = -kPageSize;  // fully out of bounds: TMA fills zeros
      } else {
        tok = page * kPageSize + (k0 % kPageSize);
      }
      if (a.tiles != nullptr && r == 0 && !v_side) {
        atomicAdd(a.tiles, 1ull);
        atomicAdd(a.tiles + 1, static_cast<unsigned long long>(w));
      }
      const uint32_t s = ring_slot(ring);
      if (!wait_bar(sh, bar_empty + 8 * s, ring_parity(ring) ^ 1)) { ok = false; break; }
      ++ring;
      const uint32_t dst = ring_base + s * kRingSlotBytes;
      if (!v_side) {
        // Keys at or beyond seq_len (unwritten cache slots of the last page)
        // only meet masked scores, which select -inf whatever they hold.
        const int32_t half = w / 2;
        const CUtensorMap* km = w == kTileKeys ? tk64 : tk32;
        ptx::mbar_arrive_expect_tx_cluster(bar_full + 8 * s,
                                           static_cast<uint32_t>(half) * kHeadDim * 2);
        for (int dh = 0; dh < 2; ++dh) {
          ptx::tma_load_3d_pair(dst + dh * kKHalfBytes, km, dh * 64, it.kv_head,
                                tok + static_cast<int32_t>(r) * half, bar_full + 8 * s);
        }
      } else if (k0 + w <= req_seq_len) {
        ptx::mbar_arrive_expect_tx_cluster(bar_full + 8 * s, static_cast<uint32_t>(w) * 64 * 2);
        for (int sub = 0; sub < w / 64; ++sub) {
          ptx::tma_load_3d_pair(dst + sub * 8192, tv, static_cast<int32_t>(r) * 64, it.kv_head,
                                tok + sub * 64, bar_full + 8 * s);
        }
      } else {
        // Values at or beyond seq_len may be unwritten cache slots: load the
        // tile into this CTA's slot here, zero those rows so P = 0 never
        // meets a NaN, then release the slot with a plain arrival.
        ptx::mbar_arrive_expect_tx(sh.bar(kBarTail), static_cast<uint32_t>(w) * 64 * 2);
        for (int sub = 0; sub < w / 64; ++sub) {
          ptx::tma_load_3d(dst + sub * 8192, tv, static_cast<int32_t>(r) * 64, it.kv_head,
                           tok + sub * 64, sh.bar(kBarTail));
        }
        if (!wait_bar(sh, sh.bar(kBarTail), tail_iter & 1)) { ok = false; break; }
        ++tail_iter;
        for (int32_t row = req_seq_len - k0; row < w; ++row) {
          uint4* d4 = reinterpret_cast<uint4*>(sh.base + (dst - sh.base_u32) + row * 128);
#pragma unroll
          for (int j = 0; j < 8; ++j) d4[j] = make_uint4(0, 0, 0, 0);
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive_cluster(bar_full + 8 * s);
      }
      if (r == 0) TPSA_TR(v_side ? 4 : 0, 22, t);
    }
  }
  if (!v_side) {
    // The last two items' outputs, oldest first, complete before the CTA
    // exits (flush_store gives up if the softmax aborted).
    if (ok && !*sh.abort_flag()) {
      if (q_iter % 2 == 0) {
        flush_store(sh, tout, pend0, 0);
        flush_store(sh, tout, pend1, 1);
      } else {
        flush_store(sh, tout, pend1, 1);
        flush_store(sh, tout, pend0, 0);
      }
    }
    ptx::bulk_wait_group<0>();
  }
  if (!ok || *sh.abort_flag()) {
    // Aborted: give in-flight TMA loads time to land before the CTA exits.
    const uint64_t t0 = ptx::globaltimer_ns();
    while (ptx::globaltimer_ns() - t0 < kAbortSettleNs) {
    }
  }
}

// ------------------------------------------------------------ MMA issuer
// The whole warp runs this role: operands are computed by every lane (they
// are warp-uniform) and one elected lane issues each tcgen05 instruction.
__device__ void mma_role(const KernelArgs& a, const Shared& sh, uint32_t tmem, int lane) {
  const tpsa_plan& p = a.plan;
  TPSA_TRACE_STATE;
  // tcgen05.mma issue blocks once about three MMAs are queued, so this
  // warp's own instructions between MMA batches leave the tensor pipe idle.
  // The loop below therefore keeps its per-tile work to barrier waits,
  // commits and additions to operands prepared once: descriptor bases
  // (32-bit additions to their low word, which holds the start address),
  // barrier addresses, instruction descriptors and incremental ring
  // positions.  (Measured: the same loop run by one thread of the warp is
  // slower.)
  const uint32_t bar_k_full = sh.bar(kBarKFull), bar_k_empty = sh.bar(kBarKEmpty);
  const uint32_t bar_v_full = sh.bar(kBarVFull), bar_v_empty = sh.bar(kBarVEmpty);
  const uint32_t bar_s_full = sh.bar(kBarSFull), bar_p_full = sh.bar(kBarPFull);
  const uint32_t bar_pv_done = sh.bar(kBarPvDone), bar_q_full = sh.bar(kBarQFull);
  const uint32_t bar_q_empty = sh.bar(kBarQEmpty), bar_o_empty = sh.bar(kBarOEmpty);
  // Descriptor start addresses are in 16-byte units, in the low word.
  const uint64_t q_desc0 = ptx::smem_desc_sw128(sh.base_u32 + kOffQ, 16, 1024);
  const uint64_t k_desc0 = ptx::smem_desc_sw128(sh.base_u32 + kOffK, 16, 1024);
  const uint64_t v_desc0 = ptx::smem_desc_sw128(sh.base_u32 + kOffV, kKHalfBytes, 1024);
  const uint32_t q_hi = static_cast<uint32_t>(q_desc0 >> 32);
  const uint32_t k_hi = static_cast<uint32_t>(k_desc0 >> 32);
  const uint32_t v_hi = static_cast<uint32_t>(v_desc0 >> 32);
  auto desc = [](uint32_t lo, uint32_t hi) { return (static_cast<uint64_t>(hi) << 32) | lo; };
  constexpr uint32_t kSlotUnits = kRingSlotBytes >> 4;
  constexpr uint32_t kQUnits = kQBytes >> 4;
  constexpr uint32_t kIdQk128 = ptx::idesc_bf16_f32(256, 128, 0);
  constexpr uint32_t kIdQk64 = ptx::idesc_bf16_f32(256, 64, 0);
  constexpr uint32_t kIdPv = ptx::idesc_bf16_f32(256, 128, 1);

  // One lane, elected once, issues every tcgen05 instruction of this role
  // under a predicate (an elect.sync per instruction costs more).
  const uint32_t leader = ptx::elect_one();
  auto warp_wait = [&](uint32_t bar, uint32_t parity) -> bool {
    return __all_sync(0xffffffffu, wait_bar(sh, bar, parity));
  };

  // S(buf) = Q K^T for the key tile in ring slot `slot` (M = 256 over the
  // pair, N = 128 or 64).
  auto issue_qk = [&](uint32_t q_lo, uint32_t slot, uint32_t buf, bool narrow) {
    const uint32_t d = tmem + (buf << 7);
    const uint32_t idesc = narrow ? kIdQk64 : kIdQk128;
    const uint32_t k_lo = static_cast<uint32_t>(k_desc0) + slot * kSlotUnits;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t qo = (k / 4) * (kQHalfBytes >> 4) + (k % 4) * 2;
      const uint32_t ko = (k / 4) * (kKHalfBytes >> 4) + (k % 4) * 2;
      ptx::umma_ss_pair_if(leader, d, desc(q_lo + qo, q_hi), desc(k_lo + ko, k_hi), idesc, k > 0 ? 1u : 0u);
    }
  };
  // O += P V: P (bf16 pairs) over columns 64-127 of S buffer buf, V the
  // d-half of this CTA in ring slot `slot`.
  auto issue_pv = [&](uint32_t slot, uint32_t buf, bool narrow, bool first) {
    const uint32_t d = tmem + kTmemO;
    const uint32_t pa = tmem + (buf << 7) + 64;
    const uint32_t v_lo = static_cast<uint32_t>(v_desc0) + slot * kSlotUnits;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k < 4 || !narrow) {
        ptx::umma_ts_pair_if(leader, d, pa + k * 8, desc(v_lo + k * (2048 >> 4), v_hi), kIdPv,
                             (first && k == 0) ? 0u : 1u);
      }
    }
  };

  // The key tiles of all items form one stream over three S buffers (tile
  // gt uses buffer gt % 3): after PV(t) this warp issues QK(t + 3), which may
  // belong to a later item (S buffer t % 3 is free once PV(t), which reads
  // its P, is issued).  Only the first PV of an item waits for the previous
  // item's O to be released.  A QK cursor takes items from the ring; each QK
  // leaves a control word for its tile's PV up to three tiles later.  The QK
  // cursor stays within one item of the PV cursor: the Q buffer of item k + 2
  // is released by the epilogue of item k, which needs item k's PVs.
  enum : uint32_t {
    kTNarrow = 1u,     // 64-key tile
    kTFirst = 2u,      // first tile of its item (PV overwrites O)
    kTItemStart = 4u,  // first tile of an item that is not the first item
    kTItemOdd = 8u,    // with kTItemStart: the O-empty phase to wait for
    kTIssued = 16u,    // a QK was issued (no control word otherwise)
    kTItemShift = 8,   // bits 8 and up: the tile's item number (1-based)
  };
  uint32_t slot_q = 0, phase_q = 0, slot_v = 0, phase_v = 0, q_iter = 0;
  uint32_t sb_q = 0, sb_v = 0, pass_v = 0;  // S buffers of the QK / PV cursors
  uint32_t n_item = 0;                      // items taken from the ring
  int32_t q_n = 0, q_ntiles = 0;
  uint32_t q_narrow = 0, q_qb = 0;
  uint32_t q_qd = static_cast<uint32_t>(q_desc0);
  bool q_done = false;
  bool ok = true;
  // The next QK is prepared (its item taken, its Q and K waited for, its
  // control word computed) by plan_qk and issued by fire_qk, so that in the
  // steady state the QK that follows PV(t) is prepared while this warp waits
  // for P(t), and PV(t) and QK(t + 3) go to the tensor pipe back to back.
  uint32_t plan_info = 0;
  bool plan_narrow = false;
  // Prepares the next tile's QK; false when none may be issued now (no tile
  // left, or it starts an item more than one ahead of item `bound`, 0 for
  // no bound), or when a wait gave up (then ok is cleared).
  auto plan_qk = [&](uint32_t bound) -> bool {
    if (q_done) return false;
    if (q_n == q_ntiles) {
      if (bound != 0 && n_item > bound) return false;
      ItemBrief rec;
      const bool got = take_item_brief(sh, n_item, &rec);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        return false;
      }
      __syncwarp();
      if (lane == 0) release_item(sh, n_item);
      if (rec.idx >= p.total_items) {
        q_done = true;
        return false;
      }
      if (lane == 0) TPSA_TR(1, 10, rec.idx);
      ++n_item;
      q_n = 0;
      q_ntiles = rec.ntiles;
      q_narrow = rec.narrow;
      q_qb = q_iter & 1;
      if (!warp_wait(bar_q_full + 8 * q_qb, (q_iter >> 1) & 1)) {
        ok = false;
        return false;
      }
      ++q_iter;
      q_qd = static_cast<uint32_t>(q_desc0) + q_qb * kQUnits;
    }
    const int32_t last = q_ntiles - 1;
    plan_narrow = (q_n < 2 && ((q_narrow >> q_n) & 1u)) || (q_n == last && (q_narrow & 4u));
    plan_info = kTIssued | (plan_narrow ? kTNarrow : 0u) | (q_n == 0 ? kTFirst : 0u) |
                (q_n == 0 && n_item > 1 ? kTItemStart : 0u) |
                (((n_item - 1) & 1) ? kTItemOdd : 0u) | (n_item << kTItemShift);
    if (lane == 0) TPSA_TR(1, 19, sb_q);
    if (!warp_wait(bar_k_full + 8 * slot_q, phase_q)) {
      ok = false;
      return false;
    }
    if (lane == 0) TPSA_TR(1, 17, sb_q);
    return true;
  };
  // Issues the planned QK and returns its control word.
  auto fire_qk = [&]() -> uint32_t {
    ptx::tc_fence_after();
    issue_qk(q_qd, slot_q, sb_q, plan_narrow);
    if (lane == 0) TPSA_TR(1, 18, sb_q);
    ptx::umma_commit_pair_mc_if(leader, bar_s_full + 8 * sb_q, kPairMask);
    ptx::umma_commit_pair_mc_if(leader, bar_k_empty + 8 * slot_q, kPairMask);
    if (q_n == q_ntiles - 1) ptx::umma_commit_pair_mc_if(leader, bar_q_empty + 8 * q_qb, kPairMask);
    slot_q = (slot_q + 1) & (kRing - 1);
    phase_q ^= slot_q == 0 ? 1u : 0u;
    sb_q = sb_q == kNumSBufs - 1 ? 0 : sb_q + 1;
    ++q_n;
    return plan_info;
  };

  // Control words of the (up to three) tiles whose QK is issued and whose
  // PV is not, oldest first; 0 for none.
  uint32_t info0 = 0, info1 = 0, info2 = 0;
  int have = 0;
  auto push = [&](uint32_t info) {
    if (have == 0) {
      info0 = info;
    } else if (have == 1) {
      info1 = info;
    } else {
      info2 = info;
    }
    ++have;
  };
  // Issues QKs up to three ahead.  A QK that starts item n_item + 1 waits
  // until the oldest pending PV is in item n_item: that item's Q buffer is
  // released by the epilogue of item n_item - 1.
  auto refill = [&]() {
    while (ok && have < 3 && plan_qk(have > 0 ? (info0 >> kTItemShift) : 0u)) push(fire_qk());
  };
  refill();
  while (ok && have > 0) {
    // The QK to follow PV(t), prepared before P(t) is waited for.  Starting
    // a new item here needs PV(t) itself to be in item n_item or later (the
    // Q wait may not depend on PV(t)); otherwise refill takes it after PV(t).
    const bool planned = plan_qk(info0 >> kTItemShift);
    if (!ok) break;
    if (lane == 0) TPSA_TR(1, 12, sb_v);
    if (info0 & kTItemStart) {
      // O of the previous item (item index k - 1) has been read by its
      // epilogue: phase (k - 2) & 1 of o_empty.
      if (!warp_wait(bar_o_empty, (info0 & kTItemOdd) ? 0u : 1u)) { ok = false; break; }
      if (lane == 0) TPSA_TR(1, 11, sb_v);
    }
    if (!warp_wait(bar_p_full + 8 * sb_v, pass_v & 1)) { ok = false; break; }
    if (lane == 0) TPSA_TR(1, 13, sb_v);
    if (!warp_wait(bar_v_full + 8 * slot_v, phase_v)) { ok = false; break; }
    if (lane == 0) TPSA_TR(1, 14, sb_v);
    ptx::tc_fence_after();
    issue_pv(slot_v, sb_v, (info0 & kTNarrow) != 0, (info0 & kTFirst) != 0);
    if (lane == 0) TPSA_TR(1, 15, sb_v);
    ptx::umma_commit_pair_mc_if(leader, bar_v_empty + 8 * slot_v, kPairMask);
    ptx::umma_commit_pair_mc_if(leader, bar_pv_done + 8 * sb_v, kPairMask);
    const uint32_t fired = planned ? fire_qk() : 0u;
    if (lane == 0) TPSA_TR(1, 16, sb_v);
    slot_v = (slot_v + 1) & (kRing - 1);
    phase_v ^= slot_v == 0 ? 1u : 0u;
    if (sb_v == kNumSBufs - 1) {
      sb_v = 0;
      ++pass_v;
    } else {
      ++sb_v;
    }
    info0 = info1;
    info1 = info2;
    info2 = 0;
    --have;
    if (fired != 0) push(fired);
    refill();
    if (lane == 0) TPSA_TR(1, 23, have);
  }
  // All MMAs issued by this warp complete before TMEM is released.
  ptx::umma_commit_pair_elect(sh.bar(kBarDrain));
  if (lane == 0) drain_bar(sh.bar(kBarDrain), 0);
  __syncwarp();
}

// ------------------------------------------------------------ softmax
template <int W>
__device__ __forceinline__ void load_s(uint32_t taddr, float (&s)[W]) {
  uint32_t r[W];
#pragma unroll
  for (int c = 0; c < W / 32; ++c) {
    ptx::tmem_ld32(taddr + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * c]));
  }
  ptx::tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < W; ++c) s[c] = __uint_as_float(r[c]);
}

// Multiplies the 128 O columns of this thread's row by `factor`.
__device__ __forceinline__ void rescale_o(uint32_t o_addr, float factor) {
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    ptx::tmem_ld32(o_addr + 32 * c, r);
    ptx::tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * factor);
    ptx::tmem_st32(o_addr + 32 * c, r);
  }
}

// Bits c of the result: key kc + c (c < 32) is in the key set of query row
// q.  Dense rows see keys <= q; sparse rows additionally drop keys in
// [8, q - 512).
__device__ __forceinline__ uint32_t bits_below(int32_t x) {
  return x <= 0 ? 0u : (x >= 32 ? ~0u : (1u << x) - 1u);
}
__device__ __forceinline__ uint32_t chunk_mask(int32_t q, bool sparse, int32_t kc) {
  uint32_t m = bits_below(q - kc + 1);
  if (sparse) m &= ~bits_below(q - kLocalWindow - kc) | bits_below(kSinkTokens - kc);
  return m;
}

// Lazy online-softmax reference of a row: the reference max moves to the
// tile's row max m_tile only when that exceeds it by more than 2^kRescaleLog2
// after scaling (or when the row had no key yet), so O and l are rescaled
// rarely and exponentials stay below 2^kRescaleLog2.
__device__ __forceinline__ float next_ref(float m_ref, float m_tile, float scale_log2) {
  const bool move =
      m_tile > m_ref && (m_ref == -INFINITY || (m_tile - m_ref) * scale_log2 > kRescaleLog2);
  return move ? m_tile : m_ref;
}

// Row values passed from one softmax warp to the warp holding the same 32
// rows in the other warpgroup (warps quad + 4 and quad + 8), in order,
// through a kChanSlots-deep ring per direction.  Publishing counts on the
// publisher's counter; reading counts on the reader's, and a publisher
// reuses a slot only once the reader has counted the value it held.
struct RowChannel {
  uint32_t mine, theirs;   // shared addresses of this row in the two rings
  uint32_t pub_cnt;        // this warp's publication counter; the partner's is
                           // peer_pub below, the read counters follow at +32 bytes
  uint32_t peer_pub;
  uint32_t n_pub, n_read;

  __device__ __forceinline__ bool publish(const Shared& sh, float v) {
    if (n_pub >= kChanSlots &&
        !__all_sync(0xffffffffu, wait_count_at(sh, peer_pub + 32, n_pub - kChanSlots + 1))) {
      return false;
    }
    ptx::st_shared_f32(mine + (n_pub % kChanSlots) * 512, v);
    __syncwarp();
    if ((threadIdx.x & 31) == 0) ptx::red_release_add_shared(pub_cnt, 1);
    ++n_pub;
    return true;
  }
  // The partner's next value; false if the wait gave up.
  __device__ __forceinline__ bool read(const Shared& sh, float* v) {
    if (!__all_sync(0xffffffffu, wait_count_at(sh, peer_pub, n_read + 1))) return false;
    *v = ptx::ld_shared_f32(theirs + (n_read % kChanSlots) * 512);
    __syncwarp();
    if ((threadIdx.x & 31) == 0) ptx::red_release_add_shared(pub_cnt + 32, 1);
    ++n_read;
    return true;
  }
};

// Replaces the keys of a 32-key chunk of S (fp32 bits) that are outside the
// row's key set (bit c of m clear) by -inf.
__device__ __forceinline__ void mask_chunk(uint32_t (&r)[32], uint32_t m) {
#pragma unroll
  for (int c = 0; c < 32; ++c) r[c] = ((m >> c) & 1u) ? r[c] : 0xff800000u;
}

// Exponentials of one 32-key chunk of S (fp32 bits in r): P as 16 bf16
// pairs stored to tensor memory at p_addr, their sum added to (sum0, sum1).
// Pair c of the chunk uses the FMA-pipe polynomial when bit c of kPoly is
// set, MUFU ex2 otherwise.
template <uint32_t kPoly = TPSA_POLY_MASK>
__device__ __forceinline__ void exp_chunk(const uint32_t (&r)[32], float scale_log2, float neg_mb,
                                          uint32_t p_addr, float& sum0, float& sum1) {
  uint32_t pk[16];
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const float v0 = __uint_as_float(r[2 * c]), v1 = __uint_as_float(r[2 * c + 1]);
    float x0, x1;
    fma2(v0, v1, scale_log2, neg_mb, x0, x1);
    float e0, e1;
    if ((kPoly >> c) & 1u) {
      poly_exp2_x2(x0, x1, e0, e1);
    } else {
      e0 = mufu_exp2(x0);
      e1 = mufu_exp2(x1);
    }
    add2(sum0, sum1, e0, e1);
    pk[c] = pack_bf16x2(e0, e1);
  }
  ptx::tmem_st16(p_addr, pk);
}

__device__ __forceinline__ float chunk_max(const uint32_t (&r)[32]) {
  float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
  for (int c = 0; c < 32; c += 8) {
    mx0 = max3(mx0, __uint_as_float(r[c]), __uint_as_float(r[c + 1]));
    mx1 = max3(mx1, __uint_as_float(r[c + 2]), __uint_as_float(r[c + 3]));
    mx2 = max3(mx2, __uint_as_float(r[c + 4]), __uint_as_float(r[c + 5]));
    mx3 = max3(mx3, __uint_as_float(r[c + 6]), __uint_as_float(r[c + 7]));
  }
  return fmaxf(max3(mx0, mx1, mx2), mx3);
}

// Per-row state of the online softmax over one item's tiles, per warpgroup:
// the reference max as of the last tile this warpgroup knows of, and the
// warpgroup's partial row sum (over its own tiles) relative to it.
struct RowState {
  float m_ref;
  float l_part;
};

// Moves this warpgroup's reference to m (from a tile of the other
// warpgroup), rescaling the partial sum.  References only grow.
__device__ __forceinline__ void adopt_ref(RowState& st, float m, float scale_log2) {
  if (m != st.m_ref) {
    st.l_part *= st.m_ref == -INFINITY ? 0.0f : mufu_exp2((st.m_ref - m) * scale_log2);
    st.m_ref = m;
  }
}

// Where a tile lives and what its owner needs to know.
struct TileArgs {
  uint32_t s_addr;      // the tile's S buffer (P goes to its columns 64-127)
  uint32_t o_addr;      // O (128 columns)
  int32_t k0;           // first key of the tile
  bool wide;            // 128 keys (else 64)
  bool masked;          // some key of the tile is outside some row's key set
  bool first;           // first tile of the item (its PV overwrites O)
  bool last;            // last tile of the item (its decision is not passed on)
  uint32_t prev_bar;    // pv_done barrier of the previous tile, and its parity
  uint32_t prev_parity;
  uint32_t* trn;        // trace counter of this thread when it records (TPSA_TRACE)
  uint32_t trole;
};
#ifdef TPSA_TRACE
#define TPSA_TILE_TR(t, ev)                                   \
  do {                                                        \
    if ((t).trn != nullptr) {                                 \
      uint32_t& tr_n_ = *(t).trn;                             \
      TPSA_TR((t).trole, ev, 0);                              \
    }                                                         \
  } while (0)
#else
#define TPSA_TILE_TR(t, ev) \
  do {                      \
  } while (0)
#endif

// Keeps the visited bits of a 32-key chunk (debug output) and masks it.
template <bool kVisit>
__device__ __forceinline__ void prepare_chunk(uint32_t (&r)[32], bool mk, int32_t q, bool sparse,
                                              int32_t kc, uint32_t* visit_row,
                                              int32_t words_per_row) {
  const uint32_t m = mk ? chunk_mask(q, sparse, kc) : ~0u;
  if (kVisit && visit_row != nullptr && m != 0 && kc / 32 < words_per_row) {
    atomicOr(visit_row + kc / 32, m);
  }
  if (mk) mask_chunk(r, m);
}

// One key tile of this warpgroup, the whole row of this thread: load S,
// mask, row max; take the reference the previous tile (the other
// warpgroup's) left, move it if this tile's maxima require, and pass it on;
// exponentials and P into tensor memory; rescale O (after the previous
// tile's PV completed) when the reference moved.  P (bf16 pairs) goes to
// columns 64-127 of the S buffer.  A 64-key tile stays in registers; of a
// 128-key tile, keys 64-127 stay in registers while keys 0-63 are loaded
// twice (for the max, then for the exponentials), which keeps 64 of them
// live at a time: their P lands over S columns 64-127 only after those
// were read.  Returns false if a wait gave up.
template <bool kVisit>
__device__ __forceinline__ bool softmax_tile(const Shared& sh, const tpsa_plan& p,
                                             const TileArgs& t, int32_t q, bool sparse,
                                             RowChannel& ch, RowState& st,
                                             uint32_t* visit_row, int32_t words_per_row) {
  uint32_t ra[32], rb[32];
  ptx::tmem_ld32(t.s_addr, ra);
  ptx::tmem_ld32(t.s_addr + 32, rb);
  ptx::tmem_wait_ld_regs(ra);
  ptx::tmem_fence_regs(rb);
  prepare_chunk<kVisit>(ra, t.masked, q, sparse, t.k0, visit_row, words_per_row);
  prepare_chunk<kVisit>(rb, t.masked, q, sparse, t.k0 + 32, visit_row, words_per_row);
  float lm = fmaxf(chunk_max(ra), chunk_max(rb));
  if (t.wide) {
    ptx::tmem_ld32(t.s_addr + 64, ra);
    ptx::tmem_ld32(t.s_addr + 96, rb);
    ptx::tmem_wait_ld_regs(ra);
    ptx::tmem_fence_regs(rb);
    prepare_chunk<kVisit>(ra, t.masked, q, sparse, t.k0 + 64, visit_row, words_per_row);
    prepare_chunk<kVisit>(rb, t.masked, q, sparse, t.k0 + 96, visit_row, words_per_row);
    lm = fmaxf(lm, fmaxf(chunk_max(ra), chunk_max(rb)));
  }
  TPSA_TILE_TR(t, 30);
  const float sl2 = p.scale_log2;
  // Optimistic agreement: the exponentials use this warpgroup's reference
  // as of its previous tile; the other warpgroup's decision for the tile in
  // between is read after the reloaded keys 0-63 (it is usually published
  // by then) and, in the rare case that it changes this tile's reference,
  // those are redone; keys 64-127, still in registers, follow with the
  // final reference.
  float m_new = next_ref(st.m_ref, lm, sl2);
  bool agreed = t.first;
  float sum0 = 0.0f, sum1 = 0.0f;
  const uint32_t p_addr = t.s_addr + 64;
#pragma unroll 1
  while (true) {
    if (t.wide) {
      const float neg_mb = m_new == -INFINITY ? 0.0f : -m_new * sl2;
      sum0 = 0.0f;
      sum1 = 0.0f;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t rc[32];
        ptx::tmem_ld32(t.s_addr + 32 * c, rc);
        ptx::tmem_wait_ld_regs(rc);
        if (t.masked) mask_chunk(rc, chunk_mask(q, sparse, t.k0 + 32 * c));
        exp_chunk(rc, sl2, neg_mb, p_addr + 16 * c, sum0, sum1);
      }
    }
    if (agreed) break;
    float mp;
    if (!ch.read(sh, &mp)) return false;
    agreed = true;
    adopt_ref(st, mp, sl2);
    const float m2 = next_ref(st.m_ref, lm, sl2);
    if (!__any_sync(0xffffffffu, m2 != m_new)) break;
    m_new = m2;
  }
  // The decision is final here: pass it on before the remaining
  // exponentials, so that the other warpgroup's next tile, which reads it
  // half-way through, does not wait for them.
  if (!t.last && !ch.publish(sh, m_new)) return false;
  TPSA_TILE_TR(t, 31);
  {
    const float neg_mb = m_new == -INFINITY ? 0.0f : -m_new * sl2;
    const uint32_t p_kept = p_addr + (t.wide ? 32 : 0);
    exp_chunk(ra, sl2, neg_mb, p_kept, sum0, sum1);
    exp_chunk(rb, sl2, neg_mb, p_kept + 16, sum0, sum1);
  }
  TPSA_TILE_TR(t, 32);
  const bool moved = m_new != st.m_ref;
  if (__any_sync(0xffffffffu, moved)) {
    float factor = 1.0f;
    if (moved) factor = st.m_ref == -INFINITY ? 0.0f : mufu_exp2((st.m_ref - m_new) * sl2);
    st.l_part *= factor;
    st.m_ref = m_new;
    if (!t.first) {
      // O holds the PVs of the earlier tiles, the last of which has
      // completed before O is rescaled; this tile's PV is issued only after
      // this warp publishes P.
      if (!__all_sync(0xffffffffu, wait_bar(sh, t.prev_bar, t.prev_parity))) return false;
      ptx::tc_fence_after();
      rescale_o(t.o_addr, factor);
    }
  }
  st.l_part += sum0 + sum1;
  ptx::tmem_wait_st();
  TPSA_TILE_TR(t, 34);
  return true;
}

// Writes columns [col, col + 32) of the 32 output rows of a softmax warp as
// bf16 (values times `scale`).  Each thread holds one row, and its 64 bytes
// are one half of a 128-byte line of `out`; storing them directly would make
// every store instruction touch 32 lines.  The warp instead passes the rows
// through its 2 KB staging buffer (16-byte chunks XOR-swizzled so both the
// writes and the reads are bank-conflict free) and each store instruction
// then writes 64 contiguous bytes of 8 rows.  Warp row R is query token
// base_q + R / 2, head base_h + R % 2; rows at or past query_tokens are not
// written.  All 32 lanes must call this.
__device__ __forceinline__ void store_rows_bf16(const float (&o)[32], float scale, uint8_t* stage,
                                                int lane, __nv_bfloat16* out, int32_t base_q,
                                                int32_t base_h, int32_t hq, int32_t query_tokens,
                                                int32_t col) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 v = make_uint4(pack_bf16x2(o[8 * j] * scale, o[8 * j + 1] * scale),
                               pack_bf16x2(o[8 * j + 2] * scale, o[8 * j + 3] * scale),
                               pack_bf16x2(o[8 * j + 4] * scale, o[8 * j + 5] * scale),
                               pack_bf16x2(o[8 * j + 6] * scale, o[8 * j + 7] * scale));
    *reinterpret_cast<uint4*>(stage + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = v;
  }
  __syncwarp();
  const int c = lane & 3;
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const int rr = 8 * jj + (lane >> 2);
    const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 64 + ((c ^ ((rr >> 1) & 3)) << 4));
    const int32_t q = base_q + (rr >> 1);
    if (q < query_tokens) {
      *reinterpret_cast<uint4*>(out + (static_cast<size_t>(q) * hq + base_h + (rr & 1)) * kHeadDim +
                                col + 8 * c) = v;
    }
  }
  __syncwarp();
}

// One arrival per softmax warp on a CTA-0 barrier.
__device__ __forceinline__ void warp_arrive0(const Shared& sh, uint32_t id, int lane) {
  __syncwarp();
  if (lane == 0) ptx::mbar_arrive_cluster(sh.bar0(id));
}

// Softmax warpgroup `wg` (warps 4-7: wg 0, warps 8-11: wg 1; warp % 4 is
// the tensor-memory lane quadrant, so each warpgroup covers all 128 rows).
// Tile gt of the pair's tile stream (in S buffer gt % 3) belongs to
// warpgroup gt % 2.  The two warpgroups share the O accumulator and hand
// each row's lazy reference max from tile to tile through RowChannel, so
// P of every tile is relative to the reference O is kept in; each keeps a
// partial row sum over its own tiles.  The warpgroup that owns an item's
// last tile finishes the item: the other hands over its (reference, partial
// sum) and goes on to the next item, and the owner normalises and writes
// all 128 O columns.
template <bool kVisit, bool kVarlen>
__device__ void softmax_role(const KernelArgs& a, const Shared& sh, uint32_t tmem) {
  const tpsa_plan& p = a.plan;
  const uint32_t r = sh.rank;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int wg = (warp - kFirstSoftmaxWarp) / 4;
  const int quad = warp % 4;
  const int row = quad * 32 + lane;  // TMEM lane == row of this CTA's M half
  const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
  const int32_t hq = p.kv_heads * kGroupSize;
  const bool visit = kVisit && a.visited != nullptr;
  // Tiles of the pair's stream before the current item.
  uint32_t g = 0;
  // Split items so far.
  uint32_t split_items = 0;
  RowChannel ch;
  static_assert(kCntCon == kCntPub + 8, "read counters follow the publication counters");
  ch.mine = sh.base_u32 + kOffXchg + (wg * kChanSlots * 128 + row) * 4;
  ch.theirs = sh.base_u32 + kOffXchg + ((1 - wg) * kChanSlots * 128 + row) * 4;
  ch.pub_cnt = sh.counter(kCntPub + wg * 4 + quad);
  ch.peer_pub = sh.counter(kCntPub + (1 - wg) * 4 + quad);
  ch.n_pub = 0;
  ch.n_read = 0;
  volatile int* split_last = reinterpret_cast<volatile int*>(sh.base + kOffSplitLast);
  uint32_t tr_sm = 0;  // trace counter (used only with TPSA_TRACE)
#define tr_n_ tr_sm
  const uint32_t o_all = tmem + lane_base + kTmemO;  // O, 128 columns

  for (uint32_t n_item = 0;; ++n_item) {
    ItemRec rec;
    const bool got = take_item(sh, n_item, &rec);
    if (!__all_sync(0xffffffffu, got)) break;
    __syncwarp();
    if (lane == 0) release_item(sh, n_item);
    if (rec.idx >= p.total_items) break;
    const uint32_t qb = n_item & 1;  // this item's Q buffer (items alternate)
    const tpsa_item& it = rec.it;
    const BlockTiles& bt = rec.bt;
    // The item's request (a batch-one launch has one, at row, item, slot and
    // counter 0).
    const ReqDesc& rq = a.reqs[kVarlen ? rec.req() : 0];
    const tpsa_plan& pr = kVarlen ? rq.plan : p;
    const int32_t q_row0 = kVarlen ? rq.q_row0 : 0;
    const int32_t ridx = kVarlen ? rec.idx - rq.item_base : rec.idx;  // item within its request
    const int32_t tok = bt.q_begin + row / 2;
    const int32_t q = tok < pr.seq_len ? tok : pr.seq_len - 1;
    const bool sparse = row_is_sparse(pr, tok);
    const int32_t qrow = it.block * kBlockQ + row / 2;  // row within the request's chunk
    const int32_t head = it.kv_head * kGroupSize + 2 * static_cast<int32_t>(r) + (row & 1);
    const bool real_row = qrow < pr.query_tokens;
    uint32_t* visit_row =
        (visit && real_row)
            ? a.visited + (static_cast<size_t>(qrow) * hq + head) * a.words_per_row
            : nullptr;
    RowState st{-INFINITY, 0.0f};
    bool ok = true;
    const int32_t ntiles = it.tile_end - it.tile_begin;
    for (int32_t n = (g + wg) & 1; n < ntiles; n += 2) {
      const uint32_t gt = g + static_cast<uint32_t>(n);
      const uint32_t sb = gt % kNumSBufs;
      int32_t k0, w;
      tile_keys(bt, it.tile_begin + n, &k0, &w);
      const bool masked = tile_needs_mask(pr, bt, k0, w);
      TileArgs ta;
      ta.s_addr = tmem + lane_base + (sb << 7);
      ta.o_addr = o_all;
      ta.k0 = k0;
      ta.wide = w > 64;
      ta.first = n == 0;
      ta.last = n == ntiles - 1;
      ta.prev_bar = sh.bar(kBarPvDone + (gt - 1) % kNumSBufs);
      ta.prev_parity = ((gt - 1) / kNumSBufs) & 1;
      ta.trn = row == 0 ? &tr_sm : nullptr;
      ta.trole = 2 + wg + 3 * r;
      const bool w_ok = wait_bar(sh, sh.bar(kBarSFull + sb), (gt / kNumSBufs) & 1);
      if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
      if (row == 0) TPSA_TR(2 + wg + 3 * r, 1, n);
      ptx::tc_fence_after();
      // One instantiation for masked and unmasked tiles (a uniform branch
      // around the masking): a second copy of this code would compete with
      // the MMA issuer's loop for the instruction cache.
      ta.masked = masked;
      const bool t_ok =
          softmax_tile<kVisit>(sh, p, ta, q, sparse, ch, st, visit_row, a.words_per_row);
      if (!t_ok) { ok = false; break; }
      ptx::tc_fence_before();
      if (row == 0) TPSA_TR(2 + wg + 3 * r, 3, n);
      warp_arrive0(sh, kBarPFull + sb, lane);
    }
    if (!ok) break;
    g += static_cast<uint32_t>(ntiles);

    // Item end.  The warpgroup that owned the item's last tile (the owner)
    // finishes the item alone: its reference is final, and the other
    // warpgroup, if it owned any tile of the item, hands over its reference
    // and partial row sum and goes on to the next item at once (whose first
    // tile is its own), so the next item's first P does not wait for this
    // epilogue.  O is complete once the item's last PV has.
    const uint32_t gl = g - 1;
    const bool owner = (gl & 1) == static_cast<uint32_t>(wg);
    const bool shared_item = ntiles >= 2;
    const bool split = it.num_splits > 1;
    const uint32_t sp_slot = split_items & 1;
    split_items += split ? 1u : 0u;
    if (!owner) {
      if (shared_item && !(ch.publish(sh, st.m_ref) && ch.publish(sh, st.l_part))) break;
      continue;
    }
    float l_total = st.l_part;
    if (shared_item) {
      float m_peer, l_peer;
      if (!ch.read(sh, &m_peer) || !ch.read(sh, &l_peer)) break;
      // The peer's reference is at most the final one (references only grow).
      if (m_peer != -INFINITY) l_total += l_peer * mufu_exp2((m_peer - st.m_ref) * p.scale_log2);
    }
    if (!__all_sync(0xffffffffu, wait_bar(sh, sh.bar(kBarPvDone + gl % kNumSBufs),
                                          (gl / kNumSBufs) & 1))) {
      break;
    }
    ptx::tc_fence_after();
    if (row == 0) TPSA_TR(2 + wg + 3 * r, 9, 0);
    float* slot =
        a.scratch + static_cast<size_t>((kVarlen ? rq.slot_base : 0) + ridx) * kSlotFloats;
    constexpr int32_t kSlotRows = 2 * kRowsPerTile;
    const int32_t srow = static_cast<int32_t>(r) * kRowsPerTile + row;
    // Output rows of this warp: packed token base_q + R / 2, head
    // base_h + R % 2 for warp row R; rows at or past row_end are not written.
    const int32_t base_q = q_row0 + it.block * kBlockQ + quad * 16;
    const int32_t base_h = it.kv_head * kGroupSize + 2 * static_cast<int32_t>(r);
    const int32_t row_end = q_row0 + pr.query_tokens;
    uint8_t* stage = sh.base + kOffStage + (warp - kFirstSoftmaxWarp) * kStageBytesPerWarp;
    if (kVarlen && !split && bt.q_end - bt.q_begin < kBlockQ) {
      // A block that ends inside its 64-token box (a request's last block):
      // a TMA store of the box would also write rows of the next packed
      // request, so these rows are stored one by one.  (In a batch-one
      // launch the tensor map's end clips the last box.)
      const float inv = 1.0f / l_total;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t x[32];
        ptx::tmem_ld32(o_all + 32 * c, x);
        ptx::tmem_wait_ld_regs(x);
        float o[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = __uint_as_float(x[j]);
        store_rows_bf16(o, inv, stage, lane, a.out, base_q, base_h, hq, row_end, 32 * c);
      }
      ptx::tc_fence_before();
      warp_arrive0(sh, kBarOEmpty, lane);
      if (row == 0) TPSA_TR(2 + wg + 3 * r, 5, 0);
      continue;
    }
    if (!split) {
      // The 128 output columns, as bf16, into the item's Q buffer, which is
      // dead (its QKs completed before the last PV) and has the output tile's
      // shape (per d-half, [64 tokens x 2 heads] rows of 64 d, 128-byte
      // swizzled as the Q tensor map loads it).
      const float inv = 1.0f / l_total;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint8_t* dst = sh.base + kOffQ + qb * kQBytes + (c >> 1) * kQHalfBytes + row * 128;
        uint32_t x[32];
        ptx::tmem_ld32(o_all + 32 * c, x);
        ptx::tmem_wait_ld_regs(x);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = 4 * (c & 1) + jj;  // 16-byte chunk within the d-half row
          const uint32_t* v = &x[8 * jj];
          *reinterpret_cast<uint4*>(dst + ((j ^ (row & 7)) << 4)) = make_uint4(
              pack_bf16x2(__uint_as_float(v[0]) * inv, __uint_as_float(v[1]) * inv),
              pack_bf16x2(__uint_as_float(v[2]) * inv, __uint_as_float(v[3]) * inv),
              pack_bf16x2(__uint_as_float(v[4]) * inv, __uint_as_float(v[5]) * inv),
              pack_bf16x2(__uint_as_float(v[6]) * inv, __uint_as_float(v[7]) * inv));
        }
      }
      // The K producer stores the staged box (TMA) before it reuses this Q
      // buffer; it counts four warps per d-half.  Each warp releases O only
      // after its staged counts: the next item's counts need its PVs, which
      // need O, so every count of this item lands before any of the next.
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        ptx::red_release_add_shared(sh.counter(kCntStaged + 0), 1);
        ptx::red_release_add_shared(sh.counter(kCntStaged + 1), 1);
      }
      ptx::tc_fence_before();
      warp_arrive0(sh, kBarOEmpty, lane);
      if (row == 0) TPSA_TR(2 + wg + 3 * r, 5, 0);
      continue;
    }

    // Split item: the fp32 partial (128 columns) into the item's
    // column-major slot ([128 columns][256 rows], then m[256] and l[256]);
    // the last split of the block (per CTA of the pair) merges all partials
    // and writes bf16.  Each split item counts four warps (its owner's).
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t x[32];
      ptx::tmem_ld32(o_all + 32 * c, x);
      ptx::tmem_wait_ld_regs(x);
      float* col = slot + static_cast<size_t>(32 * c) * kSlotRows + srow;
#pragma unroll
      for (int j = 0; j < 32; ++j) col[j * kSlotRows] = __uint_as_float(x[j]);
    }
    slot[kHeadDim * kSlotRows + srow] = st.m_ref;
    slot[(kHeadDim + 1) * kSlotRows + srow] = l_total;
    __threadfence();
    __syncwarp();
    if (lane == 0) ptx::red_release_add_shared(sh.counter(kCntSplitW), 1);
    if (row == 0) {
      if (wait_count(sh, kCntSplitW, 4 * split_items)) {
        int32_t* ctr = a.ctl + kCtlSplitBase + (kVarlen ? rq.ctr_base : 0) +
                       ((it.block - pr.tail_block0) * p.kv_heads + it.kv_head) * 2 + r;
        const int prev = atomicAdd(ctr, 1);
        split_last[sp_slot] = prev == it.num_splits - 1;
        ptx::red_release_add_shared(sh.counter(kCntSplitD), 1);
      }
    }
    const bool decided = __all_sync(0xffffffffu, wait_count(sh, kCntSplitD, split_items));
    const bool last_split = decided && split_last[sp_slot];
    ptx::tc_fence_before();
    warp_arrive0(sh, kBarOEmpty, lane);
    if (!decided) break;
    if (!last_split) continue;
    __threadfence();
    const float* first_slot = slot - static_cast<size_t>(it.split) * kSlotFloats;
    const size_t m_off = static_cast<size_t>(kHeadDim) * kSlotRows + srow;
    const size_t l_off = static_cast<size_t>(kHeadDim + 1) * kSlotRows + srow;
    float mmax = -INFINITY;
    for (int32_t sp = 0; sp < it.num_splits; ++sp) {
      mmax = fmaxf(mmax, __ldcg(first_slot + sp * kSlotFloats + m_off));
    }
    float lsum = 0.0f;
    for (int32_t sp = 0; sp < it.num_splits; ++sp) {
      const float* sl = first_slot + sp * kSlotFloats;
      const float ms = __ldcg(sl + m_off);
      if (ms != -INFINITY) lsum += mufu_exp2((ms - mmax) * p.scale_log2) * __ldcg(sl + l_off);
    }
    const float inv_sum = 1.0f / lsum;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      const int col = 32 * c;
      float acc[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
#pragma unroll 1
      for (int32_t sp = 0; sp < it.num_splits; ++sp) {
        const float* sl = first_slot + sp * kSlotFloats;
        const float ms = __ldcg(sl + m_off);
        const float wgt = ms == -INFINITY ? 0.0f : mufu_exp2((ms - mmax) * p.scale_log2);
        const float* colp = sl + static_cast<size_t>(col) * kSlotRows + srow;
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] += wgt * __ldcg(colp + j * kSlotRows);
      }
      store_rows_bf16(acc, inv_sum, stage, lane, a.out, base_q, base_h, hq, row_end, col);
    }
  }
}
#undef tr_n_

template <bool kVisit, bool kVarlen>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kNumThreads, 1)
    tpsa_paged_kernel(const __grid_constant__ KernelArgs args,
                      const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_k64,
                      const __grid_constant__ CUtensorMap tmap_k32,
                      const __grid_constant__ CUtensorMap tmap_v,
                      const __grid_constant__ CUtensorMap tmap_out) {
  extern __shared__ uint8_t smem_raw[];
  Shared sh;
  {
    const uint32_t raw = ptx::smem_u32(smem_raw);
    const uint32_t aligned = (raw + 1023u) & ~1023u;
    sh.base = smem_raw + (aligned - raw);
    sh.base_u32 = aligned;
    sh.rank = ptx::cluster_ctarank();
  }
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(sh.bar(kBarQFull + i), 2);
      ptx::mbar_init(sh.bar(kBarQEmpty + i), kQEmptyArrivals);
      ptx::mbar_init(sh.bar(kBarItemFull + i), 1);
      ptx::mbar_init(sh.bar(kBarItemEmpty + i), kItemConsumers);
    }
    for (int s = 0; s < kRing; ++s) {
      ptx::mbar_init(sh.bar(kBarKFull + s), 2);
      ptx::mbar_init(sh.bar(kBarKEmpty + s), 1);
      ptx::mbar_init(sh.bar(kBarVFull + s), 2);
      ptx::mbar_init(sh.bar(kBarVEmpty + s), 1);
    }
    for (uint32_t i = 0; i < kNumSBufs; ++i) {
      ptx::mbar_init(sh.bar(kBarSFull + i), 1);
      ptx::mbar_init(sh.bar(kBarPFull + i), kPairWgArrivals);
      ptx::mbar_init(sh.bar(kBarPvDone + i), 1);
    }
    ptx::mbar_init(sh.bar(kBarOEmpty), kPairWgArrivals);
    ptx::mbar_init(sh.bar(kBarTail), 1);
    ptx::mbar_init(sh.bar(kBarDrain), 1);
    *sh.abort_flag() = 0;
    for (uint32_t i = 0; i < kNumCounters; ++i) {
      *reinterpret_cast<volatile uint32_t*>(sh.base + kOffCounters + 4 * i) = 0;
    }
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(sh.base_u32 + kOffTmemSlot, kTmemCols);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync();  // barriers of both CTAs initialised before any remote use
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sh.base + kOffTmemSlot);

  if (warp < kFirstSoftmaxWarp) {
    ptx::setmaxnreg_dec<kControlRegs>();
    if (warp == 0) {
      if (lane == 0) {
        producer_role<kVarlen>(args, sh, &tmap_q, &tmap_k64, &tmap_k32, &tmap_v, &tmap_out,
                               false);
      }
      __syncwarp();
    } else if (warp == 1) {
      if (sh.rank == 0) mma_role(args, sh, tmem, lane);
    } else if (warp == 2 && sh.rank == 0) {
      // The scheduler has a warp of its own: it spins on the item ring, and
      // a lane of a busy warp would compete with that warp's work.
      if (lane == 0) scheduler_role<kVarlen>(args, sh);
      __syncwarp();
    } else if (warp == 3) {
      if (lane == 0) {
        producer_role<kVarlen>(args, sh, &tmap_q, &tmap_k64, &tmap_k32, &tmap_v, &tmap_out,
                               true);
      }
      __syncwarp();
    }
  } else {
    ptx::setmaxnreg_inc<kSoftmaxRegs>();
    softmax_role<kVisit, kVarlen>(args, sh, tmem);
  }

  ptx::tc_fence_before();
  ptx::cluster_sync();  // no remote traffic after this point; MMAs drained
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem, kTmemCols);
  }
}

#include "tpsa_solo_kernel.cuh"

// ================================================================ host side
thread_local std::string t_last_error;

tpsa_status fail(tpsa_status s, const std::string& msg) {
  t_last_error = "[TPSA] " + msg;
  return s;
}

// Dense-tail blocks longer than this fraction of the average work per CTA
// pair are split into several items (merged in-kernel).
#ifndef TPSA_SPLIT_FACTOR
#define TPSA_SPLIT_FACTOR 0.7
#endif
constexpr double kSplitFactor = TPSA_SPLIT_FACTOR;

// Split threshold (tiles per item) for the dense-tail blocks of a plan.  The
// B = tail blocks x kv heads longest items, each cut into ns pieces of
// ceil(T / ns) tiles, go first to the CTA pairs (longest first), so the
// busiest pair carries ceil(B ns / P) pieces; the short items fill the other
// pairs.  The estimated makespan, in tiles, is
//   max(ceil(B ns / P) (ceil(T / ns) + c), (total + B ns c) / P)
// with c the per-piece cost of a partial write and its share of the merge
// (kSplitPieceTiles); the smallest ns with the least estimate wins.  ns is
// at most what a threshold of kSplitFactor times the average work per pair
// gives, so no plan needs more split slots than that rule (the static-scratch
// entry point's limit rests on it).  (That rule alone cut the 128K-context
// tail into 5 pieces: 80 pieces for 74 pairs, six pairs with two.)
constexpr double kSplitPieceTiles = 2.0;
// `longest`: tiles of the longest dense-tail block; `tail`: dense-tail
// (block, head) items before splitting; `tiles`: all tiles of the launch.
int32_t choose_split_counts(int32_t longest, int64_t tail, int64_t tiles, int32_t pairs) {
  if (tail == 0 || longest == 0) return 1 << 30;
  const int32_t by_fraction = max_i(kMinSplitTiles, static_cast<int32_t>(
      kSplitFactor * static_cast<double>(tiles) / pairs));
  const int32_t ns_max = min_i(64, ceil_div(longest, by_fraction));
  double best = 0.0;
  int32_t best_ns = 1;
  for (int32_t ns = 1; ns <= ns_max; ++ns) {
    const double piece = static_cast<double>(ceil_div(longest, ns)) + kSplitPieceTiles;
    const double rounds = static_cast<double>((tail * ns + pairs - 1) / pairs);
    const double avg = (static_cast<double>(tiles) + kSplitPieceTiles * tail * ns) / pairs;
    const double est = std::max(rounds * piece, avg);
    if (ns == 1 || est < best - 1e-9) {
      best = est;
      best_ns = ns;
    }
  }
  return best_ns == 1 ? (1 << 30) : ceil_div(longest, best_ns);
}

int32_t choose_split(const tpsa_plan& p, int32_t b0, int64_t tiles, int32_t pairs) {
  int32_t longest = 0;
  for (int32_t b = b0; b < p.num_blocks; ++b) longest = max_i(longest, block_tiles(p, b).count);
  return choose_split_counts(longest, static_cast<int64_t>(p.num_blocks - b0) * p.kv_heads, tiles,
                             pairs);
}

tpsa_status cuda_fail(cudaError_t e, const char* what) {
  return fail(TPSA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Kernel form: one CTA per item (tpsa_solo_kernel, the default) or CTA pairs
// (tpsa_paged_kernel, selected by TPSA_KERNEL=pair in the environment; kept
// as the measured comparison).  Read once per process.
enum class Form { kPair, kSolo };

Form kernel_form() {
  static const Form form = [] {
    const char* e = std::getenv("TPSA_KERNEL");
    if (e != nullptr && std::strcmp(e, "pair") == 0) return Form::kPair;
    return Form::kSolo;
  }();
  return form;
}

struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  int major = 0;
  bool attr_set = false;
  int max_pairs = 0;  // co-resident CTA pairs (clusters of 2)
  int max_solo = 0;   // co-resident solo CTAs
  // Parallel workers of the current kernel form (CTA pairs or solo CTAs)
  // and CTAs per worker.
  int workers() const { return kernel_form() == Form::kSolo ? max_solo : max_pairs; }
};

int ctas_per_worker() { return kernel_form() == Form::kSolo ? 1 : 2; }

std::mutex g_mutex;
DeviceState g_devices[64];

tpsa_status device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(TPSA_ERR_CUDA, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState& st = g_devices[dev];
  if (!st.ready) {
    e = cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    e = cudaDeviceGetAttribute(&st.major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(major)");
    st.ready = true;
  }
  if (st.major != 10) {
    return fail(TPSA_ERR_UNSUPPORTED_DEVICE,
                "the kernel is built for sm_100a (B200); current device is not");
  }
  if (!st.attr_set) {
    e = cudaFuncSetAttribute(tpsa_paged_kernel<false, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    e = cudaFuncSetAttribute(tpsa_paged_kernel<true, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    e = cudaFuncSetAttribute(tpsa_paged_kernel<false, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (st.sm_count / 2), 1, 1);
    cfg.blockDim = dim3(kNumThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, tpsa_paged_kernel<false, false>, &cfg);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
    if (clusters <= 0) return fail(TPSA_ERR_CUDA, "no CTA pair fits on this device");
    st.max_pairs = clusters;
    e = cudaFuncSetAttribute(tpsa_solo_kernel<false, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, solo::kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    e = cudaFuncSetAttribute(tpsa_solo_kernel<true, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, solo::kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    e = cudaFuncSetAttribute(tpsa_solo_kernel<false, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, solo::kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tpsa_solo_kernel<false, false>,
                                                      solo::kNumThreads, solo::kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (per_sm <= 0) return fail(TPSA_ERR_CUDA, "the solo kernel does not fit on an SM");
    st.max_solo = per_sm * st.sm_count;
    st.attr_set = true;
  }
  *out = &st;
  return TPSA_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

tpsa_status encode_fn(EncodeTiledFn* fn) {
  static EncodeTiledFn cached = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) {
      cached = reinterpret_cast<EncodeTiledFn>(f);
    }
  });
  if (cached == nullptr) {
    return fail(TPSA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  }
  *fn = cached;
  return TPSA_OK;
}

// 3-D bf16 tensor map {128 (d), d1, d2}, SWIZZLE_128B, zero fill outside.
tpsa_status encode_map(CUtensorMap* map, const void* base, uint64_t d1, uint64_t d2,
                       uint32_t box1, uint32_t box2) {
  EncodeTiledFn fn = nullptr;
  tpsa_status st = encode_fn(&fn);
  if (st != TPSA_OK) return st;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), d1, d2};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHeadDim) * 2,
                                 static_cast<cuuint64_t>(kHeadDim) * 2 * d1};
  const cuuint32_t box[3] = {64, box1, box2};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base),
                        dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(TPSA_ERR_INVALID_ARGUMENT,
                "cuTensorMapEncodeTiled rejected a tensor (alignment or extent)");
  }
  return TPSA_OK;
}

// `pairs`: parallel workers the launch runs (CTA pairs, or single CTAs for the
// solo kernel, ctas_per_worker() CTAs each); each worker runs one item at a
// time.
// `split_override` > 0 replaces the split threshold derived from this
// request's own work (a varlen launch derives it from the whole launch).
tpsa_status build_plan(int64_t query_tokens, int64_t query_start, int64_t seq_len,
                       int64_t prompt_len, int32_t kv_heads, int32_t pairs,
                       float scale, tpsa_plan* p, int32_t split_override = 0) {
  if (p == nullptr) return fail(TPSA_ERR_INVALID_ARGUMENT, "plan pointer is NULL");
  if (!(kv_heads == 1 || kv_heads == 2 || kv_heads == 4 || kv_heads == 8)) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "kv_heads must be 1, 2, 4 or 8");
  }
  if (query_start < 0 || seq_len <= 0 || prompt_len < seq_len || !std::isfinite(scale) ||
      scale <= 0.0f) {
    return fail(TPSA_ERR_INVALID_ARGUMENT,
                "invalid query_start/seq_len/prompt_len/scale attributes");
  }
  if (query_tokens <= 0 || query_start + query_tokens != seq_len) {
    return fail(TPSA_ERR_INVALID_ARGUMENT,
                "batch-one prefill requires query_start + Tq == seq_len");
  }
  if (seq_len > kMaxSeqLen) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "seq_len above the supported 2^30");
  }
  if (prompt_len > static_cast<int64_t>(UINT32_MAX)) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "prompt lengths above UINT32_MAX are unsupported");
  }
  if (pairs <= 0) return fail(TPSA_ERR_INVALID_ARGUMENT, "sm_count must be positive");
  std::memset(p, 0, sizeof(*p));
  p->query_tokens = static_cast<int32_t>(query_tokens);
  p->query_start = static_cast<int32_t>(query_start);
  p->seq_len = static_cast<int32_t>(seq_len);
  p->sparse_begin = kSparseBegin;
  const int64_t se = prompt_len - kDenseTail > 0 ? prompt_len - kDenseTail : 0;
  p->sparse_end = static_cast<int32_t>(se < seq_len ? se : seq_len);
  p->kv_heads = kv_heads;
  p->num_blocks = ceil_div(p->query_tokens, kBlockQ);
  p->scale = scale;
  p->scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  int32_t b0 = p->num_blocks;
  while (b0 > 0 && block_tiles(*p, b0 - 1).q_end > p->sparse_end) --b0;
  p->tail_block0 = b0;
  int64_t tiles = 0;
  for (int32_t b = 0; b < p->num_blocks; ++b) tiles += block_tiles(*p, b).count;
  tiles *= kv_heads;
  int32_t split = split_override > 0 ? split_override : choose_split(*p, b0, tiles, pairs);
  if (split < kMinSplitTiles) split = kMinSplitTiles;
  // The in-kernel merge keeps per-split weights for at most 64 splits.
  for (int32_t b = b0; b < p->num_blocks; ++b) {
    const int32_t c = block_tiles(*p, b).count;
    if (ceil_div(c, split) > 64) split = ceil_div(c, 64);
  }
  if ((p->num_blocks - b0) * kv_heads * 2 > kMaxSplitCounters) split = 1 << 30;
  p->split_tiles = split;
  int64_t tail_items = 0;
  bool any_split = false;
  for (int32_t b = b0; b < p->num_blocks; ++b) {
    const int32_t ns = block_splits(*p, block_tiles(*p, b).count);
    any_split = any_split || ns > 1;
    tail_items += static_cast<int64_t>(ns) * kv_heads;
  }
  p->tail_items = static_cast<int32_t>(tail_items);
  p->total_items = static_cast<int32_t>(tail_items + static_cast<int64_t>(b0) * kv_heads);
  p->grid = ctas_per_worker() * (p->total_items < pairs ? p->total_items : pairs);
  p->total_tiles = tiles;
  p->workspace_bytes = kControlBytes + (any_split ? tail_items * kSlotBytes : 0);
  return TPSA_OK;
}

tpsa_status launch(const void* query, const void* key_cache, const void* value_cache,
                   const int32_t* block_table, void* out, int64_t query_tokens,
                   int64_t num_pages, int64_t table_cols, int64_t query_start,
                   int64_t seq_len, int64_t prompt_len, float scale, int32_t kv_heads,
                   void* workspace, uint64_t workspace_bytes, uint32_t* visited,
                   uint64_t* tile_counter, void* stream) {
  t_last_error.clear();
  if (query == nullptr || key_cache == nullptr || value_cache == nullptr ||
      block_table == nullptr || out == nullptr) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  }
  if (num_pages <= 0 || num_pages > (int64_t{1} << 24)) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "num_pages must be in [1, 2^24]");
  }
  const int64_t required_pages = (seq_len + kPageSize - 1) / kPageSize;
  if (table_cols < required_pages) {
    return fail(TPSA_ERR_INVALID_ARGUMENT,
                "block_table lacks logical pages required by seq_len");
  }
  DeviceState* dev = nullptr;
  tpsa_status st = device_state(&dev);
  if (st != TPSA_OK) return st;
  KernelArgs args;
  std::memset(&args, 0, sizeof(args));
  st = build_plan(query_tokens, query_start, seq_len, prompt_len, kv_heads, dev->workers(),
                  scale, &args.plan);
  if (st != TPSA_OK) return st;
  const tpsa_plan& p = args.plan;
  if (workspace == nullptr || workspace_bytes < static_cast<uint64_t>(p.workspace_bytes)) {
    return fail(TPSA_ERR_WORKSPACE, "workspace smaller than tpsa_workspace_size()");
  }
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) {
    return fail(TPSA_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  }
  for (const void* ptr : {query, key_cache, value_cache, static_cast<const void*>(out)}) {
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) {
      return fail(TPSA_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
    }
  }
  CUtensorMap tq, tk64, tk32, tv;
  const uint64_t hq = static_cast<uint64_t>(kv_heads) * kGroupSize;
  const uint64_t cache_tokens = static_cast<uint64_t>(num_pages) * kPageSize;
  st = encode_map(&tq, query, hq, static_cast<uint64_t>(query_tokens), 2, kBlockQ);
  if (st != TPSA_OK) return st;
  st = encode_map(&tk64, key_cache, kv_heads, cache_tokens, 1, 64);
  if (st != TPSA_OK) return st;
  st = encode_map(&tk32, key_cache, kv_heads, cache_tokens, 1, 32);
  if (st != TPSA_OK) return st;
  st = encode_map(&tv, value_cache, kv_heads, cache_tokens, 1, 64);
  if (st != TPSA_OK) return st;
  CUtensorMap tout;  // output tile stores: the Q tile's shape over `out`
  st = encode_map(&tout, out, hq, static_cast<uint64_t>(query_tokens), 2, kBlockQ);
  if (st != TPSA_OK) return st;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  args.num_reqs = 1;
  args.reqs[0].plan = p;  // one request: item, row, table, slot and counter bases 0
  args.block_table = block_table;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.num_pages = static_cast<int32_t>(num_pages);
  args.ctl = static_cast<int32_t*>(workspace);
  args.scratch = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kControlBytes);
  // The work-item counter and split counters start at zero every launch.
  cudaError_t e = cudaMemsetAsync(workspace, 0, kControlBytes, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
  args.visited = visited;
  args.tiles = reinterpret_cast<unsigned long long*>(tile_counter);
  args.words_per_row = (p.seq_len + 31) / 32;

  const bool visit = visited != nullptr || tile_counter != nullptr;
  if (kernel_form() == Form::kSolo) {
    CUtensorMap tk128, tout16;  // whole 128-key K tiles; one softmax warp's output box
    st = encode_map(&tk128, key_cache, kv_heads, cache_tokens, 1, 128);
    if (st != TPSA_OK) return st;
    st = encode_map(&tout16, out, hq, static_cast<uint64_t>(query_tokens), 2, 16);
    if (st != TPSA_OK) return st;
    if (visit) {
      tpsa_solo_kernel<true, false><<<p.grid, solo::kNumThreads, solo::kSmemBytes, s>>>(
          args, tq, tk128, tk64, tv, tout16);
    } else {
      tpsa_solo_kernel<false, false><<<p.grid, solo::kNumThreads, solo::kSmemBytes, s>>>(
          args, tq, tk128, tk64, tv, tout16);
    }
  } else if (visit) {
    tpsa_paged_kernel<true, false><<<p.grid, kNumThreads, kSmemBytes, s>>>(args, tq, tk64, tk32,
                                                                            tv, tout);
  } else {
    tpsa_paged_kernel<false, false><<<p.grid, kNumThreads, kSmemBytes, s>>>(args, tq, tk64, tk32,
                                                                             tv, tout);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return TPSA_OK;
}

// ------------------------------------------------ varlen packed batch
// Requests [first, first + count) of a packed batch as one launch: each
// request keeps its own plan; the split threshold comes from the launch's
// whole work; split counters and partial slots are laid out request after
// request in the workspace.
struct BatchLaunch {
  KernelArgs args;
  int64_t ctl_bytes;        // zeroed control words (scheduler + split counters)
  int64_t workspace_bytes;  // control words + partial slots
};

tpsa_status build_batch(int32_t first, int32_t count, const int64_t* cu_seqlens_q,
                        const int64_t* seq_lens, const int64_t* prompt_lens, int32_t kv_heads,
                        int32_t pairs, float scale, int64_t table_cols, BatchLaunch* b) {
  std::memset(&b->args, 0, sizeof(b->args));
  KernelArgs& a = b->args;
  int64_t tiles = 0, tail_items = 0;
  int32_t longest = 0;
  for (int32_t i = 0; i < count; ++i) {
    const int32_t r = first + i;
    const int64_t tq = cu_seqlens_q[r + 1] - cu_seqlens_q[r];
    tpsa_plan probe;
    tpsa_status st = build_plan(tq, seq_lens[r] - tq, seq_lens[r], prompt_lens[r], kv_heads,
                                pairs, scale, &probe, 1 << 30);
    if (st != TPSA_OK) return st;
    tiles += probe.total_tiles;
    tail_items += static_cast<int64_t>(probe.num_blocks - probe.tail_block0) * kv_heads;
    for (int32_t b = probe.tail_block0; b < probe.num_blocks; ++b) {
      longest = max_i(longest, block_tiles(probe, b).count);
    }
  }
  // One split threshold for the launch, from the makespan estimate over all
  // requests' dense-tail items (which are dispatched first).
  int32_t split = choose_split_counts(longest, tail_items, tiles, pairs);
  if (split < kMinSplitTiles) split = kMinSplitTiles;
  int32_t items = 0, slots = 0, counters = 0, tail = 0, rest = 0;
  for (int32_t i = 0; i < count; ++i) {
    const int32_t r = first + i;
    const int64_t tq = cu_seqlens_q[r + 1] - cu_seqlens_q[r];
    ReqDesc& d = a.reqs[i];
    tpsa_status st = build_plan(tq, seq_lens[r] - tq, seq_lens[r], prompt_lens[r], kv_heads,
                                pairs, scale, &d.plan, split);
    if (st != TPSA_OK) return st;
    d.item_base = items;
    d.tail_base = tail;
    d.rest_base = rest;
    tail += d.plan.tail_items;
    rest += d.plan.total_items - d.plan.tail_items;
    d.q_row0 = static_cast<int32_t>(cu_seqlens_q[r]);
    d.table_off = static_cast<int32_t>(static_cast<int64_t>(r) * table_cols);
    d.slot_base = slots;
    d.ctr_base = counters;
    items += d.plan.total_items;
    if (d.plan.workspace_bytes > kControlBytes) {  // the request splits some block
      slots += d.plan.tail_items;
      counters += (d.plan.num_blocks - d.plan.tail_block0) * kv_heads * 2;
    }
  }
  a.num_reqs = count;
  a.tail_total = tail;
  a.plan = a.reqs[0].plan;
  a.plan.query_tokens = static_cast<int32_t>(cu_seqlens_q[first + count] - cu_seqlens_q[first]);
  a.plan.total_items = items;
  a.plan.total_tiles = tiles;
  a.plan.grid = ctas_per_worker() * (items < pairs ? items : pairs);
  const int64_t ctl = (int64_t{kCtlSplitBase} + counters) * 4;
  b->ctl_bytes = std::max<int64_t>(kControlBytes, (ctl + 255) / 256 * 256);
  b->workspace_bytes = b->ctl_bytes + static_cast<int64_t>(slots) * kSlotBytes;
  a.plan.workspace_bytes = b->workspace_bytes;
  return TPSA_OK;
}

tpsa_status check_batch(int32_t batch, const int64_t* cu_seqlens_q, const int64_t* seq_lens,
                        const int64_t* prompt_lens) {
  if (batch <= 0) return fail(TPSA_ERR_INVALID_ARGUMENT, "batch must be positive");
  if (cu_seqlens_q == nullptr || seq_lens == nullptr || prompt_lens == nullptr) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "a batch metadata pointer is NULL");
  }
  if (cu_seqlens_q[0] != 0) return fail(TPSA_ERR_INVALID_ARGUMENT, "cu_seqlens_q[0] must be 0");
  for (int32_t r = 0; r < batch; ++r) {
    const int64_t tq = cu_seqlens_q[r + 1] - cu_seqlens_q[r];
    if (tq <= 0) {
      return fail(TPSA_ERR_INVALID_ARGUMENT, "each ragged query length must be positive");
    }
    if (seq_lens[r] < tq) {
      return fail(TPSA_ERR_INVALID_ARGUMENT, "seq_lens[i] must cover the request's query rows");
    }
  }
  if (cu_seqlens_q[batch] > (int64_t{1} << 31) - 1) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "packed query rows above 2^31 - 1");
  }
  return TPSA_OK;
}

tpsa_status varlen_workspace(int32_t batch, const int64_t* cu_seqlens_q, const int64_t* seq_lens,
                             const int64_t* prompt_lens, int32_t kv_heads, int32_t pairs,
                             uint64_t* bytes) {
  tpsa_status st = check_batch(batch, cu_seqlens_q, seq_lens, prompt_lens);
  if (st != TPSA_OK) return st;
  std::unique_ptr<BatchLaunch> b(new BatchLaunch);
  int64_t most = kControlBytes;
  for (int32_t first = 0; first < batch; first += kMaxReqs) {
    const int32_t count = std::min(kMaxReqs, batch - first);
    st = build_batch(first, count, cu_seqlens_q, seq_lens, prompt_lens, kv_heads, pairs,
                     1.0f, 1, b.get());
    if (st != TPSA_OK) return st;
    most = std::max(most, b->workspace_bytes);
  }
  *bytes = static_cast<uint64_t>(most);
  return TPSA_OK;
}

tpsa_status launch_varlen(const void* query, const void* key_cache, const void* value_cache,
                          const int32_t* block_tables, void* out, int32_t batch,
                          const int64_t* cu_seqlens_q, const int64_t* seq_lens,
                          const int64_t* prompt_lens, int64_t num_pages, int64_t table_cols,
                          float scale, int32_t kv_heads, void* workspace,
                          uint64_t workspace_bytes, void* stream) {
  t_last_error.clear();
  if (query == nullptr || key_cache == nullptr || value_cache == nullptr ||
      block_tables == nullptr || out == nullptr) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  }
  if (num_pages <= 0 || num_pages > (int64_t{1} << 24)) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "num_pages must be in [1, 2^24]");
  }
  tpsa_status st = check_batch(batch, cu_seqlens_q, seq_lens, prompt_lens);
  if (st != TPSA_OK) return st;
  for (int32_t r = 0; r < batch; ++r) {
    if (table_cols < (seq_lens[r] + kPageSize - 1) / kPageSize) {
      return fail(TPSA_ERR_INVALID_ARGUMENT,
                  "block_tables lack logical pages required by seq_lens");
    }
  }
  if (static_cast<int64_t>(batch) * table_cols > (int64_t{1} << 31) - 1) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "block_tables above 2^31 - 1 entries");
  }
  if (workspace == nullptr || reinterpret_cast<uintptr_t>(workspace) % 256 != 0) {
    return fail(TPSA_ERR_WORKSPACE, "workspace must be non-NULL and 256-byte aligned");
  }
  for (const void* ptr : {query, key_cache, value_cache, static_cast<const void*>(out)}) {
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) {
      return fail(TPSA_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
    }
  }
  DeviceState* dev = nullptr;
  st = device_state(&dev);
  if (st != TPSA_OK) return st;
  if (!(kv_heads == 1 || kv_heads == 2 || kv_heads == 4 || kv_heads == 8)) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "kv_heads must be 1, 2, 4 or 8");
  }
  const uint64_t total_rows = static_cast<uint64_t>(cu_seqlens_q[batch]);
  CUtensorMap tq, tk64, tk32, tv, tout;
  const uint64_t hq = static_cast<uint64_t>(kv_heads) * kGroupSize;
  const uint64_t cache_tokens = static_cast<uint64_t>(num_pages) * kPageSize;
  st = encode_map(&tq, query, hq, total_rows, 2, kBlockQ);
  if (st != TPSA_OK) return st;
  st = encode_map(&tk64, key_cache, kv_heads, cache_tokens, 1, 64);
  if (st != TPSA_OK) return st;
  st = encode_map(&tk32, key_cache, kv_heads, cache_tokens, 1, 32);
  if (st != TPSA_OK) return st;
  st = encode_map(&tv, value_cache, kv_heads, cache_tokens, 1, 64);
  if (st != TPSA_OK) return st;
  st = encode_map(&tout, out, hq, total_rows, 2, kBlockQ);
  if (st != TPSA_OK) return st;
  CUtensorMap tk128, tout16;  // solo kernel: whole 128-key K tiles, one warp's output box
  st = encode_map(&tk128, key_cache, kv_heads, cache_tokens, 1, 128);
  if (st != TPSA_OK) return st;
  st = encode_map(&tout16, out, hq, total_rows, 2, 16);
  if (st != TPSA_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::unique_ptr<BatchLaunch> b(new BatchLaunch);
  // Launches of at most kMaxReqs requests each, in stream order; each
  // reuses the workspace after the previous one.
  for (int32_t first = 0; first < batch; first += kMaxReqs) {
    const int32_t count = std::min(kMaxReqs, batch - first);
    st = build_batch(first, count, cu_seqlens_q, seq_lens, prompt_lens, kv_heads,
                     dev->workers(), scale, table_cols, b.get());
    if (st != TPSA_OK) return st;
    if (workspace_bytes < static_cast<uint64_t>(b->workspace_bytes)) {
      return fail(TPSA_ERR_WORKSPACE, "workspace smaller than tpsa_varlen_workspace_size()");
    }
    KernelArgs& args = b->args;
    args.block_table = block_tables;
    args.out = static_cast<__nv_bfloat16*>(out);
    args.num_pages = static_cast<int32_t>(num_pages);
    args.ctl = static_cast<int32_t*>(workspace);
    args.scratch = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + b->ctl_bytes);
    cudaError_t e = cudaMemsetAsync(workspace, 0, static_cast<size_t>(b->ctl_bytes), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
    if (kernel_form() == Form::kSolo) {
      tpsa_solo_kernel<false, true><<<args.plan.grid, solo::kNumThreads, solo::kSmemBytes, s>>>(
          args, tq, tk128, tk64, tv, tout16);
    } else {
      tpsa_paged_kernel<false, true><<<args.plan.grid, kNumThreads, kSmemBytes, s>>>(
          args, tq, tk64, tk32, tv, tout);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  }
  return TPSA_OK;
}

// ------------------------------------------------ static-scratch variant
// Scratch for tpsa_paged_attention_static_scratch: the same control words and
// split-KV partial slots that tpsa_paged_attention keeps in a caller-provided
// workspace, in one module-global array per device instead.  Its maximum
// size, 24 MiB, covers every batch-one plan on a 148-SM B200: the split
// count stays near one piece per CTA, so no plan needs more than 144 partial
// slots (18.3 MiB; query chunks of 64 to 16384 rows over contexts to 4M).
constexpr uint64_t kStaticScratchBytes = uint64_t{24} << 20;
constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxScratchDevices] = {};

// Device address of the static scratch on the current device.  The first
// call on a device looks the address up (cudaGetSymbolAddress, which also
// makes the runtime load this module's device globals there) and caches it.
tpsa_status static_scratch_address(void** ptr);

}  // namespace

static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

namespace {

tpsa_status static_scratch_address(void** ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxScratchDevices) {
    return fail(TPSA_ERR_CUDA, "device ordinal out of range");
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
    if (p == nullptr) return fail(TPSA_ERR_CUDA, "static scratch has no device address");
    g_scratch_ptr[dev] = p;
  }
  *ptr = g_scratch_ptr[dev];
  return TPSA_OK;
}

}  // namespace
}  // namespace tpsa

// ================================================================ C ABI
using namespace tpsa;

extern "C" {

int32_t tpsa_abi_version(void) { return TPSA_ABI_VERSION; }

const char* tpsa_status_string(tpsa_status status) {
  switch (status) {
    case TPSA_OK: return "ok";
    case TPSA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TPSA_ERR_WORKSPACE: return "workspace missing or too small";
    case TPSA_ERR_CUDA: return "CUDA error";
    case TPSA_ERR_UNSUPPORTED_DEVICE: return "unsupported device (needs sm_100)";
    case TPSA_ERR_DEVICE_FAULT: return "device status word set";
  }
  return "unknown status";
}

const char* tpsa_last_error(void) { return t_last_error.c_str(); }

tpsa_status tpsa_make_plan(int64_t query_tokens, int64_t query_start, int64_t seq_len,
                           int64_t prompt_len, int32_t kv_heads, int32_t sm_count,
                           float scale, tpsa_plan* plan) {
  t_last_error.clear();
  int32_t pairs = sm_count / ctas_per_worker();  // workers of the kernel form
  if (sm_count <= 0) {
    DeviceState* dev = nullptr;
    tpsa_status st = device_state(&dev);
    if (st != TPSA_OK) return st;
    pairs = dev->workers();
  }
  return build_plan(query_tokens, query_start, seq_len, prompt_len, kv_heads, pairs, scale,
                    plan);
}

tpsa_status tpsa_plan_item(const tpsa_plan* plan, int32_t item, tpsa_item* out) {
  if (plan == nullptr || out == nullptr || item < 0 || item >= plan->total_items) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "item index out of range");
  }
  *out = decode_item(*plan, item);
  return TPSA_OK;
}

tpsa_status tpsa_plan_tile(const tpsa_plan* plan, int32_t block, int32_t tile,
                           int32_t* key_begin, int32_t* key_count, int32_t* needs_mask) {
  if (plan == nullptr || key_begin == nullptr || key_count == nullptr ||
      needs_mask == nullptr || block < 0 || block >= plan->num_blocks) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "block index out of range");
  }
  const BlockTiles bt = block_tiles(*plan, block);
  if (tile < 0 || tile >= bt.count) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "tile index out of range");
  }
  int32_t k0, w;
  tile_keys(bt, tile, &k0, &w);
  *key_begin = k0;
  *key_count = w;
  *needs_mask = tile_needs_mask(*plan, bt, k0, w) ? 1 : 0;
  return TPSA_OK;
}

tpsa_status tpsa_workspace_size(int64_t query_tokens, int64_t query_start, int64_t seq_len,
                                int64_t prompt_len, uint64_t* bytes) {
  t_last_error.clear();
  if (bytes == nullptr) return fail(TPSA_ERR_INVALID_ARGUMENT, "bytes pointer is NULL");
  tpsa_plan p;
  tpsa_status st = tpsa_make_plan(query_tokens, query_start, seq_len, prompt_len,
                                  TPSA_KV_HEADS, 0, 1.0f, &p);
  if (st != TPSA_OK) return st;
  *bytes = static_cast<uint64_t>(p.workspace_bytes);
  return TPSA_OK;
}

tpsa_status tpsa_paged_attention(const void* query, const void* key_cache,
                                 const void* value_cache, const int32_t* block_table,
                                 void* out, int64_t query_tokens, int64_t num_pages,
                                 int64_t table_cols, int64_t query_start, int64_t seq_len,
                                 int64_t prompt_len, float scale, void* workspace,
                                 uint64_t workspace_bytes, void* stream) {
  return launch(query, key_cache, value_cache, block_table, out, query_tokens, num_pages,
                table_cols, query_start, seq_len, prompt_len, scale, TPSA_KV_HEADS,
                workspace, workspace_bytes, nullptr, nullptr, stream);
}

tpsa_status tpsa_varlen_workspace_size(int32_t batch, const int64_t* cu_seqlens_q,
                                       const int64_t* seq_lens, const int64_t* prompt_lens,
                                       uint64_t* bytes) {
  t_last_error.clear();
  if (bytes == nullptr) return fail(TPSA_ERR_INVALID_ARGUMENT, "bytes pointer is NULL");
  DeviceState* dev = nullptr;
  tpsa_status st = device_state(&dev);
  if (st != TPSA_OK) return st;
  return varlen_workspace(batch, cu_seqlens_q, seq_lens, prompt_lens, TPSA_KV_HEADS,
                          dev->workers(), bytes);
}

tpsa_status tpsa_varlen_workspace_size_heads(int32_t batch, const int64_t* cu_seqlens_q,
                                             const int64_t* seq_lens, const int64_t* prompt_lens,
                                             int32_t kv_heads, uint64_t* bytes) {
  t_last_error.clear();
  if (bytes == nullptr) return fail(TPSA_ERR_INVALID_ARGUMENT, "bytes pointer is NULL");
  if (!(kv_heads == 1 || kv_heads == 2 || kv_heads == 4 || kv_heads == 8)) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "kv_heads must be 1, 2, 4 or 8");
  }
  DeviceState* dev = nullptr;
  tpsa_status st = device_state(&dev);
  if (st != TPSA_OK) return st;
  return varlen_workspace(batch, cu_seqlens_q, seq_lens, prompt_lens, kv_heads,
                          dev->workers(), bytes);
}

tpsa_status tpsa_paged_attention_varlen(const void* query, const void* key_cache,
                                        const void* value_cache, const int32_t* block_tables,
                                        void* out, int32_t batch, const int64_t* cu_seqlens_q,
                                        const int64_t* seq_lens, const int64_t* prompt_lens,
                                        int64_t num_pages, int64_t table_cols, float scale,
                                        void* workspace, uint64_t workspace_bytes,
                                        void* stream) {
  return launch_varlen(query, key_cache, value_cache, block_tables, out, batch, cu_seqlens_q,
                       seq_lens, prompt_lens, num_pages, table_cols, scale, TPSA_KV_HEADS,
                       workspace, workspace_bytes, stream);
}

tpsa_status tpsa_paged_attention_varlen_heads(
    const void* query, const void* key_cache, const void* value_cache,
    const int32_t* block_tables, void* out, int32_t batch, const int64_t* cu_seqlens_q,
    const int64_t* seq_lens, const int64_t* prompt_lens, int64_t num_pages, int64_t table_cols,
    float scale, int32_t kv_heads, void* workspace, uint64_t workspace_bytes, void* stream) {
  return launch_varlen(query, key_cache, value_cache, block_tables, out, batch, cu_seqlens_q,
                       seq_lens, prompt_lens, num_pages, table_cols, scale, kv_heads,
                       workspace, workspace_bytes, stream);
}

tpsa_status tpsa_paged_attention_heads(const void* query, const void* key_cache,
                                       const void* value_cache, const int32_t* block_table,
                                       void* out, int64_t query_tokens, int64_t num_pages,
                                       int64_t table_cols, int64_t query_start,
                                       int64_t seq_len, int64_t prompt_len, float scale,
                                       int32_t kv_heads, void* workspace,
                                       uint64_t workspace_bytes, void* stream) {
  return launch(query, key_cache, value_cache, block_table, out, query_tokens, num_pages,
                table_cols, query_start, seq_len, prompt_len, scale, kv_heads, workspace,
                workspace_bytes, nullptr, nullptr, stream);
}

tpsa_status tpsa_paged_attention_visit(const void* query, const void* key_cache,
                                       const void* value_cache, const int32_t* block_table,
                                       void* out, int64_t query_tokens, int64_t num_pages,
                                       int64_t table_cols, int64_t query_start,
                                       int64_t seq_len, int64_t prompt_len, float scale,
                                       int32_t kv_heads, void* workspace,
                                       uint64_t workspace_bytes, uint32_t* visited,
                                       uint64_t* tile_counter, void* stream) {
  if (visited == nullptr || tile_counter == nullptr) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "visited and tile_counter are required");
  }
  return launch(query, key_cache, value_cache, block_table, out, query_tokens, num_pages,
                table_cols, query_start, seq_len, prompt_len, scale, kv_heads, workspace,
                workspace_bytes, visited, tile_counter, stream);
}

tpsa_status tpsa_paged_attention_static_scratch(const void* query, const void* key_cache,
                                                const void* value_cache,
                                                const int32_t* block_table, void* out,
                                                int64_t query_tokens, int64_t num_pages,
                                                int64_t table_cols, int64_t query_start,
                                                int64_t seq_len, int64_t prompt_len, float scale,
                                                void* stream) {
  t_last_error.clear();
  DeviceState* dev = nullptr;
  tpsa_status st = device_state(&dev);
  if (st != TPSA_OK) return st;
  tpsa_plan p;
  st = build_plan(query_tokens, query_start, seq_len, prompt_len, TPSA_KV_HEADS, dev->workers(),
                  scale, &p);
  if (st != TPSA_OK) return st;
  if (static_cast<uint64_t>(p.workspace_bytes) > kStaticScratchBytes) {
    return fail(TPSA_ERR_WORKSPACE,
                "this call needs " + std::to_string(p.workspace_bytes) +
                    " bytes of scratch; the static scratch holds " +
                    std::to_string(kStaticScratchBytes) +
                    " bytes (24 MiB): use tpsa_paged_attention with a caller workspace");
  }
  void* scratch = nullptr;
  st = static_scratch_address(&scratch);
  if (st != TPSA_OK) return st;
  return launch(query, key_cache, value_cache, block_table, out, query_tokens, num_pages,
                table_cols, query_start, seq_len, prompt_len, scale, TPSA_KV_HEADS, scratch,
                kStaticScratchBytes, nullptr, nullptr, stream);
}

#ifdef TPSA_TRACE
// Copies role `role`'s events of the last launch into out (2 x uint64 each).
TPSA_API void tpsa_debug_spans(unsigned long long* out, uint32_t ctas) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(out, g_cta_span, sizeof(unsigned long long) * 3 * (ctas < 1024 ? ctas : 1024));
}

TPSA_API void tpsa_debug_timeout(uint32_t* out5) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(out5, g_timeout_site, sizeof(uint32_t) * 5);
}

TPSA_API uint32_t tpsa_debug_trace(uint32_t role, unsigned long long* out, uint32_t max_events) {
  uint32_t n[kTraceRoles] = {};
  cudaDeviceSynchronize();
  if (role >= kTraceRoles) {  // softmax sub-phase buffers of CTA role - 4
    return 0;
  }
  cudaMemcpyFromSymbol(n, g_trace_n, sizeof(n));
  uint32_t c = n[role] < max_events ? n[role] : max_events;
  cudaMemcpyFromSymbol(out, g_trace, sizeof(unsigned long long) * 2 * c,
                       sizeof(unsigned long long) * 2 * kTraceCap * role);
  return c;
}
#endif

tpsa_status tpsa_device_status(int32_t device, uint32_t* status_bits) {
  t_last_error.clear();
  if (status_bits == nullptr) return fail(TPSA_ERR_INVALID_ARGUMENT, "status pointer is NULL");
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  uint32_t bits = 0;
  e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&bits, g_device_status, sizeof(bits));
  const uint32_t zero = 0;
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device status word");
  *status_bits = bits;
  return bits == 0 ? TPSA_OK : TPSA_ERR_DEVICE_FAULT;
}

}  // extern "C"
