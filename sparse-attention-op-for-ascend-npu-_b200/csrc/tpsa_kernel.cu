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
//   warp 0      TMA producer; in CTA 0 also the work scheduler (a global
//               counter, longest items first), which hands items to CTA 1
//               through its shared memory
//   warp 1      CTA 0: tcgen05 MMA issuer; both: TMEM owner
//   warps 2-3   idle (they complete the control warpgroup for setmaxnreg)
//   warps 4-11  two softmax warpgroups.  Key tile gt of the pair's global
//               tile sequence belongs to warpgroup gt % 2, which keeps its
//               own S buffer, O accumulator and row (max, sum) over whole
//               128-column rows; the two partial results of an item are
//               merged once at its end.  While one warpgroup exponentiates,
//               the tensor pipe runs the other's QK and PV.
// Tensor memory per CTA (fp32 columns): S0 [0,128), S1 [128,256),
// O0 [256,384), O1 [384,512).  P (bf16 pairs) overwrites the first half of
// its S buffer and PV(n) reads it from there.  MMA issue order per item:
//   QK(0), QK(1), PV(0), QK(2), PV(1), QK(3), ...
// so QK(n+1) (the other warpgroup's S) runs while tile n's softmax is
// computed.  The O rescale for a grown row max is lazy (only when the max
// grows by more than 2^8) and done by the softmax warps in tensor memory.
//
// Softmax arithmetic: scores are scaled into the log2 domain with one fused
// multiply-add, exponentiated with ex2.approx (MUFU) for 3 of every 4 column
// pairs and with poly_exp2_x2 (FMA pipe) for the fourth, summed in fp32, and
// rounded to bf16 (round-to-nearest-even) for the PV product, as the
// reference does (vendor block_epilogue_online_softmax.hpp:886-906).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "sm100_ptx.cuh"
#include "tpsa_schedule.h"

namespace tpsa {

__device__ uint32_t g_device_status = 0;

// Optional event trace of cluster 0 (build with -DTPSA_TRACE; compiled out of
// the library otherwise).  Each tracing thread owns one buffer and a register
// counter, so a trace point is two plain stores and a clock read.
#ifdef TPSA_TRACE
constexpr uint32_t kTraceRoles = 4;
constexpr uint32_t kTraceCap = 1u << 14;
__device__ unsigned long long g_trace[kTraceRoles][kTraceCap][2];
__device__ uint32_t g_trace_n[kTraceRoles];
#define TPSA_TRACE_STATE uint32_t tr_n_ = 0
#define TPSA_SM_TR(ev)                                                             \
  do {                                                                             \
    if (blockIdx.x == 0 && (threadIdx.x == 128 || threadIdx.x == 256) && trn < kTraceCap) {              \
      g_trace[trole][trn][0] = static_cast<unsigned long long>(ev) << 32;          \
      g_trace[trole][trn][1] = clock64();                                          \
      ++trn;                                                                       \
      g_trace_n[trole] = trn;                                                      \
    }                                                                              \
  } while (0)
#define TPSA_TR(role, ev, arg)                                                    \
  do {                                                                            \
    if (blockIdx.x < 2 && tr_n_ < kTraceCap) {                                    \
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
#define TPSA_SM_TR(ev) \
  do {                 \
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
constexpr uint32_t kTmemCols = 512;
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;  // 1 s per wait
constexpr uint64_t kAbortSettleNs = 200000ull;      // let in-flight TMA land
constexpr float kRescaleLog2 = 8.0f;
// Column pairs c (of 16 per 32-column chunk) whose exponentials use the FMA
// pipe polynomial rather than MUFU ex2: bit c set.
#ifndef TPSA_POLY_MASK
#define TPSA_POLY_MASK 0x8888u
#endif  // lazy O rescale threshold (log2 units)
constexpr uint16_t kPairMask = 0x3;

// Shared memory per CTA (offsets from a 1024-byte aligned base).
constexpr uint32_t kQHalfBytes = 128 * 128;        // 128 rows x 64 bf16
constexpr uint32_t kQBytes = 2 * kQHalfBytes;      // one Q buffer (2 d-halves)
constexpr uint32_t kRingSlotBytes = 32768;         // one key tile: K half + V half
constexpr uint32_t kKHalfBytes = 8192;             // d-half of a K half-tile
constexpr uint32_t kVOffset = 16384;               // V half within a slot
constexpr int kRing = 4;                           // key-tile slots (power of two)
constexpr uint32_t kOffQ = 0;                      // 2 Q buffers
constexpr uint32_t kOffKV = kOffQ + 2 * kQBytes;
constexpr uint32_t kOffBar = kOffKV + kRing * kRingSlotBytes;

enum BarId : uint32_t {
  kBarQFull = 0,                          // [2] CTA 0: both Q halves landed
  kBarQEmpty = kBarQFull + 2,             // [2] both CTAs: Q buffer free
  kBarKVFull = kBarQEmpty + 2,            // [kRing] CTA 0: K and V of both CTAs landed
  kBarKVEmpty = kBarKVFull + kRing,       // [kRing] both: slot free (its PV done)
  kBarSFull = kBarKVEmpty + kRing,        // [2] both: S buffer computed
  kBarPFull = kBarSFull + 2,              // [2] CTA 0: P of a warpgroup's tile in TMEM
  kBarPvDone = kBarPFull + 2,             // [2] both: PV of a warpgroup's tile completed
  kBarOEmpty = kBarPvDone + 2,            // CTA 0: O0 and O1 read by both epilogues
  kBarItemFull = kBarOEmpty + 1,          // [2] both: item index written
  kBarItemEmpty = kBarItemFull + 2,       // [2] CTA 0: item index consumed
  kBarSplitWritten = kBarItemEmpty + 2,   // per CTA: split partial written
  kBarSplitDecided = kBarSplitWritten + 1,
  kBarTail = kBarSplitDecided + 1,        // per CTA: V tail tile landed
  kBarDrain = kBarTail + 1,               // CTA 0: all MMAs complete
  kBarWgX = kBarDrain + 1,                // per CTA: softmax warpgroups exchanged
  kNumBars
};
// Arrivals: p_full and o_empty take one per softmax warp of both CTAs;
// item_empty takes the MMA issuer and 4 softmax warps of CTA 0 plus the
// producer and 4 softmax warps of CTA 1.
constexpr uint32_t kPairWarpArrivals = 2 * kSoftmaxWarps;
constexpr uint32_t kPairWgArrivals = kSoftmaxWarps;  // 4 warps of one warpgroup x 2 CTAs
constexpr uint32_t kItemConsumers = 2 * (1 + kSoftmaxWarps);

constexpr uint32_t kOffItemSlots = (kOffBar + kNumBars * 8 + 15) & ~15u;  // 2 x ItemRec
constexpr uint32_t kOffTmemSlot = kOffItemSlots + 2 * 64;
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
constexpr uint32_t kOffSplitLast = kOffAbort + 4;
// (row max, row sum) exchange between the two softmax warpgroups at the
// end of an item: float [2 buffers][2 warpgroups][2 values][128 rows].
constexpr uint32_t kOffXchg = (kOffSplitLast + 4 + 15) & ~15u;
// Output staging: 2 KB per softmax warp (32 rows x 64 bytes), used to turn
// row-per-thread results into coalesced global stores.
constexpr uint32_t kStageBytesPerWarp = 32 * 64;
constexpr uint32_t kOffStage = (kOffXchg + 2 * 2 * 2 * 128 * 4 + 127) & ~127u;
constexpr uint32_t kSmemUsed = kOffStage + 8 * kStageBytesPerWarp;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // alignment slack
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

// Workspace control words (first kControlBytes of the workspace, zeroed by
// the launcher): [0] next work item, [64..] one split counter per
// (tail block, kv head, pair rank).
constexpr int kCtlNextItem = 0;
constexpr int kCtlSplitBase = 64;

struct KernelArgs {
  tpsa_plan plan;
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
  __device__ uint4* item_slot(uint32_t i) const {
    return reinterpret_cast<uint4*>(base + kOffItemSlots + 64 * i);
  }
  __device__ uint32_t item_slot_addr(uint32_t i) const { return base_u32 + kOffItemSlots + 64 * i; }
};

__device__ __forceinline__ void raise_status(uint32_t bits) {
  atomicOr(&g_device_status, bits);
}

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
  // or key range that starts or ends half-way through a page).
  uint32_t narrow;
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

__device__ __forceinline__ void release_item(const Shared& sh, uint32_t n) {
  ptx::mbar_arrive_cluster(sh.bar0(kBarItemEmpty + n % 2));
}

// ------------------------------------------------------------ producer
__device__ void producer_role(const KernelArgs& a, const Shared& sh,
                              const CUtensorMap* tq, const CUtensorMap* tk64,
                              const CUtensorMap* tk32, const CUtensorMap* tv) {
  const tpsa_plan& p = a.plan;
  const uint32_t r = sh.rank;
  ptx::prefetch_tmap(tq);
  ptx::prefetch_tmap(tk64);
  ptx::prefetch_tmap(tk32);
  ptx::prefetch_tmap(tv);
  uint32_t ring = 0, q_iter = 0, tail_iter = 0;
  bool ok = true;
  TPSA_TRACE_STATE;
  int32_t next = r == 0 ? atomicAdd(a.ctl + kCtlNextItem, 1) : 0;
  for (uint32_t n = 0; ok; ++n) {
    ItemRec rec;
    const uint32_t slot = n % 2;
    if (r == 0) {
      rec = make_item_rec(p, next);
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
      next = atomicAdd(a.ctl + kCtlNextItem, 1);  // latency hidden by the loads below
    } else {
      if (!take_item(sh, n, &rec)) break;
      release_item(sh, n);
      if (rec.idx >= p.total_items) break;
    }
    if (r == 0) TPSA_TR(0, 20, rec.idx);
    const tpsa_item& it = rec.it;
    const BlockTiles& bt = rec.bt;

    // Q: this CTA's 128 rows (64 tokens x query heads 4h + 2r, 4h + 2r + 1).
    const uint32_t qb = q_iter % 2;
    if (q_iter >= 2 && !wait_bar(sh, sh.bar(kBarQEmpty + qb), ((q_iter / 2) - 1) & 1)) break;
    ptx::mbar_arrive_expect_tx_cluster(sh.bar0(kBarQFull + qb), kQBytes);
    for (int dh = 0; dh < 2; ++dh) {
      ptx::tma_load_3d_pair(sh.base_u32 + kOffQ + qb * kQBytes + dh * kQHalfBytes, tq, dh * 64,
                            it.kv_head * kGroupSize + 2 * r, it.block * kBlockQ,
                            sh.bar0(kBarQFull + qb));
    }
    ++q_iter;
    if (r == 0) TPSA_TR(0, 21, rec.idx);

    for (int32_t t = it.tile_begin; t < it.tile_end && ok; ++t) {
      int32_t k0, w;
      tile_keys(bt, t, &k0, &w);
      const int32_t page = __ldg(a.block_table + k0 / kPageSize);
      int32_t tok;
      if (page < 0 || page >= a.num_pages) {
        raise_status(TPSA_DEVICE_BAD_PAGE);
        tok = -kPageSize;  // fully out of bounds: TMA fills zeros
      } else {
        tok = page * kPageSize + (k0 % kPageSize);
      }
      if (a.tiles != nullptr && r == 0) {
        atomicAdd(a.tiles, 1ull);
        atomicAdd(a.tiles + 1, static_cast<unsigned long long>(w));
      }
      const int32_t half = w / 2;
      // One slot per key tile: K keys [k0 + r*half, +half) (all 128 d, two
      // d-halves) at +0 and V keys [k0, k0 + w) (d-half r) at +kVOffset,
      // both completing on the slot's full barrier.
      const uint32_t s = ring_slot(ring);
      if (!wait_bar(sh, sh.bar(kBarKVEmpty + s), ring_parity(ring) ^ 1)) { ok = false; break; }
      ++ring;
      const uint32_t kdst = sh.base_u32 + kOffKV + s * kRingSlotBytes;
      const uint32_t vdst = kdst + kVOffset;
      const uint32_t kbytes = static_cast<uint32_t>(half) * kHeadDim * 2;
      const uint32_t vbytes = static_cast<uint32_t>(w) * 64 * 2;
      const CUtensorMap* km = w == kTileKeys ? tk64 : tk32;
      if (k0 + w <= p.seq_len) {
        ptx::mbar_arrive_expect_tx_cluster(sh.bar0(kBarKVFull + s), kbytes + vbytes);
        for (int dh = 0; dh < 2; ++dh) {
          ptx::tma_load_3d_pair(kdst + dh * kKHalfBytes, km, dh * 64, it.kv_head,
                                tok + static_cast<int32_t>(r) * half, sh.bar0(kBarKVFull + s));
        }
        for (int sub = 0; sub < w / 64; ++sub) {
          ptx::tma_load_3d_pair(vdst + sub * 8192, tv, static_cast<int32_t>(r) * 64, it.kv_head,
                                tok + sub * 64, sh.bar0(kBarKVFull + s));
        }
      } else {
        // Keys at or beyond seq_len may be unwritten cache slots: load the
        // tile into this CTA's slot here, zero those V rows so P = 0 never
        // meets a NaN, then release the slot with a plain arrival.
        ptx::mbar_arrive_expect_tx(sh.bar(kBarTail), kbytes + vbytes);
        for (int dh = 0; dh < 2; ++dh) {
          ptx::tma_load_3d(kdst + dh * kKHalfBytes, km, dh * 64, it.kv_head,
                           tok + static_cast<int32_t>(r) * half, sh.bar(kBarTail));
        }
        for (int sub = 0; sub < w / 64; ++sub) {
          ptx::tma_load_3d(vdst + sub * 8192, tv, static_cast<int32_t>(r) * 64, it.kv_head,
                           tok + sub * 64, sh.bar(kBarTail));
        }
        if (!wait_bar(sh, sh.bar(kBarTail), tail_iter & 1)) { ok = false; break; }
        ++tail_iter;
        for (int32_t row = p.seq_len - k0; row < w; ++row) {
          uint4* dst = reinterpret_cast<uint4*>(sh.base + (vdst - sh.base_u32) + row * 128);
#pragma unroll
          for (int j = 0; j < 8; ++j) dst[j] = make_uint4(0, 0, 0, 0);
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive_cluster(sh.bar0(kBarKVFull + s));
      }
      if (r == 0) TPSA_TR(0, 22, t);
    }
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
  // tcgen05.mma issue blocks once about three MMAs are queued, so this warp's
  // own instructions between MMA batches leave the tensor pipe idle.  The
  // loop below therefore keeps its per-tile work to barrier waits, commits
  // and additions to operands prepared once: descriptor bases, barrier
  // addresses, instruction descriptors and incremental ring positions.
  const uint32_t bar_kv_full = sh.bar(kBarKVFull), bar_kv_empty = sh.bar(kBarKVEmpty);
  const uint32_t bar_s_full = sh.bar(kBarSFull), bar_p_full = sh.bar(kBarPFull);
  const uint32_t bar_pv_done = sh.bar(kBarPvDone), bar_q_full = sh.bar(kBarQFull);
  const uint32_t bar_q_empty = sh.bar(kBarQEmpty), bar_o_empty = sh.bar(kBarOEmpty);
  // Descriptor start addresses are in 16-byte units.
  const uint64_t q_desc0 = ptx::smem_desc_sw128(sh.base_u32 + kOffQ, 16, 1024);
  const uint64_t k_desc0 = ptx::smem_desc_sw128(sh.base_u32 + kOffKV, 16, 1024);
  const uint64_t v_desc0 =
      ptx::smem_desc_sw128(sh.base_u32 + kOffKV + kVOffset, kKHalfBytes, 1024);
  constexpr uint32_t kSlotUnits = kRingSlotBytes >> 4;
  constexpr uint32_t kQUnits = kQBytes >> 4;
  constexpr uint32_t kIdQk128 = ptx::idesc_bf16_f32(256, 128, 0);
  constexpr uint32_t kIdQk64 = ptx::idesc_bf16_f32(256, 64, 0);
  constexpr uint32_t kIdPv = ptx::idesc_bf16_f32(256, 128, 1);

  auto warp_wait = [&](uint32_t bar, uint32_t parity) -> bool {
    return __all_sync(0xffffffffu, wait_bar(sh, bar, parity));
  };
  // S(buf) = Q K^T for the key tile in ring slot `slot` (M = 256 over the
  // pair, N = 128 or 64).
  auto issue_qk = [&](uint64_t qd, uint32_t slot, uint32_t buf, bool narrow) {
    const uint32_t d = tmem + (buf << 7);
    const uint32_t idesc = narrow ? kIdQk64 : kIdQk128;
    const uint64_t kd = k_desc0 + slot * kSlotUnits;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint64_t qo = (k / 4) * (kQHalfBytes >> 4) + (k % 4) * 2;
      const uint64_t ko = (k / 4) * (kKHalfBytes >> 4) + (k % 4) * 2;
      ptx::umma_ss_pair_elect(d, qd + qo, kd + ko, idesc, k > 0 ? 1u : 0u);
    }
  };
  // O(buf) += P(buf) V: P (bf16 pairs) over the first half of S buffer buf,
  // V the d-half of this CTA in ring slot `slot`.  Tile gt belongs to
  // softmax warpgroup buf = gt % 2, which owns S and O buffer buf.
  auto issue_pv = [&](uint32_t slot, uint32_t buf, bool narrow, bool first) {
    const uint32_t d = tmem + 256 + (buf << 7);
    const uint32_t pa = tmem + (buf << 7);
    const uint64_t vd = v_desc0 + slot * kSlotUnits;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k < 4 || !narrow) {
        ptx::umma_ts_pair_elect(d, pa + k * 8, vd + k * (2048 >> 4), kIdPv,
                                (first && k == 0) ? 0u : 1u);
      }
    }
  };

  // Ring cursors: the slot and phase of the next tile whose K/V is awaited
  // (QK), and the slot of the next tile whose PV is issued (two tiles
  // behind within an item).
  uint32_t slot_q = 0, phase_q = 0, slot_v = 0, q_iter = 0, gt = 0, item_iter = 0;
  bool ok = true;
  auto next_q = [&]() {
    slot_q = (slot_q + 1) & (kRing - 1);
    phase_q ^= slot_q == 0 ? 1u : 0u;
  };
  auto wait_kv = [&]() -> bool {
    return warp_wait(bar_kv_full + 8 * slot_q, phase_q);
  };

  for (uint32_t n_item = 0; ok; ++n_item) {
    ItemRec rec;
    const bool got = take_item(sh, n_item, &rec);
    if (!__all_sync(0xffffffffu, got)) break;
    __syncwarp();
    if (lane == 0) release_item(sh, n_item);
    if (rec.idx >= p.total_items) break;
    if (lane == 0) TPSA_TR(1, 10, rec.idx);
    const int32_t ntiles = rec.it.tile_end - rec.it.tile_begin;
    const int32_t last = ntiles - 1;
    const uint32_t narrow = rec.narrow;
    auto is_narrow = [&](int32_t t) -> bool {
      return (t < 2 && ((narrow >> t) & 1u)) || (t == last && (narrow & 4u));
    };
    const uint32_t qb = q_iter & 1;
    if (!warp_wait(bar_q_full + 8 * qb, (q_iter >> 1) & 1)) break;
    ++q_iter;
    ptx::tc_fence_after();
    const uint64_t qd = q_desc0 + qb * kQUnits;

    // QK for the first two tiles.
    for (int32_t t = 0; t < 2 && t < ntiles; ++t) {
      if (!wait_kv()) { ok = false; break; }
      ptx::tc_fence_after();
      issue_qk(qd, slot_q, (gt + t) & 1, is_narrow(t));
      ptx::umma_commit_pair_mc_elect(bar_s_full + 8 * ((gt + t) & 1), kPairMask);
      if (t == last) ptx::umma_commit_pair_mc_elect(bar_q_empty + 8 * qb, kPairMask);
      next_q();
    }
    for (int32_t n = 0; n < ntiles && ok; ++n, ++gt) {
      const uint32_t buf = gt & 1;
      if (lane == 0) TPSA_TR(1, 13, n);
      if (n == 0 && item_iter > 0 && !warp_wait(bar_o_empty, (item_iter - 1) & 1)) {
        ok = false;
        break;
      }
      if (!warp_wait(bar_p_full + 8 * buf, (gt >> 1) & 1)) { ok = false; break; }
      if (lane == 0) TPSA_TR(1, 14, n);
      ptx::tc_fence_after();
      // Each warpgroup's first tile of the item overwrites its O buffer.
      issue_pv(slot_v, buf, is_narrow(n), n < 2);
      if (lane == 0) TPSA_TR(1, 15, n);
      ptx::umma_commit_pair_mc_elect(bar_kv_empty + 8 * slot_v, kPairMask);
      slot_v = (slot_v + 1) & (kRing - 1);
      // A warpgroup learns that its earlier PVs completed from the S of its
      // next tile (whose QK is issued after them); only its last tile of the
      // item needs an explicit completion signal.
      if (n + 2 > last) ptx::umma_commit_pair_mc_elect(bar_pv_done + 8 * buf, kPairMask);
      if (lane == 0) TPSA_TR(1, 16, n);
      if (n + 2 <= last) {
        if (!wait_kv()) { ok = false; break; }
        if (lane == 0) TPSA_TR(1, 17, n + 2);
        ptx::tc_fence_after();
        issue_qk(qd, slot_q, buf, is_narrow(n + 2));
        if (lane == 0) TPSA_TR(1, 18, n + 2);
        ptx::umma_commit_pair_mc_elect(bar_s_full + 8 * buf, kPairMask);
        if (n + 2 == last) ptx::umma_commit_pair_mc_elect(bar_q_empty + 8 * qb, kPairMask);
        next_q();
      }
    }
    ++item_iter;
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
  ptx::tmem_wait_st();
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

// Online-softmax state of one row over one warpgroup's tiles of an item.
struct RowState {
  float m_run;
  float l_run;
};

// Publishes this warpgroup's (m, l) of the row and returns the other
// warpgroup's.  `xc` counts exchanges; both warpgroups run the same sequence.
__device__ __forceinline__ bool exchange_ml(const Shared& sh, uint32_t& xc, int wg, int row,
                                            int lane, float m, float l, float* m_other,
                                            float* l_other) {
  volatile float* buf = reinterpret_cast<volatile float*>(sh.base + kOffXchg) + (xc & 1) * 512;
  buf[wg * 256 + row] = m;
  buf[wg * 256 + 128 + row] = l;
  __syncwarp();
  if (lane == 0) ptx::mbar_arrive(sh.bar(kBarWgX));
  const bool ok = wait_bar(sh, sh.bar(kBarWgX), xc & 1);
  ++xc;
  if (!__all_sync(0xffffffffu, ok)) return false;
  *m_other = buf[(1 - wg) * 256 + row];
  *l_other = buf[(1 - wg) * 256 + 128 + row];
  return true;
}

struct SoftmaxCtx {
  const tpsa_plan* p;
  uint32_t s_addr;  // this warpgroup's S buffer (P overwrites its first half)
  uint32_t o_addr;  // this warpgroup's O buffer
  int32_t q;
  bool sparse;
};

// Converts one 32-column chunk of S to floats, masking the keys outside the
// row's key set when kMasked.
template <bool kMasked>
__device__ __forceinline__ void chunk_values(const uint32_t (&r)[32], uint32_t m, float (&v)[32]) {
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    const float x = __uint_as_float(r[c]);
    v[c] = (!kMasked || ((m >> c) & 1u)) ? x : -INFINITY;
  }
}

// One key tile of w keys (64 or 128) starting at k0, the whole row: mask,
// row max, online-softmax update, P -> tensor memory.  `first`: the
// warpgroup's first tile of the item, whose PV overwrites O (so O is not
// rescaled).  Two passes over the S columns in tensor memory, 64 columns at
// a time, keep at most 64 of them in registers: pass 1 takes the row max
// (and the visited bits), pass 2 reloads, exponentiates and writes P (bf16
// pairs) over the first half of the S buffer, which it has already read.
// The loops over 64-column halves are not unrolled: one body serves both
// tile widths, which keeps the kernel's code small.
template <bool kMasked>
__device__ __forceinline__ void softmax_tile(const SoftmaxCtx& cx, int32_t k0, int32_t w,
                                             bool first, RowState& st, uint32_t* visit_row,
                                             int32_t words_per_row, uint32_t trole,
                                             uint32_t& trn) {
  const tpsa_plan& p = *cx.p;
  const int32_t halves = w / 64;
  float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll 1
  for (int32_t h = 0; h < halves; ++h) {
    uint32_t ra[32], rb[32];
    ptx::tmem_ld32(cx.s_addr + 64 * h, ra);
    ptx::tmem_ld32(cx.s_addr + 64 * h + 32, rb);
    ptx::tmem_wait_ld_regs(ra);
    ptx::tmem_fence_regs(rb);
    const int32_t kc = k0 + 64 * h;
    const uint32_t ma = kMasked ? chunk_mask(cx.q, cx.sparse, kc) : ~0u;
    const uint32_t mb = kMasked ? chunk_mask(cx.q, cx.sparse, kc + 32) : ~0u;
    if (visit_row != nullptr) {
      const int32_t word = kc / 32;
      if (ma != 0 && word < words_per_row) atomicOr(visit_row + word, ma);
      if (mb != 0 && word + 1 < words_per_row) atomicOr(visit_row + word + 1, mb);
    }
    float v[32];
    chunk_values<kMasked>(ra, ma, v);
#pragma unroll
    for (int c = 0; c < 32; c += 8) {
      mx0 = max3(mx0, v[c], v[c + 1]);
      mx1 = max3(mx1, v[c + 2], v[c + 3]);
      mx2 = max3(mx2, v[c + 4], v[c + 5]);
      mx3 = max3(mx3, v[c + 6], v[c + 7]);
    }
    chunk_values<kMasked>(rb, mb, v);
#pragma unroll
    for (int c = 0; c < 32; c += 8) {
      mx0 = max3(mx0, v[c], v[c + 1]);
      mx1 = max3(mx1, v[c + 2], v[c + 3]);
      mx2 = max3(mx2, v[c + 4], v[c + 5]);
      mx3 = max3(mx3, v[c + 6], v[c + 7]);
    }
  }
  TPSA_SM_TR(2);
  const float mx = fmaxf(max3(mx0, mx1, mx2), mx3);
  const float m_new = fmaxf(st.m_run, mx);
  const bool need = (m_new - st.m_run) * p.scale_log2 > kRescaleLog2;
  const bool any_need = __any_sync(0xffffffffu, need);
  float factor = 1.0f;
  if (any_need) {
    factor = need ? mufu_exp2((st.m_run - m_new) * p.scale_log2) : 1.0f;
    st.l_run *= factor;
    if (need) st.m_run = m_new;
  }
  const float neg_mb = st.m_run == -INFINITY ? 0.0f : -st.m_run * p.scale_log2;
  TPSA_SM_TR(6);
  float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll 1
  for (int32_t h = 0; h < halves; ++h) {
    uint32_t ra[32], rb[32];
    ptx::tmem_ld32(cx.s_addr + 64 * h, ra);
    ptx::tmem_ld32(cx.s_addr + 64 * h + 32, rb);
    ptx::tmem_wait_ld_regs(ra);
    ptx::tmem_fence_regs(rb);
    const int32_t kc = k0 + 64 * h;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float v[32];
      if (half == 0) {
        chunk_values<kMasked>(ra, kMasked ? chunk_mask(cx.q, cx.sparse, kc) : ~0u, v);
      } else {
        chunk_values<kMasked>(rb, kMasked ? chunk_mask(cx.q, cx.sparse, kc + 32) : ~0u, v);
      }
      uint32_t pk[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float x0, x1;
        fma2(v[2 * c], v[2 * c + 1], p.scale_log2, neg_mb, x0, x1);
        float e0, e1;
        if ((TPSA_POLY_MASK >> c) & 1u) {
          poly_exp2_x2(x0, x1, e0, e1);
        } else {
          e0 = mufu_exp2(x0);
          e1 = mufu_exp2(x1);
        }
        add2(sum0, sum1, e0, e1);
        pk[c] = pack_bf16x2(e0, e1);
      }
      ptx::tmem_st16(cx.s_addr + 32 * h + 16 * half, pk);
    }
  }
  st.l_run += sum0 + sum1;
  // O is rescaled after the exponentials; it only has to be done before P is
  // published (the PV of this tile accumulates into O).  The PVs of earlier
  // tiles into O have completed (the caller waited).
  if (any_need && !first) rescale_o(cx.o_addr, factor);
  ptx::tmem_wait_st();
  TPSA_SM_TR(7);
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
// the tensor-memory lane quadrant, so each warpgroup covers all 128 rows).  Tile
// gt of the pair's global tile sequence belongs to warpgroup gt % 2, which
// keeps its own S buffer, O accumulator and (m, l) per row; the two partial
// results of an item are merged once at its end, each warpgroup producing 64
// of the 128 output columns.
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
  const bool visit = a.visited != nullptr;
  // own: tiles of this warpgroup so far (tile gt = 2 * own + wg);
  // pv_items0/1: items in which warpgroup 0/1 had tiles (one PV-done phase
  // each on that warpgroup's barrier).
  uint32_t g = 0, own = 0, pv_items0 = 0, pv_items1 = 0, split_iter = 0, xc = 0;
  volatile int* split_last = reinterpret_cast<volatile int*>(sh.base + kOffSplitLast);
  uint32_t tr_sm = 0;  // trace counter (used only with TPSA_TRACE)
#define tr_n_ tr_sm
  const uint32_t o_base = tmem + lane_base + 256;  // O0; O1 at +128
  SoftmaxCtx cx;
  cx.p = &p;
  cx.s_addr = tmem + lane_base + wg * 128;
  cx.o_addr = o_base + wg * 128;

  for (uint32_t n_item = 0;; ++n_item) {
    ItemRec rec;
    const bool got = take_item(sh, n_item, &rec);
    if (!__all_sync(0xffffffffu, got)) break;
    __syncwarp();
    if (lane == 0) release_item(sh, n_item);
    if (rec.idx >= p.total_items) break;
    const int32_t idx = rec.idx;
    const tpsa_item& it = rec.it;
    const BlockTiles& bt = rec.bt;
    const int32_t tok = bt.q_begin + row / 2;
    cx.q = tok < p.seq_len ? tok : p.seq_len - 1;
    cx.sparse = row_is_sparse(p, tok);
    const int32_t qrow = it.block * kBlockQ + row / 2;  // row within the chunk
    const int32_t head = it.kv_head * kGroupSize + 2 * static_cast<int32_t>(r) + (row & 1);
    const bool real_row = qrow < p.query_tokens;
    uint32_t* visit_row =
        (visit && real_row)
            ? a.visited + (static_cast<size_t>(qrow) * hq + head) * a.words_per_row
            : nullptr;
    RowState st{-INFINITY, 0.0f};
    bool ok = true, first = true;
    const int32_t ntiles = it.tile_end - it.tile_begin;
    // Which warpgroups own at least one tile of this item.
    const bool has_wg0 = ntiles >= 2 || (g & 1) == 0;
    const bool has_wg1 = ntiles >= 2 || (g & 1) == 1;
    for (int32_t n = (g + wg) & 1; n < ntiles; n += 2) {
      int32_t k0, w;
      tile_keys(bt, it.tile_begin + n, &k0, &w);
      const bool masked = tile_needs_mask(p, bt, k0, w);
      const bool w_ok = wait_bar(sh, sh.bar(kBarSFull + wg), own & 1);
      if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
      // S of this tile being full also means this warpgroup's earlier PVs
      // into O completed (their MMAs were issued before this tile's QK).
      if (row == 0 && r == 0) TPSA_TR(2 + wg, 1, n);
      ptx::tc_fence_after();
      if (masked) {
        softmax_tile<true>(cx, k0, w, first, st, visit_row, a.words_per_row, 2 + wg, tr_sm);
      } else {
        softmax_tile<false>(cx, k0, w, first, st, visit_row, a.words_per_row, 2 + wg, tr_sm);
      }
      ptx::tc_fence_before();
      if (row == 0 && r == 0) TPSA_TR(2 + wg, 3, n);
      warp_arrive0(sh, kBarPFull + wg, lane);
      first = false;
      ++own;
    }
    if (!ok) break;
    g += static_cast<uint32_t>(ntiles);
    // O0 and O1 are final once each warpgroup's last PV of the item
    // completed (signalled once per item in which that warpgroup had tiles;
    // both warpgroups observe both signals).
    if (has_wg0) {
      const bool pv_ok = wait_bar(sh, sh.bar(kBarPvDone + 0), pv_items0 & 1);
      if (!__all_sync(0xffffffffu, pv_ok)) break;
      ++pv_items0;
    }
    if (has_wg1) {
      const bool pv_ok = wait_bar(sh, sh.bar(kBarPvDone + 1), pv_items1 & 1);
      if (!__all_sync(0xffffffffu, pv_ok)) break;
      ++pv_items1;
    }
    if (row == 0 && r == 0) TPSA_TR(2 + wg, 8, 0);
    float m_o, l_o;
    if (!exchange_ml(sh, xc, wg, row, lane, st.m_run, st.l_run, &m_o, &l_o)) break;
    ptx::tc_fence_after();
    if (row == 0 && r == 0) TPSA_TR(2 + wg, 9, 0);
    const float m0 = wg == 0 ? st.m_run : m_o, m1 = wg == 0 ? m_o : st.m_run;
    const float l0 = wg == 0 ? st.l_run : l_o, l1 = wg == 0 ? l_o : st.l_run;
    const float m_all = fmaxf(m0, m1);
    const float a0 = m0 == -INFINITY ? 0.0f : mufu_exp2((m0 - m_all) * p.scale_log2);
    const float a1 = m1 == -INFINITY ? 0.0f : mufu_exp2((m1 - m_all) * p.scale_log2);
    const float l_total = l0 * a0 + l1 * a1;
    // Columns [64 wg, 64 wg + 64) of the merged output row, 32 at a time:
    // bf16 into `out`, or for a split item the unnormalised fp32 partial
    // (O, m, l) into the item's workspace slot.  A slot is column-major
    // ([128 columns][256 rows], then m[256] and l[256]), so a warp's row-per-
    // thread writes and reads of one column are 128 contiguous bytes.
    const bool split = it.num_splits > 1;
    float* slot = a.scratch + static_cast<size_t>(idx) * kSlotFloats;
    constexpr int32_t kSlotRows = 2 * kRowsPerTile;
    const int32_t srow = static_cast<int32_t>(r) * kRowsPerTile + row;
    const int32_t base_q = it.block * kBlockQ + quad * 16;
    const int32_t base_h = it.kv_head * kGroupSize + 2 * static_cast<int32_t>(r);
    uint8_t* stage = sh.base + kOffStage + (warp - kFirstSoftmaxWarp) * kStageBytesPerWarp;
    const float inv = 1.0f / l_total;
    // Both 32-column chunks are merged into registers first and the O
    // buffers released, so the next item's PVs need not wait for the
    // stores.
    float om[2][32];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint32_t col = static_cast<uint32_t>(wg * 64 + 32 * c);
      uint32_t x0[32], x1[32];
      if (has_wg0) ptx::tmem_ld32(o_base + col, x0);
      if (has_wg1) ptx::tmem_ld32(o_base + 128 + col, x1);
      ptx::tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float v0 = has_wg0 ? a0 * __uint_as_float(x0[j]) : 0.0f;
        om[c][j] = has_wg1 ? fmaf(a1, __uint_as_float(x1[j]), v0) : v0;
      }
    }
    ptx::tc_fence_before();
    warp_arrive0(sh, kBarOEmpty, lane);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint32_t col = static_cast<uint32_t>(wg * 64 + 32 * c);
      const float (&o)[32] = om[c];
      if (!split) {
        store_rows_bf16(o, inv, stage, lane, a.out, base_q, base_h, hq, p.query_tokens,
                        static_cast<int32_t>(col));
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) slot[(col + j) * kSlotRows + srow] = o[j];
      }
    }
    if (row == 0 && r == 0) TPSA_TR(2 + wg, 5, 0);
    if (!split) continue;

    // Split item: the last split of the block (per CTA of the pair) merges
    // all partials and writes bf16.
    if (wg == 0) {
      slot[kHeadDim * kSlotRows + srow] = m_all;
      slot[(kHeadDim + 1) * kSlotRows + srow] = l_total;
    }
    __threadfence();
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(sh.bar(kBarSplitWritten));
    bool w_ok = wait_bar(sh, sh.bar(kBarSplitWritten), split_iter & 1);
    if (!__all_sync(0xffffffffu, w_ok)) break;
    if (row == 0 && wg == 0) {
      int32_t* ctr = a.ctl + kCtlSplitBase +
                     ((it.block - p.tail_block0) * p.kv_heads + it.kv_head) * 2 + r;
      const int prev = atomicAdd(ctr, 1);
      *split_last = prev == it.num_splits - 1;
      ptx::mbar_arrive(sh.bar(kBarSplitDecided));
    }
    w_ok = wait_bar(sh, sh.bar(kBarSplitDecided), split_iter & 1);
    ++split_iter;
    if (!__all_sync(0xffffffffu, w_ok)) break;
    if (!*split_last) continue;
    __threadfence();
    const float* first_slot = a.scratch + static_cast<size_t>(idx - it.split) * kSlotFloats;
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
    for (int c = 0; c < 2; ++c) {
      const int col = wg * 64 + 32 * c;
      float acc[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
      for (int32_t sp = 0; sp < it.num_splits; ++sp) {
        const float* sl = first_slot + sp * kSlotFloats;
        const float ms = __ldcg(sl + m_off);
        const float wgt = ms == -INFINITY ? 0.0f : mufu_exp2((ms - mmax) * p.scale_log2);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          acc[j] += wgt * __ldcg(sl + static_cast<size_t>(col + j) * kSlotRows + srow);
        }
      }
      store_rows_bf16(acc, inv_sum, stage, lane, a.out, base_q, base_h, hq, p.query_tokens, col);
    }
  }
}
#undef tr_n_

template <bool kVisit>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kNumThreads, 1)
    tpsa_paged_kernel(const __grid_constant__ KernelArgs args,
                      const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_k64,
                      const __grid_constant__ CUtensorMap tmap_k32,
                      const __grid_constant__ CUtensorMap tmap_v) {
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
      ptx::mbar_init(sh.bar(kBarQEmpty + i), 1);
      ptx::mbar_init(sh.bar(kBarSFull + i), 1);
      ptx::mbar_init(sh.bar(kBarItemFull + i), 1);
      ptx::mbar_init(sh.bar(kBarItemEmpty + i), kItemConsumers);
    }
    for (int s = 0; s < kRing; ++s) {
      ptx::mbar_init(sh.bar(kBarKVFull + s), 2);
      ptx::mbar_init(sh.bar(kBarKVEmpty + s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(sh.bar(kBarPFull + i), kPairWgArrivals);
      ptx::mbar_init(sh.bar(kBarPvDone + i), 1);
    }
    ptx::mbar_init(sh.bar(kBarOEmpty), kPairWarpArrivals);
    ptx::mbar_init(sh.bar(kBarSplitWritten), kSoftmaxWarps);
    ptx::mbar_init(sh.bar(kBarSplitDecided), 1);
    ptx::mbar_init(sh.bar(kBarTail), 1);
    ptx::mbar_init(sh.bar(kBarDrain), 1);
    ptx::mbar_init(sh.bar(kBarWgX), kSoftmaxWarps);
    *sh.abort_flag() = 0;
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
      if (lane == 0) producer_role(args, sh, &tmap_q, &tmap_k64, &tmap_k32, &tmap_v);
      __syncwarp();
    } else if (warp == 1) {
      if (sh.rank == 0) mma_role(args, sh, tmem, lane);
    }
  } else {
    ptx::setmaxnreg_inc<kSoftmaxRegs>();
    softmax_role(args, sh, tmem);
  }

  ptx::tc_fence_before();
  ptx::cluster_sync();  // no remote traffic after this point; MMAs drained
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem, kTmemCols);
  }
}

// ================================================================ host side
thread_local std::string t_last_error;

tpsa_status fail(tpsa_status s, const std::string& msg) {
  t_last_error = "[TPSA] " + msg;
  return s;
}

tpsa_status cuda_fail(cudaError_t e, const char* what) {
  return fail(TPSA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  int major = 0;
  bool attr_set = false;
  int max_pairs = 0;  // co-resident CTA pairs (clusters of 2)
};

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
    e = cudaFuncSetAttribute(tpsa_paged_kernel<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    e = cudaFuncSetAttribute(tpsa_paged_kernel<true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (st.sm_count / 2), 1, 1);
    cfg.blockDim = dim3(kNumThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, tpsa_paged_kernel<false>, &cfg);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
    if (clusters <= 0) return fail(TPSA_ERR_CUDA, "no CTA pair fits on this device");
    st.max_pairs = clusters;
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

// `pairs`: CTA pairs (2-SM clusters) the launch runs; each pair runs one item
// at a time.
tpsa_status build_plan(int64_t query_tokens, int64_t query_start, int64_t seq_len,
                       int64_t prompt_len, int32_t kv_heads, int32_t pairs,
                       float scale, tpsa_plan* p) {
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
  const double target = static_cast<double>(tiles) / pairs;
  int32_t split = static_cast<int32_t>(0.7 * target);
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
  p->grid = 2 * (p->total_items < pairs ? p->total_items : pairs);
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
  st = build_plan(query_tokens, query_start, seq_len, prompt_len, kv_heads, dev->max_pairs,
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

  cudaStream_t s = static_cast<cudaStream_t>(stream);
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

  if (visited != nullptr || tile_counter != nullptr) {
    tpsa_paged_kernel<true><<<p.grid, kNumThreads, kSmemBytes, s>>>(args, tq, tk64, tk32, tv);
  } else {
    tpsa_paged_kernel<false><<<p.grid, kNumThreads, kSmemBytes, s>>>(args, tq, tk64, tk32, tv);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return TPSA_OK;
}

// ------------------------------------------------ static-scratch variant
// Scratch for tpsa_paged_attention_static_scratch: the same control words and
// split-KV partial slots that tpsa_paged_attention keeps in a caller-provided
// workspace, in one module-global array per device instead.  Its maximum
// size, 16 MiB, covers 8192-token query chunks over contexts up to 128K
// tokens (10.2 MiB there).
constexpr uint64_t kStaticScratchBytes = uint64_t{16} << 20;
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
  int32_t pairs = sm_count / 2;
  if (sm_count <= 0) {
    DeviceState* dev = nullptr;
    tpsa_status st = device_state(&dev);
    if (st != TPSA_OK) return st;
    pairs = dev->max_pairs;
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
  st = build_plan(query_tokens, query_start, seq_len, prompt_len, TPSA_KV_HEADS, dev->max_pairs,
                  scale, &p);
  if (st != TPSA_OK) return st;
  if (static_cast<uint64_t>(p.workspace_bytes) > kStaticScratchBytes) {
    return fail(TPSA_ERR_WORKSPACE,
                "this call needs " + std::to_string(p.workspace_bytes) +
                    " bytes of scratch; the static scratch holds " +
                    std::to_string(kStaticScratchBytes) +
                    " bytes (16 MiB): use tpsa_paged_attention with a caller workspace");
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
TPSA_API uint32_t tpsa_debug_trace(uint32_t role, unsigned long long* out, uint32_t max_events) {
  uint32_t n[kTraceRoles] = {0, 0, 0, 0};
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
