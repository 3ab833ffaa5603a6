// TriangleMix paged sparse prefill attention for B200 (sm_100a).
//
// One persistent launch computes, for every query row, the dense causal
// prefix / sink+local-window middle / dense causal tail key set of the
// reference operator (operator/op_kernel/triangle_paged_fia_fast_path.h:
// 209-438) under one online softmax, reading K/V pages straight from the
// BSND paged cache through the block table and writing bf16 output into the
// caller's buffer.
//
// A work item is (64-token query block, kv head, key-tile range).  Its 256
// rows (64 tokens x 4 GQA heads) are two M=128 query tiles of one CTA:
// tile 0 holds query heads {4h, 4h+1}, tile 1 heads {4h+2, 4h+3}.  Both read
// the same K/V tile from shared memory, so every K/V byte loaded serves 4
// query heads, and both have the same key set.  Softmax warpgroup x owns
// query tile x for the whole item: its rows' running reference max, row sum
// and O accumulator never leave it, so the two warpgroups run independently.
//
// Roles (384 threads, one CTA per SM, persistent):
//   warp 0      K producer: Q tiles of each item, K tiles into the K ring
//   warp 1      tcgen05 MMA issuer (one elected lane) and TMEM owner
//   warp 2      work scheduler (global counter, longest items first)
//   warp 3      V producer: V tiles into the V ring
//   warps 4-7   softmax + epilogue of query tile 0
//   warps 8-11  softmax + epilogue of query tile 1
// Tensor memory (512 fp32 columns): S0 [0,128), S1 [128,256), O0 [256,384),
// O1 [384,512).  P of tile x (bf16 pairs) overwrites columns 64-127 of Sx
// and PV reads it there.  Per query tile the MMA order is
//   QK(t) -> softmax(t) -> PV(t) -> QK(t+1)
// (QK(t+1) may be issued right after PV(t): the tensor pipe runs them in
// order, so PV(t) has read P before QK(t+1) overwrites Sx), and the issuer
// interleaves the two tiles: PV0(t), QK0(t+1), PV1(t), QK1(t+1), so one
// tile's softmax overlaps the other tile's MMAs.  PV(t) runs in two 64-key
// halves; the first starts as soon as P of keys 0-63 is written.
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

// Optional event trace of one CTA (build with -DTPSA_TRACE; the CTA is
// TPSA_TRACE_CTA), compiled out of the library otherwise.  Each tracing
// thread owns one buffer and a register counter, so a trace point is two
// plain stores and a clock read.
#ifdef TPSA_TRACE
#ifndef TPSA_TRACE_CTA
#define TPSA_TRACE_CTA 0  // CTA whose events are recorded
#endif
// Roles: 0 K producer, 1 MMA issuer, 2-3 softmax warpgroups, 4 V producer.
constexpr uint32_t kTraceRoles = 5;
constexpr uint32_t kTraceCap = 1u << 14;
__device__ unsigned long long g_trace[kTraceRoles][kTraceCap][2];
__device__ uint32_t g_trace_n[kTraceRoles];
#define TPSA_TRACE_STATE uint32_t tr_n_ = 0
#ifndef TPSA_TRACE_EVMASK
#define TPSA_TRACE_EVMASK ~0ull  // events recorded (bit ev)
#endif
#define TPSA_TR(role, ev, arg)                                                    \
  do {                                                                            \
    if (((TPSA_TRACE_EVMASK >> (ev)) & 1ull) && blockIdx.x == TPSA_TRACE_CTA &&   \
        tr_n_ < kTraceCap) {                                                      \
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
constexpr int kSoftmaxWarps = 8;  // two warpgroups, one per query tile
constexpr int kFirstSoftmaxWarp = 4;
// Register split (setmaxnreg): the control warpgroup (warps 0-3) keeps 40
// registers a thread, the two softmax warpgroups 232, within the launch's
// 384 x 168: 128 x 40 + 256 x 232 = 64512.  (Measured against 56 / 224: 0.4 %
// faster at 8K and 32K/q8K, bit-identical output.)
constexpr uint32_t kControlRegs = 40;
constexpr uint32_t kSoftmaxRegs = 232;
static_assert(128 * kControlRegs + 256 * kSoftmaxRegs <= 384 * 168, "register split");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 256;  // O0 at 256, O1 at 384 (S0 at 0, S1 at 128)
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;  // 1 s per wait
constexpr uint64_t kAbortSettleNs = 200000ull;      // let in-flight TMA land
constexpr float kRescaleLog2 = 8.0f;  // lazy O rescale threshold (log2 units)

// Shared memory per CTA (offsets from a 1024-byte aligned base).
constexpr uint32_t kQHalfBytes = 128 * 128;           // 128 rows x 64 bf16
constexpr uint32_t kQTileBytes = 2 * kQHalfBytes;     // one query tile (two d-halves)
constexpr uint32_t kKvHalfBytes = 128 * 128;          // 128 keys x 64 d
constexpr uint32_t kKvSlotBytes = 2 * kKvHalfBytes;   // one key tile of K, or of V
constexpr int kKRing = 2;
constexpr int kVRing = 2;
// Output staging: 4 KB per softmax warp (its 32 rows x 64 columns as bf16,
// 128-byte swizzled), stored to `out` by the warp's own TMA store.
// (Measured: giving this space to a third K slot, with the staging in the K
// slot of the item's last tile, was 3.5 % slower at 8K, although the K loads
// then run a tile further ahead.)
constexpr uint32_t kOutStageBytes = 32 * 128;
constexpr uint32_t kOffQ = 0;                                   // [query tile][d half]
constexpr uint32_t kOffK = kOffQ + 2 * kQTileBytes;              // K ring
constexpr uint32_t kOffV = kOffK + kKRing * kKvSlotBytes;        // V ring
constexpr uint32_t kOffOut = kOffV + kVRing * kKvSlotBytes;      // output staging
constexpr uint32_t kOffBar = kOffOut + 8 * kOutStageBytes;

enum BarId : uint32_t {
  kBarQFull = 0,                        // [2] query tile x landed
  kBarQEmpty = kBarQFull + 2,           // [2] query tile x free (its last QK done)
  kBarKFull = kBarQEmpty + 2,           // [kKRing] K tile landed
  kBarKEmpty = kBarKFull + kKRing,      // [kKRing] K slot free (both QKs done)
  kBarVFull = kBarKEmpty + kKRing,      // [kVRing] V tile landed (tail rows zeroed)
  kBarVEmpty = kBarVFull + kVRing,      // [kVRing] V slot free (both PVs done)
  kBarSFull = kBarVEmpty + kVRing,      // [2] S of tile x computed
  kBarPFull = kBarSFull + 2,            // [2] P of tile x written (4 warps)
  kBarPHalf = kBarPFull + 2,            // [2] P of keys 0-63 of tile x written (4 warps)
  kBarOFull = kBarPHalf + 2,            // [2] the item's last PV of tile x done
  kBarItemFull = kBarOFull + 2,         // [2] item record written
  kBarItemEmpty = kBarItemFull + 2,     // [2] item record consumed
  kBarTail = kBarItemEmpty + 2,         // V producer: a tail tile landed
  kBarDrain = kBarTail + 1,             // MMA issuer: all MMAs complete
  kBarProbe = kBarDrain + 1,            // test hook: never arrived on
  kBarPieceDone = kBarProbe + 1,        // softmax warps: a split piece merged
  kNumBars
};
// item_empty: K producer, V producer, MMA warp, 8 softmax warps.
constexpr uint32_t kItemConsumers = 3 + kSoftmaxWarps;

constexpr uint32_t kOffItemSlots = (kOffBar + kNumBars * 8 + 15) & ~15u;  // 2 x ItemRec
constexpr uint32_t kOffTmemSlot = kOffItemSlots + 2 * 64;
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
constexpr uint32_t kOffSplitLast = kOffAbort + 4;      // int32 [query tile][2]
constexpr uint32_t kOffCounters = kOffSplitLast + 16;  // uint32 [4]: split written / decided per tile
constexpr uint32_t kOffLastCta = kOffCounters + 16;    // int32: this CTA finished the launch last
constexpr uint32_t kSmemUsed = kOffLastCta + 16;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // alignment slack
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

// Control words: [0] next work item, [1] CTAs that have finished, [64..] one
// split counter per (tail block, kv head, query tile).  They start every
// launch at zero.  Either they live in a library-owned control block of the
// launching stream, which the last CTA of each launch zeroes again on its
// way out (KernelArgs::ctl_reset_words), or in the first bytes of the
// caller's workspace, which the launcher clears before the kernel.
constexpr int kCtlNextItem = 0;
constexpr int kCtlExited = 1;
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
  uint32_t probe_wait_ns;      // test hook (0 = off): see scheduler_role
  int32_t coop_merge;          // split pieces merge together (softmax_role)
  int32_t ctl_reset_words;     // > 0: the last CTA zeroes ctl[0, ctl_reset_words)
};



struct Smem {
  uint8_t* base;
  uint32_t base_u32;
  __device__ uint32_t bar(uint32_t id) const { return base_u32 + kOffBar + 8 * id; }
  __device__ volatile int* abort_flag() const {
    return reinterpret_cast<volatile int*>(base + kOffAbort);
  }
  __device__ uint32_t counter(uint32_t id) const { return base_u32 + kOffCounters + 4 * id; }
  __device__ uint4* item_slot(uint32_t i) const {
    return reinterpret_cast<uint4*>(base + kOffItemSlots + 64 * i);
  }
};

__device__ __forceinline__ void raise_status(uint32_t bits) {
  atomicOr(&g_device_status, bits);
}

#ifdef TPSA_TRACE
// Start and end (globaltimer ns) and items run of every CTA of the last launch.
__device__ unsigned long long g_cta_span[1024][3];
// Per CTA, softmax warpgroup and item (first 8): {idx | splits << 32,
// globaltimer before taking the item, after taking it, after O is complete,
// and for a split piece after its partial is written, after the wait for the
// other pieces, after the merge}.
__device__ unsigned long long g_item_trace[1024][2][8][8];
#define TPSA_ITEM_REC(n, f, v)                                          \
  do {                                                                  \
    if (row == 0 && blockIdx.x < 1024 && (n) < 8) g_item_trace[blockIdx.x][x][n][f] = (v); \
  } while (0)
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
#define TPSA_ITEM_REC(n, f, v) \
  do {                         \
  } while (0)
#endif



// Bounded wait: gives up after limit_ns or as soon as another role of this
// CTA has aborted; on timeout it sets the CTA's abort flag and records
// TPSA_DEVICE_WAIT_TIMEOUT.
__device__ __forceinline__ bool wait_bar_slow(uint32_t bar, uint32_t parity,
                                           volatile int* abort_flag,
                                           uint64_t limit_ns = kWaitTimeoutNs) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (true) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (ptx::globaltimer_ns() - t0 > limit_ns) {
      *abort_flag = 1;
      raise_status(TPSA_DEVICE_WAIT_TIMEOUT);
      TPSA_NOTE_TIMEOUT(bar, parity);
      return false;
    }
  }
}

__device__ __forceinline__ bool wait(const Smem& sh, uint32_t bar, uint32_t parity) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  return wait_bar_slow(bar, parity, sh.abort_flag());
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
// (wrap-safe comparison); gives up like wait.
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

__device__ __forceinline__ bool wait_count(const Smem& sh, uint32_t id, uint32_t target) {
  const uint32_t addr = sh.counter(id);
  if (static_cast<int32_t>(ptx::ld_acquire_shared(addr) - target) >= 0) return true;
  return wait_count_slow(sh.abort_flag(), addr, target);
}

// Bounded wait until the global counter at `addr` (written by other CTAs
// with release adds) reaches `target`; gives up like wait.  Polls back off
// with a short sleep so that waiting CTAs do not flood the L2 slice.
__device__ __noinline__ bool wait_global_count(const Smem& sh, const int32_t* addr,
                                               int32_t target) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (ptx::ld_acquire_global(addr) < target) {
    if (*sh.abort_flag()) return false;
    if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
      *sh.abort_flag() = 1;
      raise_status(TPSA_DEVICE_WAIT_TIMEOUT);
      TPSA_NOTE_TIMEOUT(0u, static_cast<uint32_t>(target) | 0x80000000u);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

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
// Work items flow from the CTA's scheduler to every consumer through a
// 2-slot ring in shared memory.  A slot holds an item record: the item
// index (total_items or above ends the kernel), the decoded item and its
// block's tile geometry, decoded once by the scheduler so that no consumer
// repeats that integer arithmetic.
struct alignas(16) ItemRec {
  int32_t idx;
  tpsa_item it;
  BlockTiles bt;
  // Item tiles only 64 keys wide (the others are 128, or 80 for the
  // composite tile): bit 0 the item's tile 0, bit 1 its tile 1, bit 2 its
  // last tile (the sink tile and a band or key range that starts or ends
  // half-way through a page).  Bit 3: the item's tile 0 is the 80-key
  // composite tile.  Bits 8 and up: the item's request within the launch.
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
    rec.narrow |= w == kKeyGrain ? 1u : 0u;
    rec.narrow |= w == kCompositeKeys ? 8u : 0u;
    if (last >= 1) {
      tile_keys(rec.bt, rec.it.tile_begin + 1, &k0, &w);
      rec.narrow |= w == kKeyGrain ? 2u : 0u;
    }
    tile_keys(rec.bt, rec.it.tile_begin + last, &k0, &w);
    rec.narrow |= w == kKeyGrain ? 4u : 0u;
  }
  return rec;
}


// The fields of item record n the MMA issuer uses: its index, tile count
// and narrow-tile bits.
struct ItemBrief {
  int32_t idx, ntiles;
  uint32_t narrow;
  bool piece;  // a split piece of a cooperative-merge launch: the scheduler
               // publishes the next item only after this one is merged
};

__device__ __forceinline__ bool take_item(const Smem& sh, uint32_t n, ItemRec* rec) {
  const uint32_t slot = n % 2;
  if (!wait(sh, sh.bar(kBarItemFull + slot), (n / 2) & 1)) return false;
  const uint4* src = sh.item_slot(slot);
  uint4* dst = reinterpret_cast<uint4*>(rec);
#pragma unroll
  for (int j = 0; j < 4; ++j) dst[j] = src[j];
  return true;
}

// The fields of item record n the MMA issuer uses (index, tile count,
// narrow-tile bits).
__device__ __forceinline__ bool take_item_brief(const Smem& sh, uint32_t n, ItemBrief* b,
                                                bool coop) {
  const uint32_t slot = n % 2;
  if (!wait(sh, sh.bar(kBarItemFull + slot), (n / 2) & 1)) return false;
  const int32_t* w = reinterpret_cast<const int32_t*>(sh.item_slot(slot));
  b->idx = w[offsetof(ItemRec, idx) / 4];
  b->ntiles = w[(offsetof(ItemRec, it) + offsetof(tpsa_item, tile_end)) / 4] -
              w[(offsetof(ItemRec, it) + offsetof(tpsa_item, tile_begin)) / 4];
  b->narrow = static_cast<uint32_t>(w[offsetof(ItemRec, narrow) / 4]);
  b->piece = coop && w[(offsetof(ItemRec, it) + offsetof(tpsa_item, num_splits)) / 4] > 1;
  return true;
}

__device__ __forceinline__ void release_item(const Smem& sh, uint32_t n) {
  ptx::mbar_arrive(sh.bar(kBarItemEmpty + n % 2));
}

// Key count class of tile j of an item (see ItemRec::narrow): 64 keys,
// the 80-key composite tile, or 128 keys.
enum TileWidth : uint32_t { kWide = 0, kNarrow = 1, kComposite = 2 };
__device__ __forceinline__ uint32_t tile_width(uint32_t narrow, int32_t j, int32_t ntiles) {
  if ((j < 2 && ((narrow >> j) & 1u)) || (j == ntiles - 1 && (narrow & 4u))) return kNarrow;
  return (j == 0 && (narrow & 8u)) ? kComposite : kWide;
}


// ------------------------------------------------------------ scheduler
// One thread: takes items from the grid-wide counter (longest first),
// decodes each into an item record
// and publishes it into the CTA's two-slot item ring.  An item is claimed
// only once its ring slot is free, i.e. once the softmax warpgroups have
// finished the item two before it: a CTA then holds at most the item it
// runs and the next one, so CTAs finish the launch within about one item of
// each other.
//
// Test hook (probe_wait_ns != 0): before claiming anything, the scheduler
// waits on kBarProbe, which nothing arrives on, with that short limit.  The
// wait runs out, sets the abort flag and TPSA_DEVICE_WAIT_TIMEOUT; the other
// roles, all still waiting for their first item record, leave through their
// abort paths.  No item is claimed, so no load, MMA or store is ever issued.
template <bool kVarlen>
__device__ void scheduler_role(const KernelArgs& a, const Smem& sh) {
  const tpsa_plan& p = a.plan;
  if (a.probe_wait_ns != 0) {
    wait_bar_slow(sh.bar(kBarProbe), 0, sh.abort_flag(), a.probe_wait_ns);
    return;
  }
  uint32_t piece_par = 0;
  for (uint32_t n = 0;; ++n) {
    const uint32_t slot = n % 2;
    if (!wait(sh, sh.bar(kBarItemEmpty + slot), ((n / 2) & 1) ^ 1)) break;
    const int32_t next = atomicAdd(a.ctl + kCtlNextItem, 1);
#ifdef TPSA_TRACE
    if (blockIdx.x < 1024 && next < p.total_items) g_cta_span[blockIdx.x][2] = n + 1;
#endif
    ItemRec rec;
    if (kVarlen) {
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
    const uint4* words = reinterpret_cast<const uint4*>(&rec);
#pragma unroll
    for (int j = 0; j < 4; ++j) sh.item_slot(slot)[j] = words[j];
    ptx::mbar_arrive(sh.bar(kBarItemFull + slot));
    if (rec.idx >= p.total_items) break;
    // A split piece waits for the other pieces of its block (softmax_role):
    // claim nothing more until it is merged.
    if (a.coop_merge && rec.it.num_splits > 1) {
      if (!wait(sh, sh.bar(kBarPieceDone), piece_par)) break;
      piece_par ^= 1u;
    }
  }
}

// ------------------------------------------------------------ producers
// K side: for each item the first K tile, then the two query tiles (each
// waits until the previous item's last QK of that tile completed), then the
// remaining K tiles.  V side: the V tiles.  One thread each.  A 128-key tile
// (always from one page) is one 128-row box per 64-column half (tk128 /
// tv128); a 64-key tile one 64-row box; the composite tile a 64-row box of
// the band edge into rows 0-63 and a 16-row box of the sink into rows 64-79
// (tk16 / tv16).
// (Measured at 8K: 128-row V boxes and no L2 prefetch of the query rows, 2.7 %
// faster than 64-row V boxes with the prefetch; L2 prefetches of the next
// item's K/V tiles were 10 % slower.)
template <bool kVarlen>
__device__ void producer_role(const KernelArgs& a, const Smem& sh, const CUtensorMap* tq,
                              const CUtensorMap* tk128, const CUtensorMap* tk64,
                              const CUtensorMap* tk16, const CUtensorMap* tv,
                              const CUtensorMap* tv128, const CUtensorMap* tv16, bool v_side) {
  const tpsa_plan& p = a.plan;
  if (v_side) {
    ptx::prefetch_tmap(tv);
    ptx::prefetch_tmap(tv128);
    ptx::prefetch_tmap(tv16);
  } else {
    ptx::prefetch_tmap(tq);
    ptx::prefetch_tmap(tk128);
    ptx::prefetch_tmap(tk64);
    ptx::prefetch_tmap(tk16);
  }
  const uint32_t bar_full = sh.bar(v_side ? kBarVFull : kBarKFull);
  const uint32_t bar_empty = sh.bar(v_side ? kBarVEmpty : kBarKEmpty);
  const uint32_t ring_base = sh.base_u32 + (v_side ? kOffV : kOffK);
  const uint32_t ring_n = v_side ? kVRing : kKRing;
  uint32_t ring = 0, q_iter = 0, tail_iter = 0;
  bool ok = true;
  TPSA_TRACE_STATE;
  const uint32_t trole = v_side ? 4 : 0;
  (void)trole;
  for (uint32_t n = 0; ok; ++n) {
    ItemRec rec;
    if (!take_item(sh, n, &rec)) break;
    release_item(sh, n);
    if (rec.idx >= p.total_items) break;
    TPSA_TR(trole, 20, rec.idx);
    const tpsa_item& it = rec.it;
    const BlockTiles& bt = rec.bt;
    const ReqDesc& rq = a.reqs[kVarlen ? rec.req() : 0];
    const int32_t* table = kVarlen ? a.block_table + rq.table_off : a.block_table;
    const int32_t req_seq_len = kVarlen ? rq.plan.seq_len : p.seq_len;
    const int32_t q_row0 = kVarlen ? rq.q_row0 : 0;

    // Cache row (page * 128 + slot) of logical key k; a block-table entry
    // outside the cache is flagged and points fully out of bounds, where
    // TMA fills zeros.
    auto cache_row = [&](int32_t k) -> int32_t {
      const int32_t page = __ldg(table + k / kPageSize);
      if (page < 0 || page >= a.num_pages) {
        raise_status(TPSA_DEVICE_BAD_PAGE);
        return -kPageSize;
      }
      return page * kPageSize + (k % kPageSize);
    };
    for (int32_t t = it.tile_begin; t < it.tile_end && ok; ++t) {
      int32_t k0, w;
      tile_keys(bt, t, &k0, &w);
      // Keys 0-63 of the tile start at k0, the keys after them at k_up (the
      // sink, key 0, in the composite tile, else k0 + 64 in the same page).
      const int32_t k_up = upper_key(bt, t, k0);
      const bool composite = w == kCompositeKeys;
      const int32_t tok = cache_row(k0);
      const int32_t tok_up = composite ? cache_row(k_up) : tok + kKeyGrain;
      if (a.tiles != nullptr && !v_side) {
        atomicAdd(a.tiles, 1ull);
        atomicAdd(a.tiles + 1, static_cast<unsigned long long>(w));
      }
      const uint32_t s = ring % ring_n;
      if (!wait(sh, bar_empty + 8 * s, ((ring / ring_n) & 1) ^ 1)) { ok = false; break; }
      ++ring;
      TPSA_TR(trole, 22, t);
      const uint32_t dst = ring_base + s * kKvSlotBytes;
      if (!v_side) {
        // Keys at or beyond seq_len (unwritten slots of the last page) only
        // meet masked scores, which select -inf whatever they hold.
        const CUtensorMap* km = w == kTileKeys ? tk128 : tk64;
        ptx::mbar_arrive_expect_tx(bar_full + 8 * s, static_cast<uint32_t>(w) * kHeadDim * 2);
        for (int dh = 0; dh < 2; ++dh) {
          ptx::tma_load_3d(dst + dh * kKvHalfBytes, km, dh * 64, it.kv_head, tok,
                           bar_full + 8 * s);
          if (composite) {
            ptx::tma_load_3d(dst + dh * kKvHalfBytes + 64 * 128, tk16, dh * 64, it.kv_head, tok_up,
                             bar_full + 8 * s);
          }
        }
        if (t == it.tile_begin) {
          // The item's query tiles, after its first K tile: query tile x
          // (heads 4h + 2x, 4h + 2x + 1) frees when the previous item's last
          // QK of that tile completes.
          for (uint32_t x = 0; x < 2; ++x) {
            if (q_iter > 0 && !wait(sh, sh.bar(kBarQEmpty + x), (q_iter - 1) & 1)) {
              ok = false;
              break;
            }
            ptx::mbar_arrive_expect_tx(sh.bar(kBarQFull + x), kQTileBytes);
            for (int dh = 0; dh < 2; ++dh) {
              ptx::tma_load_3d(sh.base_u32 + kOffQ + x * kQTileBytes + dh * kQHalfBytes, tq,
                               dh * 64, it.kv_head * kGroupSize + 2 * static_cast<int32_t>(x),
                               q_row0 + it.block * kBlockQ, sh.bar(kBarQFull + x));
            }
            TPSA_TR(trole, 21, x);
          }
          ++q_iter;
        }
      } else {
        const bool tail = k0 + min_i(w, kKeyGrain) > req_seq_len ||
                          (w > kKeyGrain && k_up + (w - kKeyGrain) > req_seq_len);
        // Values at or beyond seq_len may be unwritten cache slots: such a
        // tile lands on a private barrier, those rows are zeroed (so that
        // P = 0 never meets a NaN), then the slot is published.
        const uint32_t lbar = tail ? sh.bar(kBarTail) : bar_full + 8 * s;
        ptx::mbar_arrive_expect_tx(lbar, static_cast<uint32_t>(w) * kHeadDim * 2);
        for (int dh = 0; dh < 2; ++dh) {
          if (w == kTileKeys) {
            ptx::tma_load_3d(dst + dh * kKvHalfBytes, tv128, dh * 64, it.kv_head, tok, lbar);
          } else {
            ptx::tma_load_3d(dst + dh * kKvHalfBytes, tv, dh * 64, it.kv_head, tok, lbar);
            if (composite) {
              ptx::tma_load_3d(dst + dh * kKvHalfBytes + 64 * 128, tv16, dh * 64, it.kv_head,
                               tok_up, lbar);
            }
          }
        }
        if (tail) {
          if (!wait(sh, sh.bar(kBarTail), tail_iter & 1)) { ok = false; break; }
          ++tail_iter;
          for (int32_t row = 0; row < w; ++row) {
            const int32_t key = row < kKeyGrain ? k0 + row : k_up + row - kKeyGrain;
            if (key < req_seq_len) continue;
            for (int dh = 0; dh < 2; ++dh) {
              uint4* d4 = reinterpret_cast<uint4*>(sh.base + (dst - sh.base_u32) +
                                                   dh * kKvHalfBytes + row * 128);
#pragma unroll
              for (int j = 0; j < 8; ++j) d4[j] = make_uint4(0, 0, 0, 0);
            }
          }
          ptx::fence_proxy_async_smem();
          ptx::mbar_arrive(bar_full + 8 * s);
        }
      }
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
// The whole warp runs this role; operands are warp-uniform and one lane,
// elected once, issues every tcgen05 instruction.
__device__ void mma_role(const KernelArgs& a, const Smem& sh, uint32_t tmem) {
  const tpsa_plan& p = a.plan;
  const uint32_t leader = ptx::elect_one();
  auto warp_wait = [&](uint32_t bar, uint32_t parity) -> bool {
    return __all_sync(0xffffffffu, wait(sh, bar, parity));
  };
  const uint64_t q_desc0 = ptx::smem_desc_sw128(sh.base_u32 + kOffQ, 16, 1024);
  const uint64_t k_desc0 = ptx::smem_desc_sw128(sh.base_u32 + kOffK, 16, 1024);
  const uint64_t v_desc0 = ptx::smem_desc_sw128(sh.base_u32 + kOffV, kKvHalfBytes, 1024);
  constexpr uint32_t kIdQk128 = ptx::idesc_bf16_f32(128, 128, 0);
  constexpr uint32_t kIdQk64 = ptx::idesc_bf16_f32(128, 64, 0);
  constexpr uint32_t kIdQk80 = ptx::idesc_bf16_f32(128, kCompositeKeys, 0);
  static_assert(kCompositeKeys % 16 == 0, "an M = 128 MMA takes N in steps of 16");
  constexpr uint32_t kIdPv = ptx::idesc_bf16_f32(128, 128, 1);

  // Descriptor start addresses are in 16-byte units in the low word; the
  // loop adds offsets to 32-bit low words prepared once.
  const uint32_t q_lo = static_cast<uint32_t>(q_desc0), q_hi = static_cast<uint32_t>(q_desc0 >> 32);
  const uint32_t k_lo = static_cast<uint32_t>(k_desc0), k_hi = static_cast<uint32_t>(k_desc0 >> 32);
  const uint32_t v_lo = static_cast<uint32_t>(v_desc0), v_hi = static_cast<uint32_t>(v_desc0 >> 32);
  auto desc = [](uint32_t lo, uint32_t hi) { return (static_cast<uint64_t>(hi) << 32) | lo; };
  constexpr uint32_t kHalfUnits = kQHalfBytes >> 4;
  constexpr uint32_t kQTileUnits = kQTileBytes >> 4;
  constexpr uint32_t kSlotUnits = kKvSlotBytes >> 4;
  static_assert(kQHalfBytes == kKvHalfBytes, "Q and K d-halves share offsets");
  auto commit = [&](uint32_t bar) { ptx::umma_commit_if(leader, bar); };
  // S_x = Q_x K^T for the K tile in ring slot ks (N = 128, 64 or 80).
  auto issue_qk = [&](uint32_t x, uint32_t ks, uint32_t width) {
    const uint32_t d = tmem + (x << 7);
    const uint32_t idesc =
        width == kNarrow ? kIdQk64 : (width == kComposite ? kIdQk80 : kIdQk128);
    const uint32_t qb = q_lo + x * kQTileUnits;
    const uint32_t kb = k_lo + ks * kSlotUnits;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t o = (k / 4) * kHalfUnits + (k % 4) * 2;
      ptx::umma_ss_if(leader, d, desc(qb + o, q_hi), desc(kb + o, k_hi), idesc, k > 0 ? 1u : 0u);
    }
  };
  // O_x (+)= P_x V for keys [64 half, 64 half + 16 steps) of the V tile in
  // ring slot vs (16 keys a step: 4 steps, or 1 for the sink slice of the
  // composite tile).
  auto issue_pv = [&](uint32_t x, uint32_t vs, uint32_t half, bool first, int steps) {
    const uint32_t d = tmem + kTmemO + (x << 7);
    const uint32_t pa = tmem + (x << 7) + 64 + half * 32;
    const uint32_t vb = v_lo + vs * kSlotUnits + half * (8192 >> 4);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (k < steps) {
        ptx::umma_ts_if(leader, d, pa + k * 8, desc(vb + k * (2048 >> 4), v_hi), kIdPv,
                        (first && half == 0 && k == 0) ? 0u : 1u);
      }
    }
  };
  static_assert(kSinkSlice == 16, "the sink slice is one 16-key PV step");

  TPSA_TRACE_STATE;
  const bool tr = (threadIdx.x & 31) == 0;
  uint32_t n_item = 0;
  uint32_t ks = 0, k_phase = 0;  // K ring cursor of the next QK
  uint32_t vs = 0, v_phase = 0;  // V ring cursor of the next PV
  uint32_t p_par = 0;            // P-full phase (same for both tiles)
  bool ok = true;
  // Current item.
  ItemBrief cur;
  bool got = take_item_brief(sh, n_item, &cur, a.coop_merge != 0);
  if (!__all_sync(0xffffffffu, got)) ok = false;
  __syncwarp();
  if (ok && (threadIdx.x & 31) == 0) release_item(sh, n_item);
  if (ok) ++n_item;
  bool done = !ok || cur.idx >= p.total_items;
  uint32_t q_iter = 0;
  // First QKs of an item that no PV precedes: the launch's first item, and
  // the item after a split piece.
  auto first_qks = [&](const ItemBrief& it) -> bool {
    const int32_t nt = it.ntiles;
    const uint32_t wid = tile_width(it.narrow, 0, nt);
    for (uint32_t x = 0; x < 2; ++x) {
      if (!warp_wait(sh.bar(kBarQFull + x), q_iter & 1)) return false;
      if (x == 0 && !warp_wait(sh.bar(kBarKFull + ks), k_phase)) return false;
      ptx::tc_fence_after();
      issue_qk(x, ks, wid);
      commit(sh.bar(kBarSFull + x));
      if (nt == 1) commit(sh.bar(kBarQEmpty + x));
    }
    commit(sh.bar(kBarKEmpty + ks));
    ks = (ks + 1) % kKRing;
    k_phase ^= ks == 0 ? 1u : 0u;
    ++q_iter;
    return true;
  };
  if (!done) ok = first_qks(cur);
  while (ok && !done) {
    const int32_t nt = cur.ntiles;
    ItemBrief nxt;
    bool nxt_valid = false;
    for (int32_t j = 0; j < nt && ok; ++j) {
      const uint32_t wid = tile_width(cur.narrow, j, nt);
      // The QK that follows PV(j) for each tile: tile j + 1 of this item, or
      // tile 0 of the next item.
      bool has_next = j + 1 < nt;
      bool new_item = false;
      bool next_last = false;
      uint32_t next_wid = kWide;
      if (has_next) {
        next_wid = tile_width(cur.narrow, j + 1, nt);
        next_last = j + 1 == nt - 1;
      } else if (!cur.piece) {
        const bool g = take_item_brief(sh, n_item, &nxt, a.coop_merge != 0);
        if (!__all_sync(0xffffffffu, g)) { ok = false; break; }
        __syncwarp();
        if ((threadIdx.x & 31) == 0) release_item(sh, n_item);
        ++n_item;
        nxt_valid = nxt.idx < p.total_items;
        if (tr) TPSA_TR(1, 10, nxt.idx);
        if (nxt_valid) {
          const int32_t nn = nxt.ntiles;
          has_next = true;
          new_item = true;
          next_wid = tile_width(nxt.narrow, 0, nn);
          next_last = nn == 1;
        }
      }
      for (uint32_t x = 0; x < 2 && ok; ++x) {
        // PV of keys 0-63 as soon as their P is written, then keys 64-127.
        if (!warp_wait(sh.bar(kBarPHalf + x), p_par)) { ok = false; break; }
        if (tr) TPSA_TR(1, 13, x);
        if (x == 0 && !warp_wait(sh.bar(kBarVFull + vs), v_phase)) { ok = false; break; }
        if (tr && x == 0) TPSA_TR(1, 14, j);
        ptx::tc_fence_after();
        issue_pv(x, vs, 0, j == 0, 4);
        if (!warp_wait(sh.bar(kBarPFull + x), p_par)) { ok = false; break; }
        ptx::tc_fence_after();
        if (wid != kNarrow) issue_pv(x, vs, 1, false, wid == kComposite ? 1 : 4);
        if (x == 1) commit(sh.bar(kBarVEmpty + vs));
        if (j == nt - 1) commit(sh.bar(kBarOFull + x));
        if (has_next) {
          if (new_item && !warp_wait(sh.bar(kBarQFull + x), q_iter & 1)) { ok = false; break; }
          if (tr && new_item) TPSA_TR(1, 11, x);
          if (x == 0 && !warp_wait(sh.bar(kBarKFull + ks), k_phase)) { ok = false; break; }
          if (tr && x == 0) TPSA_TR(1, 17, j);
          ptx::tc_fence_after();
          issue_qk(x, ks, next_wid);
          if (tr) TPSA_TR(1, 18, x);
          commit(sh.bar(kBarSFull + x));
          if (next_last) commit(sh.bar(kBarQEmpty + x));
        }
      }
      if (!ok) break;
      p_par ^= 1;
      vs = (vs + 1) % kVRing;
      v_phase ^= vs == 0 ? 1u : 0u;
      if (has_next) {
        commit(sh.bar(kBarKEmpty + ks));
        ks = (ks + 1) % kKRing;
        k_phase ^= ks == 0 ? 1u : 0u;
        if (new_item) ++q_iter;
      }
    }
    if (ok && cur.piece) {
      // The next item is published once this piece is merged, which needs
      // its last PVs (issued above): take it only now.
      const bool g = take_item_brief(sh, n_item, &nxt, a.coop_merge != 0);
      if (!__all_sync(0xffffffffu, g)) break;
      __syncwarp();
      if ((threadIdx.x & 31) == 0) release_item(sh, n_item);
      ++n_item;
      nxt_valid = nxt.idx < p.total_items;
      if (nxt_valid) ok = first_qks(nxt);
    }
    if (!ok || !nxt_valid) break;
    cur = nxt;
  }
  // All MMAs issued by this warp complete before TMEM is released.
  commit(sh.bar(kBarDrain));
  if ((threadIdx.x & 31) == 0) drain_bar(sh.bar(kBarDrain), 0);
  __syncwarp();
}


// ------------------------------------------------------------ softmax
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

// Replaces the keys of a 32-key chunk of S (fp32 bits) that are outside the
// row's key set (bit c of m clear) by -inf, whatever the bits held.
__device__ __forceinline__ void mask_chunk(uint32_t (&r)[32], uint32_t m) {
#pragma unroll
  for (int c = 0; c < 32; ++c) r[c] = ((m >> c) & 1u) ? r[c] : 0xff800000u;
}

// Exponentials of one 32-key chunk of S (fp32 bits in r): P as 16 bf16
// pairs stored to tensor memory at p_addr, their sum added to (sum0, sum1).
// Pair c of the chunk uses the FMA-pipe polynomial when bit c of kPoly is
// set, MUFU ex2 otherwise.
template <uint32_t kPoly>
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

// Split-KV merge of one row over `ns` pieces' partials (column-major slots
// of kSlotFloats floats; this row's m at m_off, its O values at col_off +
// column * 2 kRowsPerTile), for columns [0, cw) of the thread's column
// group, written as bf16 pairs to orow.  Each round loads kCw columns of
// 32 / kCw pieces (32 independent L2 loads), so that a narrow column group
// (a slice of few rows over many pieces) needs ns kCw / 32 rounds, not
// ns / 2.  mmax and inv_sum come from merge_row_stats.
template <int kCw>
__device__ __forceinline__ void merge_columns(const float* first_slot, size_t m_off,
                                              size_t col_off, int32_t ns, int32_t cw,
                                              float mmax, float sl2, float inv_sum,
                                              uint32_t* orow) {
  constexpr int kPr = 32 / kCw;  // pieces per round
  constexpr size_t kColStride = 2 * kRowsPerTile;
#pragma unroll 1
  for (int32_t c0 = 0; c0 < cw; c0 += kCw) {
    float acc[kCw];
#pragma unroll
    for (int j = 0; j < kCw; ++j) acc[j] = 0.0f;
#pragma unroll 1
    for (int32_t sp0 = 0; sp0 < ns; sp0 += kPr) {
      float val[kPr][kCw], wgt[kPr];
#pragma unroll
      for (int u = 0; u < kPr; ++u) {
        const bool in = sp0 + u < ns;
        const float* sl = first_slot + static_cast<size_t>(sp0 + u) * kSlotFloats;
        wgt[u] = in ? __ldcg(sl + m_off) : -INFINITY;
        const float* colp = sl + col_off + static_cast<size_t>(c0) * kColStride;
#pragma unroll
        for (int j = 0; j < kCw; ++j) val[u][j] = in ? __ldcg(colp + j * kColStride) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kPr; ++u) {
        const float w = wgt[u] == -INFINITY ? 0.0f : mufu_exp2((wgt[u] - mmax) * sl2);
#pragma unroll
        for (int j = 0; j < kCw; ++j) acc[j] += w * val[u][j];
      }
    }
#pragma unroll
    for (int j = 0; j < kCw / 2; ++j) {
      orow[c0 / 2 + j] = pack_bf16x2(acc[2 * j] * inv_sum, acc[2 * j + 1] * inv_sum);
    }
  }
}

// Row max and row sum of one row over `ns` pieces' (m, l) in one pass of
// 8 pieces per round (an online log-sum-exp: the sum is rescaled when the
// max grows).  Returns 1 / sum through inv_sum.
__device__ __forceinline__ float merge_row_stats(const float* first_slot, size_t m_off,
                                                 size_t l_off, int32_t ns, float sl2,
                                                 float* inv_sum) {
  float mmax = -INFINITY, lsum = 0.0f;
#pragma unroll 1
  for (int32_t sp0 = 0; sp0 < ns; sp0 += 8) {
    float mv[8], lv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const bool in = sp0 + u < ns;
      const float* sl = first_slot + static_cast<size_t>(sp0 + u) * kSlotFloats;
      mv[u] = in ? __ldcg(sl + m_off) : -INFINITY;
      lv[u] = in ? __ldcg(sl + l_off) : 0.0f;
    }
    float bm = mmax;
#pragma unroll
    for (int u = 0; u < 8; ++u) bm = fmaxf(bm, mv[u]);
    if (bm != -INFINITY) {
      if (bm != mmax) lsum = mmax == -INFINITY ? 0.0f : lsum * mufu_exp2((mmax - bm) * sl2);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (mv[u] != -INFINITY) lsum += mufu_exp2((mv[u] - bm) * sl2) * lv[u];
      }
      mmax = bm;
    }
  }
  *inv_sum = 1.0f / lsum;
  return mmax;
}

// Per-row state of the online softmax over one item's tiles: the lazy
// reference max and the row sum relative to it.
struct RowState {
  float m_ref;
  float l_part;
};



// Where a tile lives and what its softmax needs to know.
struct TileArgs {
  uint32_t s_addr;      // the tile's S buffer (P goes to its columns 64-127)
  uint32_t o_addr;      // O (128 columns)
  uint32_t half_bar;    // P-half barrier of the tile's query tile
  int32_t k0;           // first key of the tile (keys 0-63)
  int32_t k_up;         // first key of the keys after the first 64
  bool wide;            // more than 64 keys: S columns 64-127 are scored too
  bool masked;          // some key of the tile is outside some row's key set
  bool first;           // first tile of the item (its PV overwrites O)
};


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





// Pairs of each 32-key chunk whose exponentials use the FMA-pipe polynomial
// (bit c: pair c; see exp_chunk).  None by default: measured at 8K with the
// whole row in registers (ms per launch), no pair 0.1140, 0x0001 0.1146,
// 0x0401 0.1153, 0x1111 0.1179.  (MUFU ex2 runs at 16 per clock per SM, as
// many exponentials per clock as the tensor pipe needs for this tile shape.)
#ifndef TPSA_POLY_MASK
#define TPSA_POLY_MASK 0u
#endif
constexpr uint32_t kPolyMask = TPSA_POLY_MASK;

// One key tile of query tile x, the whole row of this thread: load S (all of
// it into registers), mask, row max, move the lazy reference if this tile's
// maxima require it (O and the row sum rescaled first), exponentials and P
// into tensor memory over columns 64-127 of the S buffer.  P of keys 0-63 is
// published on t.half_bar (the P-half barrier) before the exponentials of
// keys 64-127, so their PV can start.  O holds the PVs of the earlier tiles
// of the item, all complete: S of this tile was signalled by a commit issued
// after the previous PV.  (Keeping keys 64-127 in registers and loading keys
// 0-63 twice measured 10 % slower at 8K.)
template <bool kVisit>
__device__ __forceinline__ void softmax_tile(const TileArgs& t, float sl2, int32_t q, bool sparse,
                                             RowState& st, uint32_t* visit_row,
                                             int32_t words_per_row) {
  uint32_t r0[32], r1[32], r2[32], r3[32];
  ptx::tmem_ld32(t.s_addr, r0);
  ptx::tmem_ld32(t.s_addr + 32, r1);
  if (t.wide) {
    ptx::tmem_ld32(t.s_addr + 64, r2);
    ptx::tmem_ld32(t.s_addr + 96, r3);
  }
  ptx::tmem_wait_ld_regs(r0);
  ptx::tmem_fence_regs(r1);
  ptx::tmem_fence_regs(r2);
  ptx::tmem_fence_regs(r3);
  prepare_chunk<kVisit>(r0, t.masked, q, sparse, t.k0, visit_row, words_per_row);
  prepare_chunk<kVisit>(r1, t.masked, q, sparse, t.k0 + 32, visit_row, words_per_row);
  float lm = fmaxf(chunk_max(r0), chunk_max(r1));
  if (t.wide) {
    prepare_chunk<kVisit>(r2, t.masked, q, sparse, t.k_up, visit_row, words_per_row);
    prepare_chunk<kVisit>(r3, t.masked, q, sparse, t.k_up + 32, visit_row, words_per_row);
    lm = fmaxf(lm, fmaxf(chunk_max(r2), chunk_max(r3)));
  }
  const float m_new = next_ref(st.m_ref, lm, sl2);
  const bool moved = m_new != st.m_ref;
  if (__any_sync(0xffffffffu, moved)) {
    float factor = 1.0f;
    if (moved) factor = st.m_ref == -INFINITY ? 0.0f : mufu_exp2((st.m_ref - m_new) * sl2);
    st.l_part *= factor;
    st.m_ref = m_new;
    if (!t.first) rescale_o(t.o_addr, factor);
  }
  const float neg_mb = m_new == -INFINITY ? 0.0f : -m_new * sl2;
  float sum0 = 0.0f, sum1 = 0.0f;
  const uint32_t p_addr = t.s_addr + 64;
  exp_chunk<kPolyMask>(r0, sl2, neg_mb, p_addr, sum0, sum1);
  exp_chunk<kPolyMask>(r1, sl2, neg_mb, p_addr + 16, sum0, sum1);
  ptx::tmem_wait_st();
  ptx::tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) ptx::mbar_arrive(t.half_bar);
  if (t.wide) {
    exp_chunk<kPolyMask>(r2, sl2, neg_mb, p_addr + 32, sum0, sum1);
    exp_chunk<kPolyMask>(r3, sl2, neg_mb, p_addr + 48, sum0, sum1);
  }
  st.l_part += sum0 + sum1;
  ptx::tmem_wait_st();
}

// Softmax warpgroup x (warps 4-7: x = 0, warps 8-11: x = 1) owns query tile
// x of every item: all its tiles, then the item's epilogue (normalise and
// store, or write a split partial and merge).
template <bool kVisit, bool kVarlen>
__device__ void softmax_role(const KernelArgs& a, const Smem& sh, uint32_t tmem,
                             const CUtensorMap* tout) {
  const tpsa_plan& p = a.plan;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t x = static_cast<uint32_t>(warp - kFirstSoftmaxWarp) / 4;
  const int quad = warp % 4;
  const int row = quad * 32 + lane;  // TMEM lane == row of query tile x
  const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
  const int32_t hq = p.kv_heads * kGroupSize;
  const bool visit = kVisit && a.visited != nullptr;
  const uint32_t s_addr = tmem + lane_base + (x << 7);
  const uint32_t o_addr = tmem + lane_base + kTmemO + (x << 7);
  const uint32_t bar_s = sh.bar(kBarSFull + x), bar_p = sh.bar(kBarPFull + x);
  const uint32_t bar_o = sh.bar(kBarOFull + x), bar_ph = sh.bar(kBarPHalf + x);
  // This warp's output staging (4 KB), stored by its own TMA stores (lane 0
  // issues them and waits for them to read the buffer before it is reused).
  const uint32_t wstage = kOffOut + (warp - kFirstSoftmaxWarp) * kOutStageBytes;
  uint8_t* stage = sh.base + wstage;
  auto stage_free = [&]() {
    if (lane == 0) ptx::bulk_wait_group_read<0>();
    __syncwarp();
  };
  volatile int* split_last = reinterpret_cast<volatile int*>(sh.base + kOffSplitLast) + 2 * x;
  const uint32_t cnt_w = 2 * x, cnt_d = 2 * x + 1;  // split partial written / merge decided
  uint32_t s_par = 0, o_par = 0, split_items = 0;
  uint32_t tr_sm = 0;  // trace counter (used only with TPSA_TRACE)
  (void)tr_sm;
#ifdef TPSA_TRACE
  const bool tr = row == 0 && blockIdx.x == TPSA_TRACE_CTA;
#else
  const bool tr = false;
#endif
#define tr_n_ tr_sm

  for (uint32_t n_item = 0;; ++n_item) {
    ItemRec rec;
    TPSA_ITEM_REC(n_item, 1, ptx::globaltimer_ns());
    const bool got = take_item(sh, n_item, &rec);
    if (!__all_sync(0xffffffffu, got)) break;
    TPSA_ITEM_REC(n_item, 2, ptx::globaltimer_ns());
    TPSA_ITEM_REC(n_item, 0, static_cast<unsigned long long>(rec.idx) |
                                 (static_cast<unsigned long long>(rec.it.num_splits) << 32));
    __syncwarp();
    // The previous record is released only now that this warp has finished
    // that item, so the scheduler claims an item when the one two before it
    // is done.
    if (lane == 0 && n_item > 0) release_item(sh, n_item - 1);
    if (rec.idx >= p.total_items) break;
    const tpsa_item& it = rec.it;
    const BlockTiles& bt = rec.bt;
    const ReqDesc& rq = a.reqs[kVarlen ? rec.req() : 0];
    const tpsa_plan& pr = kVarlen ? rq.plan : p;
    const int32_t q_row0 = kVarlen ? rq.q_row0 : 0;
    const int32_t ridx = kVarlen ? rec.idx - rq.item_base : rec.idx;
    const int32_t tok = bt.q_begin + row / 2;
    const int32_t q = tok < pr.seq_len ? tok : pr.seq_len - 1;
    const bool sparse = row_is_sparse(pr, tok);
    const int32_t qrow = it.block * kBlockQ + row / 2;  // row within the request's chunk
    const int32_t head = it.kv_head * kGroupSize + 2 * static_cast<int32_t>(x) + (row & 1);
    const bool real_row = qrow < pr.query_tokens;
    uint32_t* visit_row =
        (visit && real_row)
            ? a.visited + (static_cast<size_t>(qrow) * hq + head) * a.words_per_row
            : nullptr;
    RowState st{-INFINITY, 0.0f};
    bool ok = true;
    const int32_t ntiles = it.tile_end - it.tile_begin;
    for (int32_t n = 0; n < ntiles; ++n) {
      int32_t k0, w;
      tile_keys(bt, it.tile_begin + n, &k0, &w);
      TileArgs ta;
      ta.s_addr = s_addr;
      ta.o_addr = o_addr;
      ta.k0 = k0;
      ta.k_up = upper_key(bt, it.tile_begin + n, k0);
      // The 80-key composite tile runs as a 128-key one: S columns 80-127
      // hold no score of this tile, but they stand for keys 16-63, which no
      // row of a sparse block sees, so the mask replaces them by -inf (and
      // their P, zero, meets no PV).  Measured at 8K, this is faster than a
      // softmax branch for the 16-column sink slice (109.5 against 111.3 us).
      ta.wide = w > kKeyGrain;
      ta.masked = tile_needs_mask(pr, bt, k0, w);
      ta.first = n == 0;
      ta.half_bar = bar_ph;
      const bool w_ok = wait(sh, bar_s, s_par);
      s_par ^= 1;
      if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
      if (tr) TPSA_TR(2 + x, 1, n);
      ptx::tc_fence_after();
      softmax_tile<kVisit>(ta, p.scale_log2, q, sparse, st, visit_row, a.words_per_row);
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_p);
      if (tr) TPSA_TR(2 + x, 3, n);
    }
    if (!ok) break;

    // Item end: O_x is complete once the item's last PV of this tile is.
    const bool w_ok = wait(sh, bar_o, o_par);
    o_par ^= 1;
    if (!__all_sync(0xffffffffu, w_ok)) break;
    ptx::tc_fence_after();
    TPSA_ITEM_REC(n_item, 3, ptx::globaltimer_ns());
    if (tr) TPSA_TR(2 + x, 5, rec.idx);
    const bool split = it.num_splits > 1;
    const bool staged_store = !split && (!kVarlen || bt.q_end - bt.q_begin == kBlockQ);
    const uint32_t sp_slot = split_items & 1;
    split_items += split ? 1u : 0u;
    // Output rows of this warp: packed token base_q + R / 2, head
    // base_h + R % 2 for warp row R (the tensor map clips rows past the end).
    const int32_t base_q = q_row0 + it.block * kBlockQ + quad * 16;
    const int32_t base_h = it.kv_head * kGroupSize + 2 * static_cast<int32_t>(x);
    if (staged_store) {
      // Two rounds of 64 columns: the warp's 32 rows into its staging
      // buffer as bf16 (128-byte swizzled rows, the layout the tensor map
      // stores), then one TMA store of the 16-token x 2-head x 64-column box.
      // (A batch-one launch's tensor map ends at the last query row, which
      // clips the last block.)
      const float inv = 1.0f / st.l_part;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t v0[32], v1[32];
        ptx::tmem_ld32(o_addr + 64 * h, v0);
        ptx::tmem_ld32(o_addr + 64 * h + 32, v1);
        stage_free();
        ptx::tmem_wait_ld_regs(v0);
        ptx::tmem_fence_regs(v1);
        uint8_t* srow = stage + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t* v = j < 4 ? &v0[8 * j] : &v1[8 * (j - 4)];
          *reinterpret_cast<uint4*>(srow + ((j ^ (lane & 7)) << 4)) = make_uint4(
              pack_bf16x2(__uint_as_float(v[0]) * inv, __uint_as_float(v[1]) * inv),
              pack_bf16x2(__uint_as_float(v[2]) * inv, __uint_as_float(v[3]) * inv),
              pack_bf16x2(__uint_as_float(v[4]) * inv, __uint_as_float(v[5]) * inv),
              pack_bf16x2(__uint_as_float(v[6]) * inv, __uint_as_float(v[7]) * inv));
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          ptx::tma_store_3d(tout, 64 * h, base_h, base_q, sh.base_u32 + wstage);
          ptx::bulk_commit_group();
        }
      }
      if (tr) TPSA_TR(2 + x, 6, 0);
      continue;
    }
    if (!split) {
      // A block that ends inside its 64-token box (a request's last block in
      // a packed batch): a box store would also write rows of the next
      // request, so each thread writes its own row: 256 contiguous bytes of
      // `out`, in two halves of 64 columns.
      const float inv = 1.0f / st.l_part;
      uint4* dst = reinterpret_cast<uint4*>(
          a.out + (static_cast<size_t>(q_row0 + qrow) * hq + head) * kHeadDim);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t v0[32], v1[32];
        ptx::tmem_ld32(o_addr + 64 * h, v0);
        ptx::tmem_ld32(o_addr + 64 * h + 32, v1);
        ptx::tmem_wait_ld_regs(v0);
        ptx::tmem_fence_regs(v1);
        if (real_row) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            dst[8 * h + j] = make_uint4(
                pack_bf16x2(__uint_as_float(v0[8 * j]) * inv, __uint_as_float(v0[8 * j + 1]) * inv),
                pack_bf16x2(__uint_as_float(v0[8 * j + 2]) * inv, __uint_as_float(v0[8 * j + 3]) * inv),
                pack_bf16x2(__uint_as_float(v0[8 * j + 4]) * inv, __uint_as_float(v0[8 * j + 5]) * inv),
                pack_bf16x2(__uint_as_float(v0[8 * j + 6]) * inv, __uint_as_float(v0[8 * j + 7]) * inv));
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            dst[8 * h + 4 + j] = make_uint4(
                pack_bf16x2(__uint_as_float(v1[8 * j]) * inv, __uint_as_float(v1[8 * j + 1]) * inv),
                pack_bf16x2(__uint_as_float(v1[8 * j + 2]) * inv, __uint_as_float(v1[8 * j + 3]) * inv),
                pack_bf16x2(__uint_as_float(v1[8 * j + 4]) * inv, __uint_as_float(v1[8 * j + 5]) * inv),
                pack_bf16x2(__uint_as_float(v1[8 * j + 6]) * inv, __uint_as_float(v1[8 * j + 7]) * inv));
          }
        }
      }
      if (tr) TPSA_TR(2 + x, 6, 0);
      continue;
    }

    // Split item: the fp32 partial (128 columns) into the item's column-major
    // slot ([128 columns][256 rows], then m[256] and l[256]; this tile's rows
    // are 128 x + row).  Every piece of the block then merges a slice of the
    // tile's rows: once all pieces have published their partials (a global
    // counter per block, kv head and query tile reaches 4 warps x pieces),
    // piece s merges rows [s r, (s + 1) r), r = ceil(128 / pieces), reading
    // every piece's values of those rows only, so the merge and its L2
    // traffic are spread over the pieces' CTAs.  The scheduler claims
    // nothing while its CTA holds a split piece: a waiting piece's partners
    // are running on other CTAs or not yet claimed, and the CTAs that hold
    // no piece of a block with unclaimed pieces keep claiming.
    float* slot =
        a.scratch + static_cast<size_t>((kVarlen ? rq.slot_base : 0) + ridx) * kSlotFloats;
    constexpr int32_t kSlotRows = 2 * kRowsPerTile;
    const int32_t srow = static_cast<int32_t>(x) * kRowsPerTile + row;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t v[32];
      ptx::tmem_ld32(o_addr + 32 * c, v);
      ptx::tmem_wait_ld_regs(v);
      float* col = slot + static_cast<size_t>(32 * c) * kSlotRows + srow;
#pragma unroll
      for (int j = 0; j < 32; ++j) col[j * kSlotRows] = __uint_as_float(v[j]);
    }
    slot[kHeadDim * kSlotRows + srow] = st.m_ref;
    slot[(kHeadDim + 1) * kSlotRows + srow] = st.l_part;
    __threadfence();
    __syncwarp();
    TPSA_ITEM_REC(n_item, 4, ptx::globaltimer_ns());
    const int32_t ns = it.num_splits;
    int32_t* ctr = a.ctl + kCtlSplitBase + (kVarlen ? rq.ctr_base : 0) +
                   ((it.block - pr.tail_block0) * p.kv_heads + it.kv_head) * 2 +
                   static_cast<int32_t>(x);
    int32_t slice = 0, rows_per = kRowsPerTile;
    if (a.coop_merge) {
      bool all_in = true;
      if (lane == 0) {
        ptx::red_release_add_global(ctr, 1);
        all_in = wait_global_count(sh, ctr, 4 * ns);
      }
      if (!__all_sync(0xffffffffu, __shfl_sync(0xffffffffu, all_in, 0))) break;
      __syncwarp();  // lane 0's acquire orders the other lanes' loads too
      slice = it.split;
      rows_per = (kRowsPerTile + ns - 1) / ns;
      TPSA_ITEM_REC(n_item, 5, ptx::globaltimer_ns());
    } else {
      // The last piece to finish merges all rows of the tile.
      if (lane == 0) ptx::red_release_add_shared(sh.counter(cnt_w), 1);
      if (row == 0) {
        if (wait_count(sh, cnt_w, 4 * split_items)) {
          const int prev = atomicAdd(ctr, 1);
          split_last[sp_slot] = prev == ns - 1;
          ptx::red_release_add_shared(sh.counter(cnt_d), 1);
        }
      }
      const bool decided = __all_sync(0xffffffffu, wait_count(sh, cnt_d, split_items));
      if (!decided) break;
      if (!split_last[sp_slot]) continue;
      __threadfence();
    }

    // This thread's share of the merge: row slot `t % cw` of the slice and
    // columns [cw (t / cw), cw (t / cw + 1)), cw = the slice's rows rounded up
    // to a power of two (cw row slots x 128 / cw column groups = 128 threads;
    // the whole tile is one slice of 128 rows, one thread per row).  The
    // partials come from L2 (other CTAs just wrote them): the pieces' m and
    // l 8 at a time in one online pass, then 32 values per round, min(cw, 16)
    // columns of 32 / min(cw, 16) pieces, so a narrow slice over many pieces
    // (a one-head launch: 43 pieces of 3 rows at 32K) takes few rounds of L2
    // latency.  (A full-width slice keeps 2 pieces x 16 columns per round: a
    // merge out of line, or with more loads per round, measured 2 to 4 %
    // slower at 8 kv heads.)
    int32_t cw = 1;
    while (cw < rows_per) cw <<= 1;
    const int32_t t = row;
    const int32_t mr = slice * rows_per + (t & (cw - 1));  // row of tile x
    const int32_t mc0 = (t / cw) * cw;                        // first column
    const int32_t mqrow = it.block * kBlockQ + mr / 2;
    if ((t & (cw - 1)) < rows_per && mr < kRowsPerTile && mqrow < pr.query_tokens) {
      const int32_t msrow = static_cast<int32_t>(x) * kRowsPerTile + mr;
      const float* first_slot = slot - static_cast<size_t>(it.split) * kSlotFloats;
      const size_t m_off = static_cast<size_t>(kHeadDim) * kSlotRows + msrow;
      const size_t l_off = static_cast<size_t>(kHeadDim + 1) * kSlotRows + msrow;
      float inv_sum;
      const float mmax = merge_row_stats(first_slot, m_off, l_off, ns, p.scale_log2, &inv_sum);
      const int32_t mhead = it.kv_head * kGroupSize + 2 * static_cast<int32_t>(x) + (mr & 1);
      uint32_t* orow = reinterpret_cast<uint32_t*>(
          a.out + (static_cast<size_t>(q_row0 + mqrow) * hq + mhead) * kHeadDim + mc0);
      const size_t col_off = static_cast<size_t>(mc0) * kSlotRows + msrow;
      if (cw >= 16) {
        merge_columns<16>(first_slot, m_off, col_off, ns, cw, mmax, p.scale_log2, inv_sum, orow);
      } else if (cw == 8) {
        merge_columns<8>(first_slot, m_off, col_off, ns, cw, mmax, p.scale_log2, inv_sum, orow);
      } else if (cw == 4) {
        merge_columns<4>(first_slot, m_off, col_off, ns, cw, mmax, p.scale_log2, inv_sum, orow);
      } else {
        merge_columns<2>(first_slot, m_off, col_off, ns, cw, mmax, p.scale_log2, inv_sum, orow);
      }
    }
    __syncwarp();
    TPSA_ITEM_REC(n_item, 6, ptx::globaltimer_ns());
    if (a.coop_merge && lane == 0) ptx::mbar_arrive(sh.bar(kBarPieceDone));
  }
  // Output stores of this warp complete before the CTA exits.
  if (lane == 0) ptx::bulk_wait_group<0>();
}
#undef tr_n_


template <bool kVisit, bool kVarlen>
__global__ void __launch_bounds__(kNumThreads, 1)
    tpsa_paged_kernel(const __grid_constant__ KernelArgs args,
                     const __grid_constant__ CUtensorMap tmap_q,
                     const __grid_constant__ CUtensorMap tmap_k128,
                     const __grid_constant__ CUtensorMap tmap_k64,
                     const __grid_constant__ CUtensorMap tmap_k16,
                     const __grid_constant__ CUtensorMap tmap_v,
                     const __grid_constant__ CUtensorMap tmap_v128,
                     const __grid_constant__ CUtensorMap tmap_v16,
                     const __grid_constant__ CUtensorMap tmap_out) {
  extern __shared__ uint8_t smem_raw[];
  Smem sh;
  {
    const uint32_t raw = ptx::smem_u32(smem_raw);
    const uint32_t aligned = (raw + 1023u) & ~1023u;
    sh.base = smem_raw + (aligned - raw);
    sh.base_u32 = aligned;
  }
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
#ifdef TPSA_TRACE
    if (blockIdx.x < 1024) g_cta_span[blockIdx.x][0] = ptx::globaltimer_ns();
#endif
    for (uint32_t x = 0; x < 2; ++x) {
      ptx::mbar_init(sh.bar(kBarQFull + x), 1);
      ptx::mbar_init(sh.bar(kBarQEmpty + x), 1);
      ptx::mbar_init(sh.bar(kBarSFull + x), 1);
      ptx::mbar_init(sh.bar(kBarPFull + x), 4);
      ptx::mbar_init(sh.bar(kBarPHalf + x), 4);
      ptx::mbar_init(sh.bar(kBarOFull + x), 1);
      ptx::mbar_init(sh.bar(kBarItemFull + x), 1);
      ptx::mbar_init(sh.bar(kBarItemEmpty + x), kItemConsumers);
    }
    for (int s = 0; s < kKRing; ++s) {
      ptx::mbar_init(sh.bar(kBarKFull + s), 1);
      ptx::mbar_init(sh.bar(kBarKEmpty + s), 1);
    }
    for (int s = 0; s < kVRing; ++s) {
      ptx::mbar_init(sh.bar(kBarVFull + s), 1);
      ptx::mbar_init(sh.bar(kBarVEmpty + s), 1);
    }
    ptx::mbar_init(sh.bar(kBarTail), 1);
    ptx::mbar_init(sh.bar(kBarDrain), 1);
    ptx::mbar_init(sh.bar(kBarProbe), 1);
    ptx::mbar_init(sh.bar(kBarPieceDone), kSoftmaxWarps);
    *sh.abort_flag() = 0;
    for (uint32_t i = 0; i < 4; ++i) {
      *reinterpret_cast<volatile uint32_t*>(sh.base + kOffCounters + 4 * i) = 0;
    }
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(sh.base_u32 + kOffTmemSlot, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sh.base + kOffTmemSlot);

  if (warp < kFirstSoftmaxWarp) {
    ptx::setmaxnreg_dec<kControlRegs>();
    if (warp == 0) {
      if (lane == 0) {
        producer_role<kVarlen>(args, sh, &tmap_q, &tmap_k128, &tmap_k64, &tmap_k16, &tmap_v,
                               &tmap_v128, &tmap_v16, false);
      }
      __syncwarp();
    } else if (warp == 1) {
      mma_role(args, sh, tmem);
    } else if (warp == 2) {
      if (lane == 0) scheduler_role<kVarlen>(args, sh);
      __syncwarp();
    } else {
      if (lane == 0) {
        producer_role<kVarlen>(args, sh, &tmap_q, &tmap_k128, &tmap_k64, &tmap_k16, &tmap_v,
                               &tmap_v128, &tmap_v16, true);
      }
      __syncwarp();
    }
  } else {
    ptx::setmaxnreg_inc<kSoftmaxRegs>();
    softmax_role<kVisit, kVarlen>(args, sh, tmem, &tmap_out);
  }

  ptx::tc_fence_before();
  __syncthreads();  // MMAs drained, every role done
#ifdef TPSA_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_cta_span[blockIdx.x][1] = ptx::globaltimer_ns();
#endif
  if (args.ctl_reset_words > 0) {
    // Control words of a library-owned block: the last CTA to finish zeroes
    // them for the next launch on the stream.  Every other CTA has made its
    // last claim and its last split-counter update before counting itself
    // out (the fence orders them before the count).
    volatile int* last = reinterpret_cast<volatile int*>(sh.base + kOffLastCta);
    if (threadIdx.x == 0) {
      __threadfence();
      const int done = atomicAdd(args.ctl + kCtlExited, 1);
      *last = done == static_cast<int>(gridDim.x) - 1 ? 1 : 0;
      __threadfence();
    }
    __syncthreads();
    if (*last) {
      __threadfence();
      for (int32_t i = threadIdx.x; i < args.ctl_reset_words; i += kNumThreads) args.ctl[i] = 0;
    }
  }
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}


// ================================================================ host side
thread_local std::string t_last_error;
// Test hook armed by tpsa_debug_wait_probe: the limit of the probe wait of
// the next launch on this thread (0 = none).
thread_local uint32_t t_probe_wait_ns = 0;

tpsa_status fail(tpsa_status s, const std::string& msg) {
  t_last_error = "[TPSA] " + msg;
  return s;
}

// Dense-tail blocks longer than this fraction of the average work per CTA
// are split into several items (merged in-kernel).
#ifndef TPSA_SPLIT_FACTOR
#define TPSA_SPLIT_FACTOR 0.7
#endif
constexpr double kSplitFactor = TPSA_SPLIT_FACTOR;

// Split threshold (tiles per item) for the dense-tail blocks of a plan.  The
// B = tail blocks x kv heads longest items, each cut into ns pieces of
// ceil(T / ns) tiles, go first to the P CTAs (longest first), so the
// busiest CTA carries ceil(B ns / P) pieces; the short items fill the other
// CTAs.  The estimated makespan, in tiles, is
//   max(ceil(B ns / P) (ceil(T / ns) + c), (total + B ns c) / P)
// with c the per-piece cost of a partial write and its share of the merge
// (kSplitPieceTiles); the smallest ns with the least estimate wins.  ns is
// at most what a threshold of kSplitFactor times the average work per CTA
// gives, so no plan needs more split slots than that rule (the static-scratch
// entry point's limit rests on it).
constexpr double kSplitPieceTiles = 2.0;
// `longest`: tiles of the longest dense-tail block; `tail`: dense-tail
// (block, head) items before splitting; `tiles`: all tiles of the launch.
int32_t choose_split_counts(int32_t longest, int64_t tail, int64_t tiles, int32_t ctas) {
  if (tail == 0 || longest == 0) return 1 << 30;
  const int32_t by_fraction = max_i(kMinSplitTiles, static_cast<int32_t>(
      kSplitFactor * static_cast<double>(tiles) / ctas));
  const int32_t ns_max = min_i(64, ceil_div(longest, by_fraction));
  double best = 0.0;
  int32_t best_ns = 1;
  for (int32_t ns = 1; ns <= ns_max; ++ns) {
    const double piece = static_cast<double>(ceil_div(longest, ns)) + kSplitPieceTiles;
    const double rounds = static_cast<double>((tail * ns + ctas - 1) / ctas);
    const double avg = (static_cast<double>(tiles) + kSplitPieceTiles * tail * ns) / ctas;
    const double est = std::max(rounds * piece, avg);
    if (ns == 1 || est < best - 1e-9) {
      best = est;
      best_ns = ns;
    }
  }
  return best_ns == 1 ? (1 << 30) : ceil_div(longest, best_ns);
}

// Merge mode of a launch's split pieces.  With few items per CTA (a head
// slice of a multi-GPU partition, short prompts) the pieces run side by side
// and the last one's merge of every partial is the launch's tail, so all
// pieces of a block merge together, each a slice of the rows.  With many
// items per CTA the last piece merges alone: the others leave at once and
// their CTAs take the next item.  Measured at 8K and 32K/q8K (8 to 1 kv
// heads): the cooperative merge loses about 6 % at 7 items per CTA and gains
// 2 to 40 % at 3.6 or fewer.
constexpr int64_t kCoopItemsPerCta = 4;
bool coop_merge(int64_t items, int32_t grid) {
  return items <= kCoopItemsPerCta * static_cast<int64_t>(grid);
}

int32_t choose_split(const tpsa_plan& p, int32_t b0, int64_t tiles, int32_t ctas) {
  int32_t longest = 0;
  for (int32_t b = b0; b < p.num_blocks; ++b) longest = max_i(longest, block_tiles(p, b).count);
  return choose_split_counts(longest, static_cast<int64_t>(p.num_blocks - b0) * p.kv_heads, tiles,
                             ctas);
}

tpsa_status cuda_fail(cudaError_t e, const char* what) {
  return fail(TPSA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  int major = 0;
  bool attr_set = false;
  int max_ctas = 0;  // co-resident CTAs of the kernel (one per SM)
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
    e = cudaFuncSetAttribute(tpsa_paged_kernel<false, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    e = cudaFuncSetAttribute(tpsa_paged_kernel<true, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    e = cudaFuncSetAttribute(tpsa_paged_kernel<false, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tpsa_paged_kernel<false, false>,
                                                      kNumThreads, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (per_sm <= 0) return fail(TPSA_ERR_CUDA, "the kernel does not fit on an SM");
    st.max_ctas = per_sm * st.sm_count;
    st.attr_set = true;
  }
  *out = &st;
  return TPSA_OK;
}

// ------------------------------------------------ stream control blocks
// The control words of a launch (scheduler counter, exit counter, split
// counters) start at zero.  Instead of clearing them with a memset before
// every kernel (a separate operation of a few microseconds on the stream),
// each stream that calls the library gets a control block of its own in a
// module-global array; the block is cleared once when the stream first gets
// it, and the last CTA of every launch zeroes it again before exiting.
// Launches on one stream run one after another, so they never share a block
// at the same time.  Streams are told apart by cudaStreamGetId, which is
// unique for the life of the context (a destroyed stream's handle may be
// reused, its id is not).  A launch falls back to control words in the
// caller's workspace, cleared by cudaMemsetAsync, when the stream is being
// captured into a CUDA graph (a graph may be replayed on any stream), when
// all blocks are taken, or when the launch needs more words than a block
// holds.
constexpr int kCtlBlocks = 128;
constexpr int32_t kCtlBlockWords = 1024;  // 4 KiB; a 16-request launch needs at most 832
struct CtlBlocks {
  int32_t* base = nullptr;  // device address of g_ctl_blocks on this device
  unsigned long long stream_id[kCtlBlocks] = {};
  int used = 0;
};
CtlBlocks g_ctl[64];  // per device ordinal, guarded by g_mutex

}  // namespace

static __device__ __align__(256) int32_t g_ctl_blocks[kCtlBlocks * kCtlBlockWords];

namespace {

// The control block of `stream` for a launch of `words` control words, or
// nullptr in *ctl when the launch must use its workspace instead.  The first
// launch of a stream clears its block on that stream.
tpsa_status stream_ctl_block(cudaStream_t stream, int64_t words, int32_t** ctl) {
  *ctl = nullptr;
  if (words > kCtlBlockWords) return TPSA_OK;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(stream, &capture);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  if (capture != cudaStreamCaptureStatusNone) return TPSA_OK;
  unsigned long long id = 0;
  e = cudaStreamGetId(stream, &id);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamGetId");
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(TPSA_ERR_CUDA, "device ordinal out of range");
  // The array's address is looked up on every call (cheap once the module
  // is loaded): after a device reset the module loads again in a new
  // context, possibly at another address, and its blocks start from zero,
  // so a changed address starts the device's table afresh.
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_ctl_blocks);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(control blocks)");
  std::lock_guard<std::mutex> lock(g_mutex);
  CtlBlocks& cb = g_ctl[dev];
  if (cb.base != static_cast<int32_t*>(p)) {
    cb.base = static_cast<int32_t*>(p);
    cb.used = 0;
  }
  for (int i = 0; i < cb.used; ++i) {
    if (cb.stream_id[i] == id) {
      *ctl = cb.base + static_cast<size_t>(i) * kCtlBlockWords;
      return TPSA_OK;
    }
  }
  if (cb.used == kCtlBlocks) return TPSA_OK;
  int32_t* block = cb.base + static_cast<size_t>(cb.used) * kCtlBlockWords;
  e = cudaMemsetAsync(block, 0, kCtlBlockWords * sizeof(int32_t), stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(control block)");
  cb.stream_id[cb.used++] = id;
  *ctl = block;
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

// The cache's tensor maps: K boxes of 128, 64 and 16 rows, V boxes of 64,
// 128 and 16 rows (one KV head, 64 columns each).
struct KvMaps {
  CUtensorMap k128, k64, k16, v, v128, v16;
};

tpsa_status encode_kv_maps(const void* key_cache, const void* value_cache, uint64_t kv_heads,
                           uint64_t cache_tokens, KvMaps* m) {
  const struct {
    CUtensorMap* map;
    const void* base;
    uint32_t rows;
  } maps[6] = {{&m->k128, key_cache, 128},  {&m->k64, key_cache, 64},
               {&m->k16, key_cache, static_cast<uint32_t>(kSinkSlice)},
               {&m->v, value_cache, 64},    {&m->v128, value_cache, 128},
               {&m->v16, value_cache, static_cast<uint32_t>(kSinkSlice)}};
  for (const auto& e : maps) {
    const tpsa_status st = encode_map(e.map, e.base, kv_heads, cache_tokens, 1, e.rows);
    if (st != TPSA_OK) return st;
  }
  return TPSA_OK;
}

// `ctas`: co-resident CTAs the launch runs; each runs one item at a time.
// `split_override` > 0 replaces the split threshold derived from this
// request's own work (a varlen launch derives it from the whole launch).
tpsa_status build_plan(int64_t query_tokens, int64_t query_start, int64_t seq_len,
                       int64_t prompt_len, int32_t kv_heads, int32_t ctas,
                       float scale, tpsa_plan* p, int32_t split_override = 0,
                       bool dense = false) {
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
  if (ctas <= 0) return fail(TPSA_ERR_INVALID_ARGUMENT, "sm_count must be positive");
  std::memset(p, 0, sizeof(*p));
  p->query_tokens = static_cast<int32_t>(query_tokens);
  p->query_start = static_cast<int32_t>(query_start);
  p->seq_len = static_cast<int32_t>(seq_len);
  p->sparse_begin = kSparseBegin;
  const int64_t se = prompt_len - kDenseTail > 0 ? prompt_len - kDenseTail : 0;
  p->sparse_end = static_cast<int32_t>(se < seq_len ? se : seq_len);
  // All-dense control: no sparse rows, every row reads [0, q].  Every block
  // then counts as a dense-tail block (longest first, split when the
  // counters allow).
  if (dense) p->sparse_end = 0;
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
  int32_t split = split_override > 0 ? split_override : choose_split(*p, b0, tiles, ctas);
  if (split < kMinSplitTiles) split = kMinSplitTiles;
  // At most 64 pieces per block, and fewer than the CTAs: the pieces of a
  // block wait for one another before merging, which needs them to run at
  // once.
  const int32_t max_pieces = min_i(64, ctas);
  for (int32_t b = b0; b < p->num_blocks; ++b) {
    const int32_t c = block_tiles(*p, b).count;
    if (ceil_div(c, split) > max_pieces) split = ceil_div(c, max_pieces);
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
  p->grid = p->total_items < ctas ? p->total_items : ctas;
  p->total_tiles = tiles;
  p->workspace_bytes = kControlBytes + (any_split ? tail_items * kSlotBytes : 0);
  return TPSA_OK;
}

tpsa_status launch(const void* query, const void* key_cache, const void* value_cache,
                   const int32_t* block_table, void* out, int64_t query_tokens,
                   int64_t num_pages, int64_t table_cols, int64_t query_start,
                   int64_t seq_len, int64_t prompt_len, float scale, int32_t kv_heads,
                   void* workspace, uint64_t workspace_bytes, uint32_t* visited,
                   uint64_t* tile_counter, void* stream, bool dense = false,
                   bool ctl_in_workspace = false) {
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
  st = build_plan(query_tokens, query_start, seq_len, prompt_len, kv_heads, dev->max_ctas,
                  scale, &args.plan, 0, dense);
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
  CUtensorMap tq, tout;
  KvMaps kv;
  const uint64_t hq = static_cast<uint64_t>(kv_heads) * kGroupSize;
  const uint64_t cache_tokens = static_cast<uint64_t>(num_pages) * kPageSize;
  st = encode_map(&tq, query, hq, static_cast<uint64_t>(query_tokens), 2, kBlockQ);
  if (st != TPSA_OK) return st;
  st = encode_kv_maps(key_cache, value_cache, kv_heads, cache_tokens, &kv);
  if (st != TPSA_OK) return st;
  // Output boxes of one softmax warp: 16 tokens x 2 heads x 64 columns.  The
  // map's extent ends at the last query row, which clips the last block.
  st = encode_map(&tout, out, hq, static_cast<uint64_t>(query_tokens), 2, 16);
  if (st != TPSA_OK) return st;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  args.num_reqs = 1;
  args.reqs[0].plan = p;  // one request: item, row, table, slot and counter bases 0
  args.block_table = block_table;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.num_pages = static_cast<int32_t>(num_pages);
  args.scratch = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kControlBytes);
  // The work-item counter and split counters start at zero every launch: in
  // the stream's control block (left at zero by the previous launch), else
  // in the workspace, cleared here.
  args.ctl = nullptr;
  if (!ctl_in_workspace) {
    st = stream_ctl_block(s, kControlBytes / 4, &args.ctl);
    if (st != TPSA_OK) return st;
  }
  cudaError_t e = cudaSuccess;
  if (args.ctl != nullptr) {
    args.ctl_reset_words = kControlBytes / 4;
  } else {
    args.ctl = static_cast<int32_t*>(workspace);
    e = cudaMemsetAsync(workspace, 0, kControlBytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
  }
  args.visited = visited;
  args.tiles = reinterpret_cast<unsigned long long*>(tile_counter);
  args.words_per_row = (p.seq_len + 31) / 32;
  args.probe_wait_ns = t_probe_wait_ns;
  args.coop_merge = coop_merge(p.total_items, p.grid) ? 1 : 0;
  t_probe_wait_ns = 0;

  if (visited != nullptr || tile_counter != nullptr) {
    tpsa_paged_kernel<true, false><<<p.grid, kNumThreads, kSmemBytes, s>>>(
        args, tq, kv.k128, kv.k64, kv.k16, kv.v, kv.v128, kv.v16, tout);
  } else {
    tpsa_paged_kernel<false, false><<<p.grid, kNumThreads, kSmemBytes, s>>>(
        args, tq, kv.k128, kv.k64, kv.k16, kv.v, kv.v128, kv.v16, tout);
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
                        int32_t ctas, float scale, int64_t table_cols, BatchLaunch* b) {
  std::memset(&b->args, 0, sizeof(b->args));
  KernelArgs& a = b->args;
  int64_t tiles = 0, tail_items = 0;
  int32_t longest = 0;
  for (int32_t i = 0; i < count; ++i) {
    const int32_t r = first + i;
    const int64_t tq = cu_seqlens_q[r + 1] - cu_seqlens_q[r];
    tpsa_plan probe;
    tpsa_status st = build_plan(tq, seq_lens[r] - tq, seq_lens[r], prompt_lens[r], kv_heads,
                                ctas, scale, &probe, 1 << 30);
    if (st != TPSA_OK) return st;
    tiles += probe.total_tiles;
    tail_items += static_cast<int64_t>(probe.num_blocks - probe.tail_block0) * kv_heads;
    for (int32_t b = probe.tail_block0; b < probe.num_blocks; ++b) {
      longest = max_i(longest, block_tiles(probe, b).count);
    }
  }
  // One split threshold for the launch, from the makespan estimate over all
  // requests' dense-tail items (which are dispatched first).
  int32_t split = choose_split_counts(longest, tail_items, tiles, ctas);
  if (split < kMinSplitTiles) split = kMinSplitTiles;
  int32_t items = 0, slots = 0, counters = 0, tail = 0, rest = 0;
  for (int32_t i = 0; i < count; ++i) {
    const int32_t r = first + i;
    const int64_t tq = cu_seqlens_q[r + 1] - cu_seqlens_q[r];
    ReqDesc& d = a.reqs[i];
    tpsa_status st = build_plan(tq, seq_lens[r] - tq, seq_lens[r], prompt_lens[r], kv_heads,
                                ctas, scale, &d.plan, split);
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
  a.plan.grid = items < ctas ? items : ctas;
  a.coop_merge = coop_merge(items, a.plan.grid) ? 1 : 0;
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
                             const int64_t* prompt_lens, int32_t kv_heads, int32_t ctas,
                             uint64_t* bytes) {
  tpsa_status st = check_batch(batch, cu_seqlens_q, seq_lens, prompt_lens);
  if (st != TPSA_OK) return st;
  std::unique_ptr<BatchLaunch> b(new BatchLaunch);
  int64_t most = kControlBytes;
  for (int32_t first = 0; first < batch; first += kMaxReqs) {
    const int32_t count = std::min(kMaxReqs, batch - first);
    st = build_batch(first, count, cu_seqlens_q, seq_lens, prompt_lens, kv_heads, ctas,
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
  CUtensorMap tq, tout;
  KvMaps kv;
  const uint64_t hq = static_cast<uint64_t>(kv_heads) * kGroupSize;
  const uint64_t cache_tokens = static_cast<uint64_t>(num_pages) * kPageSize;
  st = encode_map(&tq, query, hq, total_rows, 2, kBlockQ);
  if (st != TPSA_OK) return st;
  st = encode_kv_maps(key_cache, value_cache, kv_heads, cache_tokens, &kv);
  if (st != TPSA_OK) return st;
  st = encode_map(&tout, out, hq, total_rows, 2, 16);
  if (st != TPSA_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::unique_ptr<BatchLaunch> b(new BatchLaunch);
  // Launches of at most kMaxReqs requests each, in stream order; each
  // reuses the workspace after the previous one.
  for (int32_t first = 0; first < batch; first += kMaxReqs) {
    const int32_t count = std::min(kMaxReqs, batch - first);
    st = build_batch(first, count, cu_seqlens_q, seq_lens, prompt_lens, kv_heads,
                     dev->max_ctas, scale, table_cols, b.get());
    if (st != TPSA_OK) return st;
    if (workspace_bytes < static_cast<uint64_t>(b->workspace_bytes)) {
      return fail(TPSA_ERR_WORKSPACE, "workspace smaller than tpsa_varlen_workspace_size()");
    }
    KernelArgs& args = b->args;
    args.block_table = block_tables;
    args.out = static_cast<__nv_bfloat16*>(out);
    args.num_pages = static_cast<int32_t>(num_pages);
    args.scratch = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + b->ctl_bytes);
    st = stream_ctl_block(s, b->ctl_bytes / 4, &args.ctl);
    if (st != TPSA_OK) return st;
    cudaError_t e = cudaSuccess;
    if (args.ctl != nullptr) {
      args.ctl_reset_words = static_cast<int32_t>(b->ctl_bytes / 4);
    } else {
      args.ctl = static_cast<int32_t*>(workspace);
      e = cudaMemsetAsync(workspace, 0, static_cast<size_t>(b->ctl_bytes), s);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
    }
    tpsa_paged_kernel<false, true><<<args.plan.grid, kNumThreads, kSmemBytes, s>>>(
        args, tq, kv.k128, kv.k64, kv.k16, kv.v, kv.v128, kv.v16, tout);
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

// Device address of the static scratch on the current device, looked up on
// every call (cudaGetSymbolAddress; the first call on a device also makes
// the runtime load this module's device globals there), so that it stays
// right after a device reset, which loads the module again.
tpsa_status static_scratch_address(void** ptr);

}  // namespace

static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

namespace {

tpsa_status static_scratch_address(void** ptr) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
  if (p == nullptr) return fail(TPSA_ERR_CUDA, "static scratch has no device address");
  *ptr = p;
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
  int32_t ctas = sm_count;  // one CTA per SM
  if (sm_count <= 0) {
    DeviceState* dev = nullptr;
    tpsa_status st = device_state(&dev);
    if (st != TPSA_OK) return st;
    ctas = dev->max_ctas;
  }
  return build_plan(query_tokens, query_start, seq_len, prompt_len, kv_heads, ctas, scale,
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
                           int32_t* key_begin, int32_t* key_count, int32_t* upper_begin,
                           int32_t* needs_mask) {
  if (plan == nullptr || key_begin == nullptr || key_count == nullptr ||
      upper_begin == nullptr || needs_mask == nullptr || block < 0 ||
      block >= plan->num_blocks) {
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
  *upper_begin = upper_key(bt, tile, k0);
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

tpsa_status tpsa_dense_workspace_size(int64_t query_tokens, int64_t query_start,
                                      int64_t seq_len, uint64_t* bytes) {
  t_last_error.clear();
  if (bytes == nullptr) return fail(TPSA_ERR_INVALID_ARGUMENT, "bytes pointer is NULL");
  DeviceState* dev = nullptr;
  tpsa_status st = device_state(&dev);
  if (st != TPSA_OK) return st;
  tpsa_plan p;
  st = build_plan(query_tokens, query_start, seq_len, seq_len, TPSA_KV_HEADS, dev->max_ctas,
                  1.0f, &p, 0, true);
  if (st != TPSA_OK) return st;
  *bytes = static_cast<uint64_t>(p.workspace_bytes);
  return TPSA_OK;
}

tpsa_status tpsa_paged_attention_dense(const void* query, const void* key_cache,
                                       const void* value_cache, const int32_t* block_table,
                                       void* out, int64_t query_tokens, int64_t num_pages,
                                       int64_t table_cols, int64_t query_start,
                                       int64_t seq_len, float scale, void* workspace,
                                       uint64_t workspace_bytes, void* stream) {
  return launch(query, key_cache, value_cache, block_table, out, query_tokens, num_pages,
                table_cols, query_start, seq_len, seq_len, scale, TPSA_KV_HEADS, workspace,
                workspace_bytes, nullptr, nullptr, stream, true);
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
                          dev->max_ctas, bytes);
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
                          dev->max_ctas, bytes);
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
  st = build_plan(query_tokens, query_start, seq_len, prompt_len, TPSA_KV_HEADS, dev->max_ctas,
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
                kStaticScratchBytes, nullptr, nullptr, stream, false, true);
}

#ifdef TPSA_TRACE
// Copies {start ns, end ns, items} of the first `ctas` CTAs of the last launch.
TPSA_API void tpsa_debug_spans(unsigned long long* out, uint32_t ctas) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(out, g_cta_span, sizeof(unsigned long long) * 3 * (ctas < 1024 ? ctas : 1024));
}

TPSA_API void tpsa_debug_items(unsigned long long* out, uint32_t ctas) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(out, g_item_trace,
                       sizeof(unsigned long long) * 128 * (ctas < 1024 ? ctas : 1024));
}

TPSA_API void tpsa_debug_timeout(uint32_t* out5) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(out5, g_timeout_site, sizeof(uint32_t) * 5);
}

// Copies role `role`'s events of the last launch into out (2 x uint64 each).
TPSA_API uint32_t tpsa_debug_trace(uint32_t role, unsigned long long* out, uint32_t max_events) {
  uint32_t n[kTraceRoles] = {};
  cudaDeviceSynchronize();
  if (role >= kTraceRoles) return 0;
  cudaMemcpyFromSymbol(n, g_trace_n, sizeof(n));
  uint32_t c = n[role] < max_events ? n[role] : max_events;
  cudaMemcpyFromSymbol(out, g_trace, sizeof(unsigned long long) * 2 * c,
                       sizeof(unsigned long long) * 2 * kTraceCap * role);
  return c;
}
#endif

tpsa_status tpsa_debug_wait_probe(uint32_t limit_ns) {
  t_last_error.clear();
  if (limit_ns != 0 && (limit_ns < 1000u || limit_ns > 100000000u)) {
    return fail(TPSA_ERR_INVALID_ARGUMENT, "probe limit must be 0 or in [1 us, 100 ms]");
  }
  t_probe_wait_ns = limit_ns;
  return TPSA_OK;
}

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
