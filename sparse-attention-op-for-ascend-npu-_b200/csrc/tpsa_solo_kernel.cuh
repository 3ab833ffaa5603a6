// Single-CTA ("solo") form of the TriangleMix kernel: each CTA runs a work
// item alone, and each of its two softmax warpgroups owns one M=128 tile.
//
// A work item is the same (64-token query block, kv head, key-tile range) as
// in the pair kernel.  Its 256 rows (64 tokens x 4 GQA heads) are two M=128
// query tiles in one CTA: tile 0 holds query heads {4h, 4h+1}, tile 1 heads
// {4h+2, 4h+3}.  Both read the same K/V tile from shared memory, so every
// K/V byte loaded serves 4 query heads, and both have the same key set.
// Softmax warpgroup x owns query tile x for the whole item: its rows' running
// reference max, row sum and O accumulator never leave it, so the two
// warpgroups run independently of each other.
//
// Roles (384 threads):
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
// tile's softmax overlaps the other tile's MMAs.
#ifndef TPSA_SOLO_KERNEL_CUH_
#define TPSA_SOLO_KERNEL_CUH_

namespace solo {

// Event trace of one CTA (build with -DTPSA_TRACE; CTA 2 * TPSA_TRACE_CLUSTER).
// Roles: 0 K producer, 1 MMA issuer, 2-3 softmax warpgroups, 4 V producer.
#ifdef TPSA_TRACE
#define TPSA_STR(role, ev, arg)                                      \
  do {                                                               \
    if (blockIdx.x == 2 * TPSA_TRACE_CLUSTER) TPSA_TR(role, ev, arg); \
  } while (0)
#else
#define TPSA_STR(role, ev, arg) \
  do {                          \
  } while (0)
#endif

constexpr int kNumThreads = 384;
constexpr uint32_t kQTileBytes = 2 * kQHalfBytes;     // 128 rows x 128 d (two d-halves)
constexpr uint32_t kKvHalfBytes = 128 * 128;          // 128 keys x 64 d
constexpr uint32_t kKvSlotBytes = 2 * kKvHalfBytes;   // one key tile of K, or of V
constexpr int kKRing = 2;
constexpr int kVRing = 2;
constexpr uint32_t kOffQ = 0;                                   // [query tile][d half]
constexpr uint32_t kOffK = kOffQ + 2 * kQTileBytes;              // K ring
constexpr uint32_t kOffV = kOffK + kKRing * kKvSlotBytes;        // V ring
// Output staging: 4 KB per softmax warp (its 32 rows x 64 columns as bf16,
// 128-byte swizzled), stored to `out` by the warp's own TMA store.
constexpr uint32_t kOutStageBytes = 32 * 128;
constexpr uint32_t kOffOut = kOffV + kVRing * kKvSlotBytes;
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
  kNumBars
};
// item_empty: K producer, V producer, MMA warp, 8 softmax warps.
constexpr uint32_t kItemConsumers = 3 + kSoftmaxWarps;

constexpr uint32_t kOffItemSlots = (kOffBar + kNumBars * 8 + 15) & ~15u;  // 2 x ItemRec
constexpr uint32_t kOffTmemSlot = kOffItemSlots + 2 * 64;
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
constexpr uint32_t kOffSplitLast = kOffAbort + 4;    // int32 [query tile][2]
constexpr uint32_t kOffCounters = kOffSplitLast + 16;  // uint32 [4]: split written / decided per tile
constexpr uint32_t kSmemUsed = kOffCounters + 16;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // alignment slack
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

constexpr uint32_t kTmemO = 256;

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

__device__ __forceinline__ bool wait(const Smem& sh, uint32_t bar, uint32_t parity) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  return wait_bar_slow<false>(bar, parity, sh.abort_flag());
}

__device__ __forceinline__ bool wait_count(const Smem& sh, uint32_t id, uint32_t target) {
  const uint32_t addr = sh.counter(id);
  if (static_cast<int32_t>(ptx::ld_acquire_shared(addr) - target) >= 0) return true;
  return wait_count_slow(sh.abort_flag(), addr, target);
}

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
__device__ __forceinline__ bool take_item_brief(const Smem& sh, uint32_t n, ItemBrief* b) {
  const uint32_t slot = n % 2;
  if (!wait(sh, sh.bar(kBarItemFull + slot), (n / 2) & 1)) return false;
  const int32_t* w = reinterpret_cast<const int32_t*>(sh.item_slot(slot));
  b->idx = w[offsetof(ItemRec, idx) / 4];
  b->ntiles = w[(offsetof(ItemRec, it) + offsetof(tpsa_item, tile_end)) / 4] -
              w[(offsetof(ItemRec, it) + offsetof(tpsa_item, tile_begin)) / 4];
  b->narrow = static_cast<uint32_t>(w[offsetof(ItemRec, narrow) / 4]);
  return true;
}

__device__ __forceinline__ void release_item(const Smem& sh, uint32_t n) {
  ptx::mbar_arrive(sh.bar(kBarItemEmpty + n % 2));
}

// Tile j of an item is 64 keys wide (the others are 128): see ItemRec::narrow.
__device__ __forceinline__ bool tile_narrow(uint32_t narrow, int32_t j, int32_t ntiles) {
  return (j < 2 && ((narrow >> j) & 1u)) || (j == ntiles - 1 && (narrow & 4u));
}

// ------------------------------------------------------------ scheduler
// One thread: takes items from the grid-wide counter (longest first, the
// same dispatch order as the pair kernel), decodes each into an item record
// and publishes it into the CTA's two-slot item ring.  An item is claimed
// only once its ring slot is free, i.e. once the softmax warpgroups have
// finished the item two before it: a CTA then holds at most the item it
// runs and the next one, so CTAs finish the launch within about one item of
// each other.
template <bool kVarlen>
__device__ void scheduler_role(const KernelArgs& a, const Smem& sh) {
  const tpsa_plan& p = a.plan;
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
  }
}

// ------------------------------------------------------------ producers
// K side: for each item the first K tile, then the two query tiles (each
// waits until the previous item's last QK of that tile completed), then the
// remaining K tiles.  V side: the V tiles.  One thread each.
template <bool kVarlen>
__device__ void producer_role(const KernelArgs& a, const Smem& sh, const CUtensorMap* tq,
                              const CUtensorMap* tk128, const CUtensorMap* tk64,
                              const CUtensorMap* tv, bool v_side) {
  const tpsa_plan& p = a.plan;
  if (v_side) {
    ptx::prefetch_tmap(tv);
  } else {
    ptx::prefetch_tmap(tq);
    ptx::prefetch_tmap(tk128);
    ptx::prefetch_tmap(tk64);
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
    TPSA_STR(trole, 20, rec.idx);
    const tpsa_item& it = rec.it;
    const BlockTiles& bt = rec.bt;
    const ReqDesc& rq = a.reqs[kVarlen ? rec.req() : 0];
    const int32_t* table = kVarlen ? a.block_table + rq.table_off : a.block_table;
    const int32_t req_seq_len = kVarlen ? rq.plan.seq_len : p.seq_len;
    const int32_t q_row0 = kVarlen ? rq.q_row0 : 0;
    if (!v_side) {
      // The item's query rows into L2 now: the shared-memory copy waits until
      // the previous item's last QK, and then reads them from L2.
      for (int32_t c = 0; c < 4; ++c) {
        ptx::tma_prefetch_3d(tq, (c & 1) * 64, it.kv_head * kGroupSize + 2 * (c >> 1),
                             q_row0 + it.block * kBlockQ);
      }
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
      if (a.tiles != nullptr && !v_side) {
        atomicAdd(a.tiles, 1ull);
        atomicAdd(a.tiles + 1, static_cast<unsigned long long>(w));
      }
      const uint32_t s = ring % ring_n;
      if (!wait(sh, bar_empty + 8 * s, ((ring / ring_n) & 1) ^ 1)) { ok = false; break; }
      ++ring;
      TPSA_STR(trole, 22, t);
      const uint32_t dst = ring_base + s * kKvSlotBytes;
      if (!v_side) {
        // Keys at or beyond seq_len (unwritten slots of the last page) only
        // meet masked scores, which select -inf whatever they hold.
        const CUtensorMap* km = w == kTileKeys ? tk128 : tk64;
        ptx::mbar_arrive_expect_tx(bar_full + 8 * s, static_cast<uint32_t>(w) * kHeadDim * 2);
        for (int dh = 0; dh < 2; ++dh) {
          ptx::tma_load_3d(dst + dh * kKvHalfBytes, km, dh * 64, it.kv_head, tok,
                           bar_full + 8 * s);
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
            TPSA_STR(trole, 21, x);
          }
          ++q_iter;
        }
      } else {
        const bool tail = k0 + w > req_seq_len;
        // Values at or beyond seq_len may be unwritten cache slots: such a
        // tile lands on a private barrier, those rows are zeroed (so that
        // P = 0 never meets a NaN), then the slot is published.
        const uint32_t lbar = tail ? sh.bar(kBarTail) : bar_full + 8 * s;
        ptx::mbar_arrive_expect_tx(lbar, static_cast<uint32_t>(w) * kHeadDim * 2);
        for (int dh = 0; dh < 2; ++dh) {
          for (int sub = 0; sub < w / 64; ++sub) {
            ptx::tma_load_3d(dst + dh * kKvHalfBytes + sub * 8192, tv, dh * 64, it.kv_head,
                             tok + sub * 64, lbar);
          }
        }
        if (tail) {
          if (!wait(sh, sh.bar(kBarTail), tail_iter & 1)) { ok = false; break; }
          ++tail_iter;
          for (int32_t row = req_seq_len - k0; row < w; ++row) {
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
  // S_x = Q_x K^T for the K tile in ring slot ks (N = 128 or 64).
  auto issue_qk = [&](uint32_t x, uint32_t ks, bool narrow) {
    const uint32_t d = tmem + (x << 7);
    const uint32_t idesc = narrow ? kIdQk64 : kIdQk128;
    const uint32_t qb = q_lo + x * kQTileUnits;
    const uint32_t kb = k_lo + ks * kSlotUnits;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t o = (k / 4) * kHalfUnits + (k % 4) * 2;
      ptx::umma_ss_if(leader, d, desc(qb + o, q_hi), desc(kb + o, k_hi), idesc, k > 0 ? 1u : 0u);
    }
  };
  // O_x (+)= P_x V for keys [64 half, 64 half + 64) of the V tile in ring
  // slot vs.
  auto issue_pv = [&](uint32_t x, uint32_t vs, uint32_t half, bool first) {
    const uint32_t d = tmem + kTmemO + (x << 7);
    const uint32_t pa = tmem + (x << 7) + 64 + half * 32;
    const uint32_t vb = v_lo + vs * kSlotUnits + half * (8192 >> 4);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      ptx::umma_ts_if(leader, d, pa + k * 8, desc(vb + k * (2048 >> 4), v_hi), kIdPv,
                      (first && half == 0 && k == 0) ? 0u : 1u);
    }
  };

  TPSA_TRACE_STATE;
  const bool tr = (threadIdx.x & 31) == 0;
  uint32_t n_item = 0;
  uint32_t ks = 0, k_phase = 0;  // K ring cursor of the next QK
  uint32_t vs = 0, v_phase = 0;  // V ring cursor of the next PV
  uint32_t p_par = 0;            // P-full phase (same for both tiles)
  bool ok = true;
  // Current item.
  ItemBrief cur;
  bool got = take_item_brief(sh, n_item, &cur);
  if (!__all_sync(0xffffffffu, got)) ok = false;
  __syncwarp();
  if (ok && (threadIdx.x & 31) == 0) release_item(sh, n_item);
  if (ok) ++n_item;
  bool done = !ok || cur.idx >= p.total_items;
  uint32_t q_iter = 0;
  if (!done) {
    // First QKs of the first item.
    const int32_t nt = cur.ntiles;
    const bool nar = tile_narrow(cur.narrow, 0, nt);
    for (uint32_t x = 0; x < 2 && ok; ++x) {
      if (!warp_wait(sh.bar(kBarQFull + x), 0)) { ok = false; break; }
      if (x == 0 && !warp_wait(sh.bar(kBarKFull + ks), k_phase)) { ok = false; break; }
      ptx::tc_fence_after();
      issue_qk(x, ks, nar);
      commit(sh.bar(kBarSFull + x));
      if (nt == 1) commit(sh.bar(kBarQEmpty + x));
    }
    commit(sh.bar(kBarKEmpty + ks));
    ks = (ks + 1) % kKRing;
    k_phase ^= ks == 0 ? 1u : 0u;
    ++q_iter;
  }
  while (ok && !done) {
    const int32_t nt = cur.ntiles;
    ItemBrief nxt;
    bool nxt_valid = false;
    for (int32_t j = 0; j < nt && ok; ++j) {
      const bool nar = tile_narrow(cur.narrow, j, nt);
      // The QK that follows PV(j) for each tile: tile j + 1 of this item, or
      // tile 0 of the next item.
      bool has_next = j + 1 < nt;
      bool new_item = false;
      bool next_nar = false, next_last = false;
      if (has_next) {
        next_nar = tile_narrow(cur.narrow, j + 1, nt);
        next_last = j + 1 == nt - 1;
      } else {
        const bool g = take_item_brief(sh, n_item, &nxt);
        if (!__all_sync(0xffffffffu, g)) { ok = false; break; }
        __syncwarp();
        if ((threadIdx.x & 31) == 0) release_item(sh, n_item);
        ++n_item;
        nxt_valid = nxt.idx < p.total_items;
        if (tr) TPSA_STR(1, 10, nxt.idx);
        if (nxt_valid) {
          const int32_t nn = nxt.ntiles;
          has_next = true;
          new_item = true;
          next_nar = tile_narrow(nxt.narrow, 0, nn);
          next_last = nn == 1;
        }
      }
      for (uint32_t x = 0; x < 2 && ok; ++x) {
        // PV of keys 0-63 as soon as their P is written, then keys 64-127.
        if (!warp_wait(sh.bar(kBarPHalf + x), p_par)) { ok = false; break; }
        if (tr) TPSA_STR(1, 13, x);
        if (x == 0 && !warp_wait(sh.bar(kBarVFull + vs), v_phase)) { ok = false; break; }
        if (tr && x == 0) TPSA_STR(1, 14, j);
        ptx::tc_fence_after();
        issue_pv(x, vs, 0, j == 0);
        if (!warp_wait(sh.bar(kBarPFull + x), p_par)) { ok = false; break; }
        ptx::tc_fence_after();
        if (!nar) issue_pv(x, vs, 1, false);
        if (x == 1) commit(sh.bar(kBarVEmpty + vs));
        if (j == nt - 1) commit(sh.bar(kBarOFull + x));
        if (has_next) {
          if (new_item && !warp_wait(sh.bar(kBarQFull + x), q_iter & 1)) { ok = false; break; }
          if (tr && new_item) TPSA_STR(1, 11, x);
          if (x == 0 && !warp_wait(sh.bar(kBarKFull + ks), k_phase)) { ok = false; break; }
          if (tr && x == 0) TPSA_STR(1, 17, j);
          ptx::tc_fence_after();
          issue_qk(x, ks, next_nar);
          if (tr) TPSA_STR(1, 18, x);
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
    if (!ok || !nxt_valid) break;
    cur = nxt;
  }
  // All MMAs issued by this warp complete before TMEM is released.
  commit(sh.bar(kBarDrain));
  if ((threadIdx.x & 31) == 0) drain_bar(sh.bar(kBarDrain), 0);
  __syncwarp();
}

// ------------------------------------------------------------ softmax
// Pairs of each 32-key chunk whose exponentials use the FMA-pipe polynomial
// (bit c: pair c; see exp_chunk).  None by default: measured at 8K with the
// whole row in registers (ms per launch), no pair 0.1140, 0x0001 0.1146,
// 0x0401 0.1153, 0x1111 0.1179.  (MUFU ex2 runs at 16 per clock per SM, as
// many exponentials per clock as the tensor pipe needs for this tile shape.)
#ifndef TPSA_SOLO_POLY_MASK
#define TPSA_SOLO_POLY_MASK 0u
#endif
constexpr uint32_t kSoloPoly = TPSA_SOLO_POLY_MASK;

// One key tile of query tile x, the whole row of this thread: load S (all of
// it into registers), mask, row max, move the lazy reference if this tile's
// maxima require it (O and the row sum rescaled first), exponentials and P
// into tensor memory over columns 64-127 of the S buffer.  P of keys 0-63 is
// published on t.prev_bar (the P-half barrier) before the exponentials of
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
    prepare_chunk<kVisit>(r2, t.masked, q, sparse, t.k0 + 64, visit_row, words_per_row);
    prepare_chunk<kVisit>(r3, t.masked, q, sparse, t.k0 + 96, visit_row, words_per_row);
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
  exp_chunk<kSoloPoly>(r0, sl2, neg_mb, p_addr, sum0, sum1);
  exp_chunk<kSoloPoly>(r1, sl2, neg_mb, p_addr + 16, sum0, sum1);
  ptx::tmem_wait_st();
  ptx::tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) ptx::mbar_arrive(t.prev_bar);
  if (t.wide) {
    exp_chunk<kSoloPoly>(r2, sl2, neg_mb, p_addr + 32, sum0, sum1);
    exp_chunk<kSoloPoly>(r3, sl2, neg_mb, p_addr + 48, sum0, sum1);
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
#ifdef TPSA_TRACE
  const bool tr = row == 0 && blockIdx.x == 2 * TPSA_TRACE_CLUSTER;
#else
  const bool tr = false;
#endif
#define tr_n_ tr_sm

  for (uint32_t n_item = 0;; ++n_item) {
    ItemRec rec;
    const bool got = take_item(sh, n_item, &rec);
    if (!__all_sync(0xffffffffu, got)) break;
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
      ta.wide = w > 64;
      ta.masked = tile_needs_mask(pr, bt, k0, w);
      ta.first = n == 0;
      ta.last = n == ntiles - 1;
      ta.trn = tr ? &tr_sm : nullptr;
      ta.trole = 2 + x;
      ta.prev_bar = bar_ph;
      const bool w_ok = wait(sh, bar_s, s_par);
      s_par ^= 1;
      if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
      if (tr) TPSA_STR(2 + x, 1, n);
      ptx::tc_fence_after();
      softmax_tile<kVisit>(ta, p.scale_log2, q, sparse, st, visit_row, a.words_per_row);
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_p);
      if (tr) TPSA_STR(2 + x, 3, n);
    }
    if (!ok) break;

    // Item end: O_x is complete once the item's last PV of this tile is.
    const bool w_ok = wait(sh, bar_o, o_par);
    o_par ^= 1;
    if (!__all_sync(0xffffffffu, w_ok)) break;
    ptx::tc_fence_after();
    if (tr) TPSA_STR(2 + x, 5, rec.idx);
    const bool split = it.num_splits > 1;
    const uint32_t sp_slot = split_items & 1;
    split_items += split ? 1u : 0u;
    // Output rows of this warp: packed token base_q + R / 2, head
    // base_h + R % 2 for warp row R; rows at or past row_end are not written.
    const int32_t base_q = q_row0 + it.block * kBlockQ + quad * 16;
    const int32_t base_h = it.kv_head * kGroupSize + 2 * static_cast<int32_t>(x);
    const int32_t row_end = q_row0 + pr.query_tokens;
    if (!split && (!kVarlen || bt.q_end - bt.q_begin == kBlockQ)) {
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
      if (tr) TPSA_STR(2 + x, 6, 0);
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
      if (tr) TPSA_STR(2 + x, 6, 0);
      continue;
    }

    // Split item: the fp32 partial (128 columns) into the item's column-major
    // slot ([128 columns][256 rows], then m[256] and l[256]; this tile's rows
    // are 128 x + row); the last split of the block (per query tile) merges
    // all partials and writes bf16.
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
    if (lane == 0) ptx::red_release_add_shared(sh.counter(cnt_w), 1);
    if (row == 0) {
      if (wait_count(sh, cnt_w, 4 * split_items)) {
        int32_t* ctr = a.ctl + kCtlSplitBase + (kVarlen ? rq.ctr_base : 0) +
                       ((it.block - pr.tail_block0) * p.kv_heads + it.kv_head) * 2 +
                       static_cast<int32_t>(x);
        const int prev = atomicAdd(ctr, 1);
        split_last[sp_slot] = prev == it.num_splits - 1;
        ptx::red_release_add_shared(sh.counter(cnt_d), 1);
      }
    }
    const bool decided = __all_sync(0xffffffffu, wait_count(sh, cnt_d, split_items));
    if (!decided) break;
    if (!split_last[sp_slot]) continue;
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
    stage_free();
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
  // Output stores of this warp complete before the CTA exits.
  if (lane == 0) ptx::bulk_wait_group<0>();
}
#undef tr_n_

}  // namespace solo

template <bool kVisit, bool kVarlen>
__global__ void __launch_bounds__(solo::kNumThreads, 1)
    tpsa_solo_kernel(const __grid_constant__ KernelArgs args,
                     const __grid_constant__ CUtensorMap tmap_q,
                     const __grid_constant__ CUtensorMap tmap_k128,
                     const __grid_constant__ CUtensorMap tmap_k64,
                     const __grid_constant__ CUtensorMap tmap_v,
                     const __grid_constant__ CUtensorMap tmap_out) {
  extern __shared__ uint8_t smem_raw[];
  solo::Smem sh;
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
      ptx::mbar_init(sh.bar(solo::kBarQFull + x), 1);
      ptx::mbar_init(sh.bar(solo::kBarQEmpty + x), 1);
      ptx::mbar_init(sh.bar(solo::kBarSFull + x), 1);
      ptx::mbar_init(sh.bar(solo::kBarPFull + x), 4);
      ptx::mbar_init(sh.bar(solo::kBarPHalf + x), 4);
      ptx::mbar_init(sh.bar(solo::kBarOFull + x), 1);
      ptx::mbar_init(sh.bar(solo::kBarItemFull + x), 1);
      ptx::mbar_init(sh.bar(solo::kBarItemEmpty + x), solo::kItemConsumers);
    }
    for (int s = 0; s < solo::kKRing; ++s) {
      ptx::mbar_init(sh.bar(solo::kBarKFull + s), 1);
      ptx::mbar_init(sh.bar(solo::kBarKEmpty + s), 1);
    }
    for (int s = 0; s < solo::kVRing; ++s) {
      ptx::mbar_init(sh.bar(solo::kBarVFull + s), 1);
      ptx::mbar_init(sh.bar(solo::kBarVEmpty + s), 1);
    }
    ptx::mbar_init(sh.bar(solo::kBarTail), 1);
    ptx::mbar_init(sh.bar(solo::kBarDrain), 1);
    *sh.abort_flag() = 0;
    for (uint32_t i = 0; i < 4; ++i) {
      *reinterpret_cast<volatile uint32_t*>(sh.base + solo::kOffCounters + 4 * i) = 0;
    }
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(sh.base_u32 + solo::kOffTmemSlot, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sh.base + solo::kOffTmemSlot);

  if (warp < kFirstSoftmaxWarp) {
    ptx::setmaxnreg_dec<kControlRegs>();
    if (warp == 0) {
      if (lane == 0) solo::producer_role<kVarlen>(args, sh, &tmap_q, &tmap_k128, &tmap_k64, &tmap_v, false);
      __syncwarp();
    } else if (warp == 1) {
      solo::mma_role(args, sh, tmem);
    } else if (warp == 2) {
      if (lane == 0) solo::scheduler_role<kVarlen>(args, sh);
      __syncwarp();
    } else {
      if (lane == 0) solo::producer_role<kVarlen>(args, sh, &tmap_q, &tmap_k128, &tmap_k64, &tmap_v, true);
      __syncwarp();
    }
  } else {
    ptx::setmaxnreg_inc<kSoftmaxRegs>();
    solo::softmax_role<kVisit, kVarlen>(args, sh, tmem, &tmap_out);
  }

  ptx::tc_fence_before();
  __syncthreads();  // MMAs drained, every role done
#ifdef TPSA_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_cta_span[blockIdx.x][1] = ptx::globaltimer_ns();
#endif
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

#endif  // TPSA_SOLO_KERNEL_CUH_
