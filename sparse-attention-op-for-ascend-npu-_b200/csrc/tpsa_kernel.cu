// TriangleMix paged sparse prefill attention for B200 (sm_100a).
//
// One persistent launch computes, for every query row, the dense causal
// prefix / sink+local-window middle / dense causal tail key set of the
// reference operator (operator/op_kernel/triangle_paged_fia_fast_path.h:
// 209-438) under one online softmax, reading K/V pages straight from the
// BSND paged cache through the block table and writing bf16 output into the
// caller's buffer.
//
// CTA organisation (one CTA per SM, 320 threads):
//   warp 0      TMA producer: Q block (4 boxes), K/V key tiles (64-row boxes)
//   warp 1      tcgen05 MMA issuer (lane 0) and TMEM owner
//   warps 2-5   softmax + epilogue of M tile 0 (query heads 4h, 4h+1)
//   warps 6-9   softmax + epilogue of M tile 1 (query heads 4h+2, 4h+3)
// A work item is (64-token query block, kv head, key-tile range).  Its 256
// rows (64 tokens x 4 GQA heads) are two M=128 tiles; both read the same
// K/V tile from shared memory, so every K/V byte loaded serves 4 heads.
//
// Tensor memory (512 columns, fp32):
//   [  0,128) S0 / P0   [128,256) S1 / P1   [256,384) O0   [384,512) O1
// P (bf16 pairs) overwrites the first half of its S tile after the softmax
// warps have read S.  Per M tile the MMA order is
//   QK(n) -> softmax(n) -> PV(n) -> QK(n+1)
// and the two M tiles alternate, so one tile's softmax overlaps the other's
// MMAs.  The O rescale for a grown row max is lazy (only when the max grows
// by more than 2^8) and is done by the softmax warps in tensor memory.
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

namespace {

constexpr int kNumThreads = 320;
constexpr int kStages = 2;
constexpr uint32_t kTmemCols = 512;
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;  // 1 s per wait
constexpr float kRescaleLog2 = 8.0f;  // lazy O rescale threshold (log2 units)

// Shared memory (offsets from a 1024-byte aligned base).
constexpr uint32_t kHalfBytes = 128 * 128;        // 128 rows x 64 bf16
constexpr uint32_t kQBytes = 4 * kHalfBytes;      // [m tile][d half]
constexpr uint32_t kStageBytes = 2 * kHalfBytes;  // [d half]
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kQBytes;
constexpr uint32_t kOffV = kOffK + kStages * kStageBytes;
constexpr uint32_t kOffBar = kOffV + kStages * kStageBytes;

enum BarId : uint32_t {
  kBarQFull = 0,
  kBarQEmpty,
  kBarKFull,                      // + stage
  kBarKEmpty = kBarKFull + kStages,
  kBarVFull = kBarKEmpty + kStages,
  kBarVEmpty = kBarVFull + kStages,
  kBarSFull = kBarVEmpty + kStages,  // + m tile
  kBarPFull = kBarSFull + 2,
  kBarOFull = kBarPFull + 2,
  kBarOEmpty = kBarOFull + 2,
  kBarSplitWritten = kBarOEmpty + 2,
  kBarSplitDecided,
  kBarDrain,
  kNumBars
};

constexpr uint32_t kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
constexpr uint32_t kOffSplitLast = kOffAbort + 4;
constexpr uint32_t kSmemUsed = kOffSplitLast + 4;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // alignment slack
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

struct KernelArgs {
  tpsa_plan plan;
  const int32_t* block_table;
  __nv_bfloat16* out;
  float* scratch;      // split partials (tail_items slots)
  int32_t* split_ctr;  // one counter per (tail block, kv head)
  int32_t num_pages;
  int32_t words_per_row;       // visit mode
  uint32_t* visited;           // visit mode
  unsigned long long* tiles;   // visit mode: [tiles, keys]
};

struct Shared {
  uint8_t* base;
  uint32_t base_u32;
  __device__ uint32_t bar(uint32_t id) const { return base_u32 + kOffBar + 8 * id; }
  __device__ volatile int* abort_flag() const {
    return reinterpret_cast<volatile int*>(base + kOffAbort);
  }
};

__device__ __forceinline__ void raise_status(uint32_t bits) {
  atomicOr(&g_device_status, bits);
}

// Bounded wait: gives up after kWaitTimeoutNs or as soon as another role has
// aborted; on timeout records TPSA_DEVICE_WAIT_TIMEOUT and aborts the CTA.
__device__ __noinline__ bool wait_bar_slow(uint32_t bar, uint32_t parity,
                                           volatile int* abort_flag) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (true) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1;
      raise_status(TPSA_DEVICE_WAIT_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ bool wait_bar(const Shared& sh, uint32_t bar,
                                         uint32_t parity) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  return wait_bar_slow(bar, parity, sh.abort_flag());
}

// Bounded wait used while draining after an abort (ignores the abort flag).
__device__ __noinline__ void drain_bar(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
      raise_status(TPSA_DEVICE_WAIT_TIMEOUT);
      return;
    }
  }
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ------------------------------------------------------------ producer
__device__ void producer_role(const KernelArgs& a, const Shared& sh,
                              const CUtensorMap* tq, const CUtensorMap* tk,
                              const CUtensorMap* tv) {
  const tpsa_plan& p = a.plan;
  ptx::prefetch_tmap(tq);
  ptx::prefetch_tmap(tk);
  ptx::prefetch_tmap(tv);
  uint32_t kv_iter = 0, item_iter = 0;
  uint32_t stage_arms[kStages] = {0, 0};
  bool ok = true;
  for (int32_t idx = blockIdx.x; ok && idx < p.total_items; idx += gridDim.x) {
    const tpsa_item it = decode_item(p, idx);
    const BlockTiles bt = block_tiles(p, it.block);
    if (item_iter > 0 && !wait_bar(sh, sh.bar(kBarQEmpty), (item_iter - 1) & 1)) {
      ok = false;
      break;
    }
    ptx::mbar_arrive_expect_tx(sh.bar(kBarQFull), kQBytes);
    for (int mt = 0; mt < 2; ++mt) {
      for (int dh = 0; dh < 2; ++dh) {
        ptx::tma_load_3d(sh.base_u32 + kOffQ + (mt * 2 + dh) * kHalfBytes, tq,
                         dh * 64, it.kv_head * kGroupSize + mt * 2,
                         it.block * kBlockQ, sh.bar(kBarQFull));
      }
    }
    ++item_iter;
    for (int32_t t = it.tile_begin; t < it.tile_end; ++t) {
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
      if (a.tiles != nullptr) {
        atomicAdd(a.tiles, 1ull);
        atomicAdd(a.tiles + 1, static_cast<unsigned long long>(w));
      }
      const uint32_t s = kv_iter % kStages;
      const uint32_t empty_parity = ((kv_iter / kStages) & 1) ^ 1;
      const uint32_t bytes = static_cast<uint32_t>(w) * kHeadDim * 2;
      if (!wait_bar(sh, sh.bar(kBarKEmpty + s), empty_parity)) {
        ok = false;
        break;
      }
      ptx::mbar_arrive_expect_tx(sh.bar(kBarKFull + s), bytes);
      for (int dh = 0; dh < 2; ++dh) {
        for (int sub = 0; sub < w / 64; ++sub) {
          ptx::tma_load_3d(
              sh.base_u32 + kOffK + s * kStageBytes + dh * kHalfBytes + sub * 8192,
              tk, dh * 64, it.kv_head, tok + sub * 64, sh.bar(kBarKFull + s));
        }
      }
      if (!wait_bar(sh, sh.bar(kBarVEmpty + s), empty_parity)) {
        // K of this stage is armed; account for it in the drain below.
        ++stage_arms[s];
        ok = false;
        break;
      }
      ptx::mbar_arrive_expect_tx(sh.bar(kBarVFull + s), bytes);
      for (int dh = 0; dh < 2; ++dh) {
        for (int sub = 0; sub < w / 64; ++sub) {
          ptx::tma_load_3d(
              sh.base_u32 + kOffV + s * kStageBytes + dh * kHalfBytes + sub * 8192,
              tv, dh * 64, it.kv_head, tok + sub * 64, sh.bar(kBarVFull + s));
        }
      }
      ++stage_arms[s];
      ++kv_iter;
    }
  }
  // Every TMA load this thread issued must land before the CTA exits.
  if (item_iter > 0) drain_bar(sh.bar(kBarQFull), (item_iter - 1) & 1);
  for (uint32_t s = 0; s < kStages; ++s) {
    if (stage_arms[s] > 0) {
      drain_bar(sh.bar(kBarKFull + s), (stage_arms[s] - 1) & 1);
    }
  }
  // V stages: the last armed phase of each stage (kv_iter counts V arms).
  for (uint32_t s = 0; s < kStages; ++s) {
    const uint32_t arms = kv_iter / kStages + (s < kv_iter % kStages ? 1 : 0);
    if (arms > 0) drain_bar(sh.bar(kBarVFull + s), (arms - 1) & 1);
  }
}

// ------------------------------------------------------------ MMA issuer
__device__ void mma_role(const KernelArgs& a, const Shared& sh, uint32_t tmem,
                         int lane) {
  const tpsa_plan& p = a.plan;
  constexpr uint32_t kIdescQK128 = ptx::idesc_bf16_f32(128, 128, 0);
  constexpr uint32_t kIdescQK64 = ptx::idesc_bf16_f32(128, 64, 0);
  constexpr uint32_t kIdescPV = ptx::idesc_bf16_f32(128, 128, 1);
  uint32_t kv_iter = 0, item_iter = 0;
  uint32_t p_parity[2] = {0, 0};
  bool ok = true;

  auto issue_qk = [&](int m, uint32_t stage, int32_t w) {
    const uint32_t d = tmem + m * 128;
    const uint32_t idesc = w == 128 ? kIdescQK128 : kIdescQK64;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t qa = sh.base_u32 + kOffQ + (m * 2 + k / 4) * kHalfBytes + (k % 4) * 32;
      const uint32_t kb = sh.base_u32 + kOffK + stage * kStageBytes + (k / 4) * kHalfBytes + (k % 4) * 32;
      ptx::umma_ss(d, ptx::smem_desc_sw128(qa, 16, 1024),
                   ptx::smem_desc_sw128(kb, 16, 1024), idesc, k > 0 ? 1u : 0u);
    }
  };
  auto issue_pv = [&](int m, uint32_t stage, int32_t w, bool first) {
    const uint32_t d = tmem + 256 + m * 128;
    const uint32_t pa = tmem + m * 128;
    for (int k = 0; k < w / 16; ++k) {
      const uint32_t vb = sh.base_u32 + kOffV + stage * kStageBytes + k * 16 * 128;
      ptx::umma_ts(d, pa + k * 8, ptx::smem_desc_sw128(vb, kHalfBytes, 1024),
                   kIdescPV, (first && k == 0) ? 0u : 1u);
    }
  };
  // Keys at or beyond seq_len in the last tile may be unwritten cache slots;
  // their V rows are zeroed so that P = 0 never meets a NaN.  Every lane
  // first observes the V-full barrier (already complete) so the TMA bytes
  // are ordered before its stores.
  auto zero_v_tail = [&](uint32_t stage, uint32_t parity, int32_t k0, int32_t w) -> bool {
    const int32_t valid = p.seq_len - k0;
    if (valid >= w) return true;
    if (!wait_bar(sh, sh.bar(kBarVFull + stage), parity)) return false;
    for (int32_t r = valid; r < w; ++r) {
      for (int dh = 0; dh < 2; ++dh) {
        uint4* row = reinterpret_cast<uint4*>(sh.base + kOffV + stage * kStageBytes +
                                              dh * kHalfBytes + r * 128);
        if (lane < 8) row[lane] = make_uint4(0, 0, 0, 0);
      }
    }
    ptx::fence_proxy_async_smem();
    return true;
  };

  for (int32_t idx = blockIdx.x; ok && idx < p.total_items; idx += gridDim.x) {
    const tpsa_item it = decode_item(p, idx);
    const BlockTiles bt = block_tiles(p, it.block);
    const int32_t ntiles = it.tile_end - it.tile_begin;
    bool w_ok = true;
    if (lane == 0) w_ok = wait_bar(sh, sh.bar(kBarQFull), item_iter & 1);
    if (!__shfl_sync(0xffffffffu, w_ok, 0)) { ok = false; break; }
    ptx::tc_fence_after();

    int32_t k0, w;
    tile_keys(bt, it.tile_begin, &k0, &w);
    {
      const uint32_t s = kv_iter % kStages;
      if (lane == 0) w_ok = wait_bar(sh, sh.bar(kBarKFull + s), (kv_iter / kStages) & 1);
      if (!__shfl_sync(0xffffffffu, w_ok, 0)) { ok = false; break; }
      ptx::tc_fence_after();
      if (lane == 0) {
        issue_qk(0, s, w);
        ptx::umma_commit(sh.bar(kBarSFull + 0));
        issue_qk(1, s, w);
        ptx::umma_commit(sh.bar(kBarSFull + 1));
        ptx::umma_commit(sh.bar(kBarKEmpty + s));
        if (ntiles == 1) ptx::umma_commit(sh.bar(kBarQEmpty));
      }
      __syncwarp();
    }
    for (int32_t n = 0; n < ntiles && ok; ++n) {
      const uint32_t s = (kv_iter + n) % kStages;
      const uint32_t ph = ((kv_iter + n) / kStages) & 1;
      if (lane == 0) w_ok = wait_bar(sh, sh.bar(kBarVFull + s), ph);
      if (!__shfl_sync(0xffffffffu, w_ok, 0)) { ok = false; break; }
      ptx::tc_fence_after();
      if (!__all_sync(0xffffffffu, zero_v_tail(s, ph, k0, w))) { ok = false; break; }
      int32_t k0n = 0, wn = 0;
      const bool has_next = n + 1 < ntiles;
      if (has_next) tile_keys(bt, it.tile_begin + n + 1, &k0n, &wn);
      const uint32_t sn = (kv_iter + n + 1) % kStages;
      const uint32_t phn = ((kv_iter + n + 1) / kStages) & 1;
      for (int m = 0; m < 2 && ok; ++m) {
        if (lane == 0) {
          if (n == 0 && item_iter > 0) {
            w_ok = wait_bar(sh, sh.bar(kBarOEmpty + m), (item_iter - 1) & 1);
          }
          if (w_ok) w_ok = wait_bar(sh, sh.bar(kBarPFull + m), p_parity[m]);
          p_parity[m] ^= 1;
        }
        if (!__shfl_sync(0xffffffffu, w_ok, 0)) { ok = false; break; }
        ptx::tc_fence_after();
        if (lane == 0) {
          issue_pv(m, s, w, n == 0);
          if (n + 1 == ntiles) ptx::umma_commit(sh.bar(kBarOFull + m));
        }
        if (has_next) {
          if (m == 0 && lane == 0) w_ok = wait_bar(sh, sh.bar(kBarKFull + sn), phn);
          if (!__shfl_sync(0xffffffffu, w_ok, 0)) { ok = false; break; }
          ptx::tc_fence_after();
          if (lane == 0) {
            issue_qk(m, sn, wn);
            ptx::umma_commit(sh.bar(kBarSFull + m));
            if (m == 1) {
              ptx::umma_commit(sh.bar(kBarKEmpty + sn));
              if (n + 2 == ntiles) ptx::umma_commit(sh.bar(kBarQEmpty));
            }
          }
        }
        __syncwarp();
      }
      if (lane == 0 && ok) ptx::umma_commit(sh.bar(kBarVEmpty + s));
      __syncwarp();
      k0 = k0n;
      w = wn;
    }
    kv_iter += ntiles;
    ++item_iter;
  }
  // All MMAs issued by this thread complete before TMEM is released.
  if (lane == 0) {
    ptx::umma_commit(sh.bar(kBarDrain));
    drain_bar(sh.bar(kBarDrain), 0);
  }
  __syncwarp();
}

// ------------------------------------------------------------ softmax
struct RowCtx {
  int32_t tok;     // absolute position of this row's query token
  int32_t sparse;  // row reads sink + window instead of the dense prefix
};

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

// One key tile of one M tile: mask, online-softmax update, P -> TMEM.
template <int W>
__device__ __forceinline__ void softmax_tile(const tpsa_plan& p, uint32_t s_addr,
                                             uint32_t o_addr, const RowCtx& rc,
                                             int32_t k0, bool masked, bool first,
                                             float& m_run, float& l_run,
                                             uint32_t* visit_row,
                                             int32_t words_per_row) {
  float s[W];
  load_s<W>(s_addr, s);
  if (masked) {
    const int32_t q = rc.tok < p.seq_len ? rc.tok : p.seq_len - 1;
    const int32_t hi = q - k0 + 1;
    const int32_t lo = rc.sparse ? q - kLocalWindow - k0 : -(1 << 30);
    const int32_t sk = kSinkTokens - k0;
#pragma unroll
    for (int c = 0; c < W; ++c) {
      const bool v = (c < hi) && (c >= lo || c < sk);
      s[c] = v ? s[c] : -INFINITY;
    }
  }
  if (visit_row != nullptr) {
#pragma unroll
    for (int j = 0; j < W / 32; ++j) {
      uint32_t bits = 0;
#pragma unroll
      for (int c = 0; c < 32; ++c) bits |= (s[32 * j + c] != -INFINITY ? 1u : 0u) << c;
      const int32_t word = k0 / 32 + j;
      if (bits != 0 && word < words_per_row) atomicOr(visit_row + word, bits);
    }
  }
  float mx = -INFINITY;
#pragma unroll
  for (int c = 0; c < W; ++c) mx = fmaxf(mx, s[c]);
  const float m_new = fmaxf(m_run, mx);
  const bool need = (m_new - m_run) * p.scale_log2 > kRescaleLog2;
  if (__any_sync(0xffffffffu, need)) {
    const float factor = need ? fast_exp2((m_run - m_new) * p.scale_log2) : 1.0f;
    if (!first) rescale_o(o_addr, factor);
    l_run *= factor;
    if (need) m_run = m_new;
  }
  const float mb = m_run == -INFINITY ? 0.0f : m_run * p.scale_log2;
  float sum = 0.0f;
  uint32_t pk[W / 2];
#pragma unroll
  for (int c = 0; c < W / 2; ++c) {
    const float e0 = fast_exp2(fmaf(s[2 * c], p.scale_log2, -mb));
    const float e1 = fast_exp2(fmaf(s[2 * c + 1], p.scale_log2, -mb));
    sum += e0 + e1;
    pk[c] = pack_bf16x2(e0, e1);
  }
  l_run += sum;
#pragma unroll
  for (int j = 0; j < W / 64; ++j) {
    ptx::tmem_st32(s_addr + 32 * j, *reinterpret_cast<uint32_t(*)[32]>(&pk[32 * j]));
  }
  ptx::tmem_wait_st();
}

__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* dst, const float* v,
                                               float scale) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 u;
    u.x = pack_bf16x2(v[8 * j + 0] * scale, v[8 * j + 1] * scale);
    u.y = pack_bf16x2(v[8 * j + 2] * scale, v[8 * j + 3] * scale);
    u.z = pack_bf16x2(v[8 * j + 4] * scale, v[8 * j + 5] * scale);
    u.w = pack_bf16x2(v[8 * j + 6] * scale, v[8 * j + 7] * scale);
    d[j] = u;
  }
}

__device__ void softmax_role(const KernelArgs& a, const Shared& sh, uint32_t tmem,
                             int m) {
  const tpsa_plan& p = a.plan;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int quad = warp % 4;
  const int row = quad * 32 + lane;  // TMEM lane == row of the M tile
  const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
  const uint32_t s_addr = tmem + lane_base + m * 128;
  const uint32_t o_addr = tmem + lane_base + 256 + m * 128;
  const int32_t hq = p.kv_heads * kGroupSize;
  const bool visit = a.visited != nullptr;
  uint32_t s_parity = 0, o_parity = 0, split_iter = 0;
  volatile int* split_last = reinterpret_cast<volatile int*>(sh.base + kOffSplitLast);

  for (int32_t idx = blockIdx.x; idx < p.total_items; idx += gridDim.x) {
    const tpsa_item it = decode_item(p, idx);
    const BlockTiles bt = block_tiles(p, it.block);
    RowCtx rc;
    rc.tok = bt.q_begin + row / 2;
    rc.sparse = row_is_sparse(p, rc.tok) ? 1 : 0;
    const int32_t qrow = it.block * kBlockQ + row / 2;  // row within the chunk
    const int32_t head = it.kv_head * kGroupSize + m * 2 + (row & 1);
    const bool real_row = qrow < p.query_tokens;
    uint32_t* visit_row =
        (visit && real_row)
            ? a.visited + (static_cast<size_t>(qrow) * hq + head) * a.words_per_row
            : nullptr;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int32_t t = it.tile_begin; t < it.tile_end; ++t) {
      int32_t k0, w;
      tile_keys(bt, t, &k0, &w);
      const bool masked = tile_needs_mask(p, bt, k0, w);
      bool w_ok = wait_bar(sh, sh.bar(kBarSFull + m), s_parity);
      s_parity ^= 1;
      if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
      ptx::tc_fence_after();
      if (w == 128) {
        softmax_tile<128>(p, s_addr, o_addr, rc, k0, masked, t == it.tile_begin,
                          m_run, l_run, visit_row, a.words_per_row);
      } else {
        softmax_tile<64>(p, s_addr, o_addr, rc, k0, masked, t == it.tile_begin,
                         m_run, l_run, visit_row, a.words_per_row);
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(sh.bar(kBarPFull + m));
    }
    if (!ok) break;
    bool w_ok = wait_bar(sh, sh.bar(kBarOFull + m), o_parity);
    o_parity ^= 1;
    if (!__all_sync(0xffffffffu, w_ok)) break;
    ptx::tc_fence_after();

    if (it.num_splits == 1) {
      const float inv = 1.0f / l_run;
      __nv_bfloat16* dst = a.out + (static_cast<size_t>(qrow) * hq + head) * kHeadDim;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        ptx::tmem_ld32(o_addr + 32 * c, r);
        ptx::tmem_wait_ld();
        if (real_row) store_row_bf16(dst + 32 * c, reinterpret_cast<const float*>(r), inv);
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(sh.bar(kBarOEmpty + m));
      continue;
    }

    // Split item: publish (O, m, l) of this row, then the last split of the
    // block merges all partials (log-sum-exp combine) and writes bf16.
    float* slot = a.scratch + static_cast<size_t>(idx) * kSlotFloats;
    const int32_t srow = m * kRowsPerTile + row;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      ptx::tmem_ld32(o_addr + 32 * c, r);
      ptx::tmem_wait_ld();
      float4* d = reinterpret_cast<float4*>(slot + static_cast<size_t>(srow) * kHeadDim + 32 * c);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        d[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                           __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
      }
    }
    ptx::tc_fence_before();
    ptx::mbar_arrive(sh.bar(kBarOEmpty + m));
    slot[2 * kRowsPerTile * kHeadDim + srow] = m_run;
    slot[2 * kRowsPerTile * (kHeadDim + 1) + srow] = l_run;
    __threadfence();
    ptx::mbar_arrive(sh.bar(kBarSplitWritten));
    w_ok = wait_bar(sh, sh.bar(kBarSplitWritten), split_iter & 1);
    if (!__all_sync(0xffffffffu, w_ok)) break;
    const int32_t ctr = (it.block - p.tail_block0) * p.kv_heads + it.kv_head;
    if (m == 0 && row == 0) {
      const int prev = atomicAdd(a.split_ctr + ctr, 1);
      const int last = prev == it.num_splits - 1;
      if (last) a.split_ctr[ctr] = 0;  // leave the counter clean
      *split_last = last;
      ptx::mbar_arrive(sh.bar(kBarSplitDecided));
    }
    w_ok = wait_bar(sh, sh.bar(kBarSplitDecided), split_iter & 1);
    ++split_iter;
    if (!__all_sync(0xffffffffu, w_ok)) break;
    if (!*split_last || !real_row) continue;
    __threadfence();
    const float* first_slot = a.scratch + static_cast<size_t>(idx - it.split) * kSlotFloats;
    float mmax = -INFINITY;
    for (int32_t sp = 0; sp < it.num_splits; ++sp) {
      const float* sl = first_slot + static_cast<size_t>(sp) * kSlotFloats;
      mmax = fmaxf(mmax, __ldcg(sl + 2 * kRowsPerTile * kHeadDim + srow));
    }
    float wts[64];  // num_splits <= 64 enforced by the planner
    float lsum = 0.0f;
    for (int32_t sp = 0; sp < it.num_splits; ++sp) {
      const float* sl = first_slot + static_cast<size_t>(sp) * kSlotFloats;
      const float ms = __ldcg(sl + 2 * kRowsPerTile * kHeadDim + srow);
      const float ls = __ldcg(sl + 2 * kRowsPerTile * (kHeadDim + 1) + srow);
      const float wgt = ms == -INFINITY ? 0.0f : fast_exp2((ms - mmax) * p.scale_log2);
      wts[sp & 63] = wgt;
      lsum += wgt * ls;
    }
    const float inv = 1.0f / lsum;
    __nv_bfloat16* dst = a.out + (static_cast<size_t>(qrow) * hq + head) * kHeadDim;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float acc[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
      for (int32_t sp = 0; sp < it.num_splits; ++sp) {
        const float wgt = wts[sp & 63];
        const float4* src = reinterpret_cast<const float4*>(
            first_slot + static_cast<size_t>(sp) * kSlotFloats +
            static_cast<size_t>(srow) * kHeadDim + 32 * c);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 v = __ldcg(src + j);
          acc[4 * j] += wgt * v.x;
          acc[4 * j + 1] += wgt * v.y;
          acc[4 * j + 2] += wgt * v.z;
          acc[4 * j + 3] += wgt * v.w;
        }
      }
      store_row_bf16(dst + 32 * c, acc, inv);
    }
  }
}

template <bool kVisit>
__global__ void __launch_bounds__(kNumThreads, 1)
    tpsa_paged_kernel(const __grid_constant__ KernelArgs args,
                      const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v) {
  extern __shared__ uint8_t smem_raw[];
  Shared sh;
  {
    const uint32_t raw = ptx::smem_u32(smem_raw);
    const uint32_t aligned = (raw + 1023u) & ~1023u;
    sh.base = smem_raw + (aligned - raw);
    sh.base_u32 = aligned;
  }
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    ptx::mbar_init(sh.bar(kBarQFull), 1);
    ptx::mbar_init(sh.bar(kBarQEmpty), 1);
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(sh.bar(kBarKFull + s), 1);
      ptx::mbar_init(sh.bar(kBarKEmpty + s), 1);
      ptx::mbar_init(sh.bar(kBarVFull + s), 1);
      ptx::mbar_init(sh.bar(kBarVEmpty + s), 1);
    }
    for (int m = 0; m < 2; ++m) {
      ptx::mbar_init(sh.bar(kBarSFull + m), 1);
      ptx::mbar_init(sh.bar(kBarPFull + m), 128);
      ptx::mbar_init(sh.bar(kBarOFull + m), 1);
      ptx::mbar_init(sh.bar(kBarOEmpty + m), 128);
    }
    ptx::mbar_init(sh.bar(kBarSplitWritten), 256);
    ptx::mbar_init(sh.bar(kBarSplitDecided), 1);
    ptx::mbar_init(sh.bar(kBarDrain), 1);
    *sh.abort_flag() = 0;
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

  if (warp == 0) {
    if (lane == 0) producer_role(args, sh, &tmap_q, &tmap_k, &tmap_v);
    __syncwarp();
  } else if (warp == 1) {
    mma_role(args, sh, tmem, lane);
  } else {
    softmax_role(args, sh, tmem, warp < 6 ? 0 : 1);
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
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

tpsa_status build_plan(int64_t query_tokens, int64_t query_start, int64_t seq_len,
                       int64_t prompt_len, int32_t kv_heads, int32_t sm_count,
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
  if (sm_count <= 0) return fail(TPSA_ERR_INVALID_ARGUMENT, "sm_count must be positive");
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
  const double target = static_cast<double>(tiles) / sm_count;
  int32_t split = static_cast<int32_t>(0.7 * target);
  if (split < kMinSplitTiles) split = kMinSplitTiles;
  // The in-kernel merge keeps per-split weights for at most 64 splits.
  for (int32_t b = b0; b < p->num_blocks; ++b) {
    const int32_t c = block_tiles(*p, b).count;
    if (ceil_div(c, split) > 64) split = ceil_div(c, 64);
  }
  if ((p->num_blocks - b0) * kv_heads > kMaxSplitCounters) split = 1 << 30;
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
  p->grid = p->total_items < sm_count ? p->total_items : sm_count;
  p->total_tiles = tiles;
  p->workspace_bytes = any_split ? kControlBytes + tail_items * kSlotBytes : 0;
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
  st = build_plan(query_tokens, query_start, seq_len, prompt_len, kv_heads, dev->sm_count,
                  scale, &args.plan);
  if (st != TPSA_OK) return st;
  const tpsa_plan& p = args.plan;
  if (p.workspace_bytes > 0) {
    if (workspace == nullptr || workspace_bytes < static_cast<uint64_t>(p.workspace_bytes)) {
      return fail(TPSA_ERR_WORKSPACE, "workspace smaller than tpsa_workspace_size()");
    }
    if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) {
      return fail(TPSA_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    }
  }
  for (const void* ptr : {query, key_cache, value_cache, static_cast<const void*>(out)}) {
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) {
      return fail(TPSA_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
    }
  }
  CUtensorMap tq, tk, tv;
  const uint64_t hq = static_cast<uint64_t>(kv_heads) * kGroupSize;
  st = encode_map(&tq, query, hq, static_cast<uint64_t>(query_tokens), 2, kBlockQ);
  if (st != TPSA_OK) return st;
  st = encode_map(&tk, key_cache, kv_heads, static_cast<uint64_t>(num_pages) * kPageSize, 1, 64);
  if (st != TPSA_OK) return st;
  st = encode_map(&tv, value_cache, kv_heads, static_cast<uint64_t>(num_pages) * kPageSize, 1,
                  64);
  if (st != TPSA_OK) return st;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  args.block_table = block_table;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.num_pages = static_cast<int32_t>(num_pages);
  if (p.workspace_bytes > 0) {
    args.split_ctr = static_cast<int32_t*>(workspace);
    args.scratch = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kControlBytes);
    cudaError_t e = cudaMemsetAsync(workspace, 0, kControlBytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
  }
  args.visited = visited;
  args.tiles = reinterpret_cast<unsigned long long*>(tile_counter);
  args.words_per_row = (p.seq_len + 31) / 32;

  if (visited != nullptr || tile_counter != nullptr) {
    tpsa_paged_kernel<true><<<p.grid, kNumThreads, kSmemBytes, s>>>(args, tq, tk, tv);
  } else {
    tpsa_paged_kernel<false><<<p.grid, kNumThreads, kSmemBytes, s>>>(args, tq, tk, tv);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
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
  if (sm_count <= 0) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    e = cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
  }
  return build_plan(query_tokens, query_start, seq_len, prompt_len, kv_heads, sm_count, scale,
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
