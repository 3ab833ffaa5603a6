// Work decomposition shared by the host planner and the sm_100a kernel.
//
// A query block is 64 consecutive query tokens of one request.  With GQA 4:1
// a block and one kv head give 64 tokens x 4 query heads = 256 rows, which the
// kernel runs as two M=128 tensor-core tiles (query heads {4h, 4h+1} and
// {4h+2, 4h+3}) that read the same key tiles.
//
// Key tiles are runs of 64 or 128 keys, each 64-key half inside one page.
// For each block the tiles cover exactly the union of the rows' key sets
// rounded out to 64-key granularity, so keys that no row of the block uses
// are never loaded:
//   * a block whose rows are all sparse (reference operator/op_kernel/
//     triangle_schedule.h:101-142, BuildTileSchedule "fullySparse") reads the
//     sink page prefix [0, 64) plus the local band [qBegin - 512, qEnd);
//     when the band starts inside page 0 the two are merged into one range.
//     The band is 576 keys (4.5 pages) long, so one of its ends is a 64-key
//     edge; tile 0 joins that edge with the first 16 keys of the sink page
//     into one 80-key composite tile (keys [edge, edge + 64) then [0, 16)),
//     so the block runs one 80-key tile where it would run two 64-key tiles;
//   * any other block reads the dense range [0, qEnd).
// A block straddling sparse_begin or sparse_end is not cut into spans as the
// reference does (triangle_schedule.h:74-99); it reads the dense range and
// the per-row mask gives each row its exact key set.
#ifndef TPSA_SCHEDULE_H_
#define TPSA_SCHEDULE_H_

#include <stdint.h>

#include "../../include/tpsa.h"

#if defined(__CUDACC__)
#define TPSA_HD __host__ __device__ __forceinline__
#else
#define TPSA_HD inline
#endif

namespace tpsa {

constexpr int32_t kHeadDim = TPSA_HEAD_DIM;
constexpr int32_t kPageSize = TPSA_PAGE_SIZE;
constexpr int32_t kGroupSize = TPSA_QUERY_HEADS / TPSA_KV_HEADS;  // 4
constexpr int32_t kSinkTokens = TPSA_SINK_TOKENS;
constexpr int32_t kLocalWindow = TPSA_LOCAL_WINDOW;
constexpr int32_t kDenseTail = TPSA_DENSE_TAIL;
constexpr int32_t kSparseBegin = kSinkTokens + kLocalWindow + 1;  // 521
constexpr int32_t kBlockQ = 64;        // query tokens per block
constexpr int32_t kRowsPerTile = 128;  // rows of one tensor-core M tile
constexpr int32_t kTileKeys = 128;     // widest key tile (one page)
constexpr int32_t kKeyGrain = 64;      // key tiles are multiples of this
// A composite tile: a 64-key band edge, then the first kSinkSlice keys of
// page 0 (the smallest N step of an M = 128 MMA that holds the sink).
constexpr int32_t kSinkSlice = 16;
constexpr int32_t kCompositeKeys = kKeyGrain + kSinkSlice;  // 80
static_assert(kSinkTokens <= kSinkSlice, "the sink fits the composite tile's sink slice");
constexpr int32_t kMinSplitTiles = 4;  // never split below this many tiles
constexpr int32_t kMaxSeqLen = 1 << 30;
// Partial result of one split item: 256 rows x (128 O values + m + l), fp32.
constexpr int64_t kSlotFloats = 2 * kRowsPerTile * (kHeadDim + 2);
constexpr int64_t kSlotBytes = kSlotFloats * 4;
// Workspace control words: work-item counter + split counters (int32), one
// per (dense-tail block, kv head, CTA of the pair).
constexpr int64_t kControlBytes = 2048;
constexpr int32_t kMaxSplitCounters = 448;  // (2048 - 64 * 4) / 4

TPSA_HD int32_t ceil_div(int32_t a, int32_t b) { return (a + b - 1) / b; }
TPSA_HD int32_t min_i(int32_t a, int32_t b) { return a < b ? a : b; }
TPSA_HD int32_t max_i(int32_t a, int32_t b) { return a > b ? a : b; }

struct BlockTiles {
  int32_t q_begin;    // absolute position of the block's first row
  int32_t q_end;      // one past its last real row (<= seq_len)
  int32_t sink;       // 1: tile 0 is the sink tile [0, 64); 2: tile 0 is the
                      // composite tile [edge, edge + 64) + [0, 16)
  int32_t key_begin;  // 64-aligned start of the contiguous key range
  int32_t key_end;    // 64-aligned end of the contiguous key range
  int32_t count;      // number of key tiles
  int32_t all_dense;  // every row of the block is a dense row
  int32_t edge;       // with sink == 2: first key of the band edge in tile 0
};

// Row q is sparse iff sparse_begin <= q < sparse_end (reference
// operator/tests/triangle_v2_reference.py:212-215).
TPSA_HD bool row_is_sparse(const tpsa_plan& p, int32_t q) {
  return q >= p.sparse_begin && q < p.sparse_end;
}

TPSA_HD BlockTiles block_tiles(const tpsa_plan& p, int32_t block) {
  BlockTiles t;
  t.q_begin = p.query_start + block * kBlockQ;
  t.q_end = min_i(t.q_begin + kBlockQ, p.seq_len);
  const int32_t sparse_lo = max_i(t.q_begin, p.sparse_begin);
  const int32_t sparse_hi = min_i(t.q_end, p.sparse_end);
  t.all_dense = sparse_lo >= sparse_hi ? 1 : 0;
  const bool all_sparse = t.q_begin >= p.sparse_begin && t.q_end <= p.sparse_end;
  t.key_end = ceil_div(t.q_end, kKeyGrain) * kKeyGrain;
  t.sink = 0;
  t.key_begin = 0;
  t.edge = 0;
  if (all_sparse) {
    // q_begin >= 521, so the band start q_begin - 512 is positive.
    const int32_t band = ((t.q_begin - kLocalWindow) / kKeyGrain) * kKeyGrain;
    if (band >= kTileKeys) {
      t.sink = 1;
      t.key_begin = band;
      // A band end half-way through a page becomes the lower 64 keys of
      // tile 0.
      if (t.key_begin % kTileKeys != 0) {
        t.sink = 2;
        t.edge = t.key_begin;
        t.key_begin += kKeyGrain;
      } else if (t.key_end % kTileKeys != 0) {
        t.sink = 2;
        t.edge = t.key_end - kKeyGrain;
        t.key_end -= kKeyGrain;
      }
    }
  }
  t.count = (t.sink != 0 ? 1 : 0) + ceil_div(t.key_end, kTileKeys) - t.key_begin / kTileKeys;
  return t;
}

// Tile `tile` of a block: *width keys (64, 80 or 128), the first 64 (or all
// of a 64-key tile) from *k0 on; the keys after the first 64 start at
// upper_key(t, tile, *k0): *k0 + 64 in a 128-key tile, key 0 in the 80-key
// composite tile (whose first 64 keys are the band edge).
TPSA_HD void tile_keys(const BlockTiles& t, int32_t tile, int32_t* k0,
                       int32_t* width) {
  if (t.sink != 0) {
    if (tile == 0) {
      *k0 = t.sink == 2 ? t.edge : 0;
      *width = t.sink == 2 ? kCompositeKeys : kKeyGrain;
      return;
    }
    tile -= 1;
  }
  const int32_t page0 = t.key_begin / kTileKeys;
  const int32_t start = tile == 0 ? t.key_begin : (page0 + tile) * kTileKeys;
  const int32_t end = min_i(t.key_end, (page0 + tile + 1) * kTileKeys);
  *k0 = start;
  *width = end - start;
}

TPSA_HD int32_t upper_key(const BlockTiles& t, int32_t tile, int32_t k0) {
  return (t.sink == 2 && tile == 0) ? 0 : k0 + kKeyGrain;
}

// True when some real row of the block excludes some key of the tile that
// starts at k0 and is w keys wide (the composite tile always has excluded
// keys: only keys 0-7 of its sink slice are in the sparse rows' sets).
// Conservative for blocks that mix dense and sparse rows.
TPSA_HD bool tile_needs_mask(const tpsa_plan& p, const BlockTiles& t,
                             int32_t k0, int32_t w) {
  if (w == kCompositeKeys) return true;
  if (k0 + w - 1 > t.q_begin) return true;  // causal edge of the first row
  if (t.all_dense) return false;
  const int32_t last_sparse = min_i(t.q_end, p.sparse_end) - 1;
  return k0 < last_sparse - kLocalWindow;  // window lower edge or sink gap
}


// Key k enters row q's softmax (reference triangle_v2_reference.py:193-232:
// dense rows read [0, q], sparse rows read [0, 8) U [q - 512, q]).
TPSA_HD bool key_visible(const tpsa_plan& p, int32_t q, int32_t k) {
  if (k > q || k >= p.seq_len) return false;
  if (!row_is_sparse(p, q)) return true;
  return k < kSinkTokens || k >= q - kLocalWindow;
}

TPSA_HD int32_t block_splits(const tpsa_plan& p, int32_t count) {
  return count <= p.split_tiles ? 1 : ceil_div(count, p.split_tiles);
}

// Work item `i` in launch order: first the blocks holding dense-tail rows
// (the longest items, split when long), last block first; then the remaining
// blocks from the last to the first, so cheap dense-prefix blocks run last.
TPSA_HD tpsa_item decode_item(const tpsa_plan& p, int32_t i) {
  tpsa_item it;
  if (i < p.tail_items) {
    int32_t rem = i;
    for (int32_t b = p.num_blocks - 1; b >= p.tail_block0; --b) {
      const BlockTiles bt = block_tiles(p, b);
      const int32_t ns = block_splits(p, bt.count);
      const int32_t n = ns * p.kv_heads;
      if (rem < n) {
        it.block = b;
        it.kv_head = rem / ns;
        it.split = rem % ns;
        it.num_splits = ns;
        it.tile_begin = it.split * bt.count / ns;
        it.tile_end = (it.split + 1) * bt.count / ns;
        return it;
      }
      rem -= n;
    }
  }
  const int32_t j = i - p.tail_items;
  it.block = p.tail_block0 - 1 - j / p.kv_heads;
  it.kv_head = j % p.kv_heads;
  it.split = 0;
  it.num_splits = 1;
  it.tile_begin = 0;
  it.tile_end = block_tiles(p, it.block).count;
  return it;
}

}  // namespace tpsa

#endif  // TPSA_SCHEDULE_H_
