/*
 * tpsa.h - C ABI of the B200 (sm_100a) TriangleMix paged sparse prefill
 * attention library, libtpsa.so.
 *
 * The ABI uses plain pointers, integers and POD structs only.  Every entry
 * point is host code; the compute entry points enqueue work on the caller's
 * CUDA stream (passed as `void*`, i.e. a cudaStream_t, NULL = legacy default
 * stream) and return without synchronising.
 *
 * Semantics per query row q (absolute position) of one request:
 *   sparse row  (521 <= q < prompt_len - 128): keys [0, 8) U [q - 512, q]
 *   dense row   (otherwise):                   keys [0, min(q + 1, seq_len))
 * All keys of a row share one softmax; output is bf16.
 *
 * Reference interfaces replaced (paths are inside the reference project):
 *   operator/torch_adapter/triangle_paged_attention_torch.cpp:101-178
 *       triangle_paged_sparse_attention[_out]  -> tpsa_paged_attention
 *   operator/torch_adapter/triangle_paged_attention_torch.cpp:180-261
 *       triangle_paged_sparse_attention_workspace_size -> tpsa_workspace_size
 *   operator/op_host/triangle_paged_sparse_attention.cpp:122-327
 *       optiling::TilingFunc (shape gate + task geometry) -> tpsa_make_plan
 *   operator/op_kernel/triangle_schedule.h:74-142
 *       SplitQueryTile / BuildTileSchedule -> tpsa_plan_item / tpsa_plan_tile
 */
#ifndef TPSA_H_
#define TPSA_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TPSA_API __attribute__((visibility("default")))
#else
#define TPSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* 3: tpsa_plan_tile reports the 80-key composite tile (band edge, then
 * the sink slice [0, 16)); 2 reported a 128-key one (sink prefix, then the
 * band edge). */
#define TPSA_ABI_VERSION 3

/* Fixed geometry (reference operator/op_kernel/triangle_schedule.h:14-21). */
#define TPSA_QUERY_HEADS 32
#define TPSA_KV_HEADS 8
#define TPSA_HEAD_DIM 128
#define TPSA_PAGE_SIZE 128
#define TPSA_SINK_TOKENS 8
#define TPSA_LOCAL_WINDOW 512
#define TPSA_DENSE_TAIL 128
#define TPSA_QUERY_TILE 32 /* reference attribute value; accepted, not used */

typedef enum tpsa_status {
  TPSA_OK = 0,
  TPSA_ERR_INVALID_ARGUMENT = 1, /* a shape / attribute gate failed      */
  TPSA_ERR_WORKSPACE = 2,        /* workspace missing or too small        */
  TPSA_ERR_CUDA = 3,             /* a CUDA runtime or driver call failed  */
  TPSA_ERR_UNSUPPORTED_DEVICE = 4, /* current device is not sm_100       */
  TPSA_ERR_DEVICE_FAULT = 5,     /* the device status word is non-zero    */
} tpsa_status;

/* Device status word bits (tpsa_device_status). */
#define TPSA_DEVICE_WAIT_TIMEOUT 0x1u /* a pipeline wait hit its bound      */
#define TPSA_DEVICE_BAD_PAGE 0x2u     /* block_table held an out-of-range page */

/*
 * Launch plan: how one call is cut into work items.  A work item is
 * (64-token query block, kv head, key-tile range); dense-tail blocks with many
 * key tiles are split into several items whose partial results are merged
 * inside the same launch.  Computed on the host by tpsa_make_plan.
 */
typedef struct tpsa_plan {
  int32_t query_tokens;  /* Tq                                         */
  int32_t query_start;   /* absolute position of query row 0           */
  int32_t seq_len;       /* query_start + Tq                           */
  int32_t sparse_begin;  /* 521                                        */
  int32_t sparse_end;    /* min(max(0, prompt_len - 128), seq_len)     */
  int32_t kv_heads;      /* kv heads held by this cache / call         */
  int32_t num_blocks;    /* ceil(Tq / 64)                              */
  int32_t tail_block0;   /* first block holding a dense-tail row       */
  int32_t tail_items;    /* items of blocks [tail_block0, num_blocks)  */
  int32_t total_items;   /* all work items                             */
  int32_t split_tiles;   /* max key tiles per item for tail blocks     */
  int32_t grid;          /* persistent CTAs launched                   */
  int64_t workspace_bytes; /* scratch needed by tpsa_paged_attention   */
  int64_t total_tiles;   /* key tiles summed over all items            */
  float scale;           /* softmax scale                              */
  float scale_log2;      /* scale * log2(e)                            */
} tpsa_plan;

typedef struct tpsa_item {
  int32_t block;      /* query block index (rows 64*block ...)      */
  int32_t kv_head;    /* kv head (query heads 4*kv_head .. +3)      */
  int32_t split;      /* split index within the block               */
  int32_t num_splits; /* number of items the block's keys are cut into */
  int32_t tile_begin; /* first key tile of this item (block-local)   */
  int32_t tile_end;   /* one past the last key tile                  */
} tpsa_item;

/* ABI version of the loaded library (TPSA_ABI_VERSION at build time). */
TPSA_API int32_t tpsa_abi_version(void);

/* Static description of a status code. */
TPSA_API const char* tpsa_status_string(tpsa_status status);

/* Message of the last failed host-side check on this thread ("" if none). */
TPSA_API const char* tpsa_last_error(void);

/*
 * Validate the scalar attributes and build the launch plan.  `sm_count` <= 0
 * means "query the current device".  Mirrors the reference TilingFunc gates
 * (operator/op_host/triangle_paged_sparse_attention.cpp:192-238):
 * query_start >= 0, seq_len > 0, prompt_len >= seq_len,
 * query_start + query_tokens == seq_len, scale finite and > 0.
 */
TPSA_API tpsa_status tpsa_make_plan(int64_t query_tokens, int64_t query_start,
                           int64_t seq_len, int64_t prompt_len,
                           int32_t kv_heads, int32_t sm_count, float scale,
                           tpsa_plan* plan);

/* Work item `item` (0 <= item < plan->total_items), in launch order. */
TPSA_API tpsa_status tpsa_plan_item(const tpsa_plan* plan, int32_t item,
                           tpsa_item* out);

/*
 * Key tile `tile` of query block `block`: *key_count keys (64, 80 or 128).
 * The first 64 (all of a 64-key tile) are [*key_begin, *key_begin + 64); the
 * rest follow from *upper_begin on: keys 64-127 of a 128-key tile are
 * [*key_begin + 64, *key_begin + 128), and the 80-key composite tile of a
 * sparse block (tile 0) is the band's 64-key edge followed by the sink
 * slice [0, 16) (*upper_begin = 0).  No 64-key half crosses a page.
 * *needs_mask is 1 when some row of the block excludes some key of the tile
 * (causal / window / sink boundary; always for the composite tile).
 */
TPSA_API tpsa_status tpsa_plan_tile(const tpsa_plan* plan, int32_t block, int32_t tile,
                           int32_t* key_begin, int32_t* key_count,
                           int32_t* upper_begin, int32_t* needs_mask);

/*
 * Scratch bytes tpsa_paged_attention needs on the current device for these
 * attributes: 2 KiB of scheduler control words, plus the partial results of
 * split dense-tail blocks when the plan splits any.  Replaces
 * triangle_paged_sparse_attention_workspace_size (reference
 * operator/torch_adapter/triangle_paged_attention_torch.cpp:180-261).
 */
TPSA_API tpsa_status tpsa_workspace_size(int64_t query_tokens, int64_t query_start,
                                int64_t seq_len, int64_t prompt_len,
                                uint64_t* bytes);

/*
 * TriangleMix paged sparse prefill attention, one request, one launch.
 * Replaces aclnnTrianglePagedSparseAttention behind the reference's
 * triangle_paged_sparse_attention[.out] (reference
 * operator/torch_adapter/triangle_paged_attention_torch.cpp:101-178).
 *
 *   query        bf16 [query_tokens, 32, 128], contiguous, device memory
 *   key_cache    bf16 [num_pages, 128, 8, 128] (BSND pages), contiguous
 *   value_cache  bf16, same shape as key_cache
 *   block_table  int32 [1, table_cols]; logical page -> physical page
 *   out          bf16 [query_tokens, 32, 128], caller-owned, not aliasing
 *                any input; written in place
 *   workspace    device scratch of at least tpsa_workspace_size() bytes,
 *                256-byte aligned, never NULL.  Its contents need not be
 *                initialised.  Calls sharing one workspace must be ordered
 *                on one stream.
 *   stream       cudaStream_t
 *
 * Control words (the work-item counter and the split-KV counters, which
 * start every launch at zero) live in a library-owned 4 KiB block per
 * stream, one of 128 per device in a module-global array: the first call on
 * a stream clears its block with cudaMemsetAsync on that stream, and the
 * last CTA of every launch zeroes it again before it exits, so later calls
 * issue only the kernel.  Streams are told apart by cudaStreamGetId.  While
 * `stream` is being captured into a CUDA graph, or once 128 streams of a
 * device hold blocks, a call keeps its control words in the first 2 KiB of
 * `workspace` instead and clears them with cudaMemsetAsync before the
 * kernel (a captured graph then carries that memset and may be replayed on
 * any stream).  The block addresses are looked up once per device; after
 * cudaDeviceReset in the same process they are stale.
 *
 * Gates (reference op_host :133-238): table_cols >= ceil(seq_len / 128),
 * num_pages > 0, query_start + query_tokens == seq_len, prompt_len >= seq_len,
 * seq_len <= 2^30.  Physical page ids are checked on the device: an id
 * outside [0, num_pages) reads zeros and sets TPSA_DEVICE_BAD_PAGE.
 * Returns without synchronising; no device memory is allocated.
 */
TPSA_API tpsa_status tpsa_paged_attention(const void* query, const void* key_cache,
                                 const void* value_cache,
                                 const int32_t* block_table, void* out,
                                 int64_t query_tokens, int64_t num_pages,
                                 int64_t table_cols, int64_t query_start,
                                 int64_t seq_len, int64_t prompt_len,
                                 float scale, void* workspace,
                                 uint64_t workspace_bytes, void* stream);

/*
 * Same computation for a head-sharded cache: this call owns `kv_heads`
 * (1, 2, 4 or 8) kv heads and the 4 * kv_heads query heads that read them,
 * i.e. query [Tq, 4*kv_heads, 128] and caches [num_pages, 128, kv_heads,
 * 128].  Used by the 1/2/4/8-GPU KV-head partition; no reference
 * counterpart (the reference forces tensor-parallel callers to fall back,
 * package/src/vllm_ascend_trianglemix/plugin.py:1251-1253).
 */
TPSA_API tpsa_status tpsa_paged_attention_heads(
    const void* query, const void* key_cache, const void* value_cache,
    const int32_t* block_table, void* out, int64_t query_tokens,
    int64_t num_pages, int64_t table_cols, int64_t query_start,
    int64_t seq_len, int64_t prompt_len, float scale, int32_t kv_heads,
    void* workspace, uint64_t workspace_bytes, void* stream);

/*
 * All-dense control: the same kernel and launch with no sparse rows, i.e.
 * plain causal attention of the chunk over its whole paged context (row
 * query_start + i reads keys [0, query_start + i]).  This is the dense
 * comparator of the chunked-prefill crossover and of all-dense timing runs;
 * no reference counterpart (the reference's dense path is the stock paged
 * attention).  Arguments and gates are tpsa_paged_attention's without
 * prompt_len; the workspace size comes from tpsa_dense_workspace_size.
 */
TPSA_API tpsa_status tpsa_dense_workspace_size(int64_t query_tokens, int64_t query_start,
                                      int64_t seq_len, uint64_t* bytes);

TPSA_API tpsa_status tpsa_paged_attention_dense(
    const void* query, const void* key_cache, const void* value_cache,
    const int32_t* block_table, void* out, int64_t query_tokens,
    int64_t num_pages, int64_t table_cols, int64_t query_start,
    int64_t seq_len, float scale, void* workspace, uint64_t workspace_bytes,
    void* stream);

/*
 * Packed ragged batch (varlen): `batch` requests whose query rows are packed
 * back to back, each computed exactly as one tpsa_paged_attention call on
 * its own rows.  Same semantics as the reference's packed-batch helper
 * reference_attention_ragged_python (operator/tests/triangle_v2_reference.py:
 * 437-487), which the reference computes by calling the batch-one op once
 * per request; the reference op itself rejects batch > 1 (op_host :151-157,
 * planning.py:149-150).  Here the whole batch shares one persistent launch
 * per 16 requests, so short requests fill the GPU together.
 *
 *   query         bf16 [cu_seqlens_q[batch], 32, 128], packed
 *   out           bf16, same shape as query
 *   key_cache,
 *   value_cache   bf16 [num_pages, 128, 8, 128], one page pool for all requests
 *   block_tables  int32 [batch, table_cols] (device): row i maps request i's
 *                 logical pages to physical pages
 *   cu_seqlens_q  int64 [batch + 1] (host): request i owns packed rows
 *                 [cu_seqlens_q[i], cu_seqlens_q[i+1]); cu_seqlens_q[0] == 0
 *   seq_lens      int64 [batch] (host): request i's query rows are the last
 *                 rows of its first seq_lens[i] tokens (query_start =
 *                 seq_lens[i] - rows)
 *   prompt_lens   int64 [batch] (host): prompt_lens[i] >= seq_lens[i]
 *   workspace     at least tpsa_varlen_workspace_size() bytes, 256-byte
 *                 aligned; reused by the launches of one call in stream order
 *
 * Every row count must be positive (reference: "each ragged query length must
 * be positive").  The other gates are tpsa_paged_attention's, per request.
 */
TPSA_API tpsa_status tpsa_varlen_workspace_size(int32_t batch, const int64_t* cu_seqlens_q,
                                       const int64_t* seq_lens,
                                       const int64_t* prompt_lens, uint64_t* bytes);

TPSA_API tpsa_status tpsa_paged_attention_varlen(
    const void* query, const void* key_cache, const void* value_cache,
    const int32_t* block_tables, void* out, int32_t batch,
    const int64_t* cu_seqlens_q, const int64_t* seq_lens,
    const int64_t* prompt_lens, int64_t num_pages, int64_t table_cols,
    float scale, void* workspace, uint64_t workspace_bytes, void* stream);

/*
 * Head-slice forms of the two entries above, for one rank of a KV-head
 * partition (the multi-GPU layout of tpsa_paged_attention_heads): query and
 * out are [rows, 4*kv_heads, 128], the caches [num_pages, 128, kv_heads,
 * 128], kv_heads in {1, 2, 4, 8}.  A rank that holds its head slice of
 * several layers in one page pool (each layer's block table pointing at its
 * own pages) runs them all as the requests of one launch, which keeps the
 * launch as large as a full 8-head layer.  No counterpart in the reference,
 * which has no multi-device path (it falls back for tensor-parallel shards,
 * package/src/vllm_ascend_trianglemix/planning.py:14-39).
 */
TPSA_API tpsa_status tpsa_varlen_workspace_size_heads(int32_t batch, const int64_t* cu_seqlens_q,
                                                      const int64_t* seq_lens,
                                                      const int64_t* prompt_lens,
                                                      int32_t kv_heads, uint64_t* bytes);

TPSA_API tpsa_status tpsa_paged_attention_varlen_heads(
    const void* query, const void* key_cache, const void* value_cache,
    const int32_t* block_tables, void* out, int32_t batch,
    const int64_t* cu_seqlens_q, const int64_t* seq_lens,
    const int64_t* prompt_lens, int64_t num_pages, int64_t table_cols,
    float scale, int32_t kv_heads, void* workspace, uint64_t workspace_bytes, void* stream);

/*
 * Debug variant that runs the identical kernel and additionally records,
 * for every (query row, query head), the key indices that entered its
 * softmax: bit k of visited[(row * 4*kv_heads + head) * words_per_row +
 * k / 32], words_per_row = ceil(seq_len / 32).  `visited` must be zeroed by
 * the caller; `tile_counter` (2 x uint64, zeroed by the caller) receives the
 * number of key tiles and of keys loaded.  Test infrastructure for the
 * visited-key-set contract; not a production entry point.
 */
TPSA_API tpsa_status tpsa_paged_attention_visit(
    const void* query, const void* key_cache, const void* value_cache,
    const int32_t* block_table, void* out, int64_t query_tokens,
    int64_t num_pages, int64_t table_cols, int64_t query_start,
    int64_t seq_len, int64_t prompt_len, float scale, int32_t kv_heads,
    void* workspace, uint64_t workspace_bytes, uint32_t* visited,
    uint64_t* tile_counter, void* stream);

/*
 * tpsa_paged_attention without a workspace argument: it allocates nothing.
 * This entry point has no counterpart in the reference.
 *
 * Some callers cannot allocate device memory at the moment they run the
 * operator: plain C or FFI hosts that bind this library without an
 * allocator of their own, and serving runtimes that reserve all device memory
 * up front, where an allocation in the middle of a step could fail or
 * fragment the pool.  This variant keeps its scratch (the control words and
 * the split-KV partials) in one module-global device array of at most
 * 24 MiB per device.  That covers every plan on a 148-SM B200 (at most
 * 18.3 MiB, for query chunks of 64 to 16384 rows over contexts up to 4M
 * tokens).  A call whose plan needs more scratch returns
 * TPSA_ERR_WORKSPACE with the required size in tpsa_last_error(); use
 * tpsa_paged_attention with a caller workspace for those shapes.  The call
 * makes no cudaMalloc or cudaFree and uses no allocating library routine.
 *
 * Set-up: every call looks up the array's device address on the current
 * device with cudaGetSymbolAddress; the library keeps no address between
 * calls.  The first lookup on a device also makes the CUDA runtime load the
 * library's device globals there: make the first call on each device before
 * any stream capture.
 *
 * Sharing: every call on a device uses the same array, and the array keeps
 * the previous call's contents.  Each call clears the control words that
 * must start at zero (cudaMemsetAsync on `stream`).  The partial slots are
 * written before they are read.  Calls that overlap on the GPU (launched on
 * different streams without ordering, or from several host threads at once)
 * race on the array and give wrong results, so order them on one stream.
 *
 * Arguments, gates and results are those of tpsa_paged_attention.
 */
TPSA_API tpsa_status tpsa_paged_attention_static_scratch(
    const void* query, const void* key_cache, const void* value_cache,
    const int32_t* block_table, void* out, int64_t query_tokens,
    int64_t num_pages, int64_t table_cols, int64_t query_start,
    int64_t seq_len, int64_t prompt_len, float scale, void* stream);

/*
 * Read and clear the device status word of `device` (TPSA_DEVICE_* bits).
 * Synchronises that device.  A non-zero word means a launch since the last
 * read hit a bounded wait or an out-of-range page id.
 */
TPSA_API tpsa_status tpsa_device_status(int32_t device, uint32_t* status_bits);

/*
 * Test hook for the bounded waits (no reference counterpart).  The next
 * single-request launch on the calling thread (tpsa_paged_attention and its
 * _heads / _visit / _static_scratch forms) runs in probe mode: in every CTA
 * the scheduler waits on a barrier that nothing arrives on, with a limit of
 * `limit_ns` instead of 1 s, before it claims any work.  The wait runs out,
 * the kernel records TPSA_DEVICE_WAIT_TIMEOUT and every role leaves through
 * its abort path; no load, MMA or output store is issued, so `out` keeps its
 * contents.  The launch itself returns TPSA_OK; tpsa_device_status reports
 * the bit.  limit_ns: 0 disarms, else 1000 (1 us) to 100000000 (100 ms).
 */
TPSA_API tpsa_status tpsa_debug_wait_probe(uint32_t limit_ns);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* TPSA_H_ */
