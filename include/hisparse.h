/*
 * hisparse.h — C ABI of libhisparse.so, the sm_100a (B200) implementation of
 * nano-hisparse's per-step sparse-decode hot path.
 *
 * The library replaces four reference operators with CUDA kernels:
 *   (1) Quest page scoring + shared top-k + page->token expansion
 *       (nano_hisparse/selection.py:69-91 and row_index.py:20-24)
 *   (2) the row resolver (nano_hisparse/row_index.py:62-140)
 *   (3) the host->pool miss gather (nano_hisparse/row_kernels.py:35-70)
 *   (4) physical-row GQA decode attention (nano_hisparse/row_kernels.py:73-135,
 *       attention.py:26-35)
 * plus the mapped-host alias query (nano_hisparse/row_kernels.py:10-32) and
 * the KV append that feeds (1): pool rows, host mirror and page metadata
 * (nano_hisparse/storage.py:296-321).
 *
 * Conventions shared by every entry point:
 *   - Pointers are borrowed. The caller owns every buffer; the library never
 *     allocates device or host memory. Kernels that need scratch take a
 *     caller-provided `workspace`, sized by the matching *_workspace_bytes().
 *   - Device pointers (tensors) live on the device current at call time.
 *     `stream` is a cudaStream_t (NULL = legacy default stream). All work is
 *     enqueued asynchronously; no entry point synchronises the host, so the
 *     resolver and gather can be captured in a CUDA graph.
 *   - Every function returns an hs_status. Host-side argument errors are
 *     reported before anything is enqueued; hs_last_error() gives a message.
 *   - `device_status` (optional, may be NULL) is a device int32 word into
 *     which kernels OR the HS_DEV_* bits below when they meet and skip an
 *     out-of-range index. Kernels never trap: a bad index is skipped and
 *     recorded, never dereferenced.
 *   - "Batched" entry points process `batch` independent requests of one
 *     layer in a single launch. Per-request tables that the caller allocates
 *     separately are passed as device arrays of `batch` 64-bit pointers.
 *
 * Memory layouts (all row-major, identical to the reference):
 *   pool   [pool_blocks, 2 (K|V), page_size, kv_heads, head_dim]  (allocator.py:18-22)
 *   host   [host_blocks, 2 (K|V), page_size, kv_heads, head_dim]  (storage.py:126-128)
 *   min/max metadata [pages, kv_heads, head_dim] in the KV dtype  (storage.py:215-219)
 *   query  [q_heads, head_dim]
 *   A physical row r addresses block r / page_size, offset r % page_size.
 */
#ifndef HISPARSE_H
#define HISPARSE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HS_ABI_VERSION 1

#if defined(__GNUC__)
#define HS_API __attribute__((visibility("default")))
#else
#define HS_API
#endif

/* Return codes. */
enum hs_status {
  HS_OK = 0,
  HS_ERR_INVALID_ARGUMENT = 1, /* a size, shape, pointer or dtype is invalid */
  HS_ERR_UNSUPPORTED = 2,      /* valid but not implemented (e.g. head_dim > 256) */
  HS_ERR_WORKSPACE = 3,        /* workspace missing or smaller than *_workspace_bytes() */
  HS_ERR_CUDA = 4,             /* a CUDA runtime call or launch failed */
  HS_ERR_NOT_MAPPED = 5        /* host memory is not page-locked/mapped for the device */
};

/* Element types of query / KV / metadata tensors. */
enum hs_dtype { HS_FLOAT32 = 0, HS_FLOAT16 = 1, HS_BFLOAT16 = 2, HS_INT32 = 3, HS_INT64 = 4 };

/* Bits written (atomicOr) into *device_status by kernels. */
enum hs_device_flag {
  HS_DEV_ROW_OUT_OF_RANGE = 1,   /* a physical/host row beyond its buffer was skipped */
  HS_DEV_PAGES_EXCEED_TABLE = 2, /* ceil(length / page_size) exceeded the table capacity */
  HS_DEV_LRU_CORRUPT = 4,        /* an LRU entry outside [0, hot_rows) was skipped */
  HS_DEV_MISSES_EXCEED_HOT = 8,  /* more misses than hot rows: tags/lru left unchanged */
  HS_DEV_WAIT_TIMEOUT = 16,      /* a bounded wait for an async copy ran out (results invalid) */
  HS_DEV_MISALIGNED = 32         /* a batched metadata pointer was not 16-byte aligned: skipped */
};

typedef void *hs_stream; /* cudaStream_t */

/* ---- library information ------------------------------------------------ */

/* HS_ABI_VERSION of the loaded library. */
HS_API int hs_version(void);

/* Static description of a status code. */
HS_API const char *hs_status_string(int status);

/* Message describing the last error returned on the calling host thread. */
HS_API const char *hs_last_error(void);

/* ---- mapped host alias ---------------------------------------------------
 * Replaces MappedHost (nano_hisparse/row_kernels.py:10-32): returns the
 * device-side alias of page-locked host memory that the caller (e.g. the
 * PyTorch pinned allocator) already owns. Nothing is registered or
 * unregistered. HS_ERR_NOT_MAPPED if `host` is not page-locked memory.
 */
HS_API int hs_host_device_pointer(const void *host, void **device_alias);

/* ---- (1) Quest page selection --------------------------------------------
 * Replaces quest_selection (nano_hisparse/selection.py:69-91) followed by
 * Selection.from_pages (selection.py:45-62) and LogicalTopK.from_selection
 * (row_index.py:20-24) for the shared-selection case.
 *
 * For pages p < n = ceil(length / page_size):
 *   s[h,p]  = sum_d max(q[h,d]*min[p,h/g,d], q[h,d]*max[p,h/g,d])   (fp32)
 *   score_p = (sum_h s[h,p]) / q_heads
 * The tail page n-1 and, when keep_sink && top_pages > 1 && n > 1, page 0
 * are forced to +inf; the top_pages highest scores are kept (equal scores:
 * lower page first). The chosen pages are expanded to their tokens in
 * ascending order, the tail page clipped at `length`. If top_pages >= n all
 * `length` tokens are selected. out_tokens receives the tokens followed by
 * -1 padding up to out_capacity (>= top_pages * page_size);
 * out_count receives the number of tokens.
 * The fp32 summation order is fixed, so scores are reproducible bit for bit:
 * with L = the smallest power of two >= ceil(head_dim / 8), lane j in [0, L)
 * owns d = 8j .. 8j+7 (d < head_dim); it adds the terms at even offsets
 * (d = 8j, 8j+2, ...) left to right and those at odd offsets left to right,
 * then even + odd; the L lane values are combined pairwise as
 * (j, j^(L/2)), (j, j^(L/4)), ..., (j, j^1). The head sums are then combined
 * with 32 lanes: lane j adds heads j, j+32, ... left to right, the 32 lane
 * values meet in the xor tree (j, j^16), ..., (j, j^1), and the total is
 * divided by q_heads.
 */
/* Workspace: per-request scores plus one completion counter per request. The
 * counters must be zero before the first use (zero-fill the whole workspace
 * once); every call overwrites the scores and leaves the counters zero, so
 * one workspace serves consecutive calls on one stream (calls that overlap on
 * the GPU need separate workspaces). */
HS_API size_t hs_quest_workspace_bytes(int batch, int64_t max_pages);

HS_API int hs_quest_select(const void *query, int query_dtype, const void *minimum,
                    const void *maximum, int kv_dtype, int q_heads, int kv_heads,
                    int head_dim, int64_t max_pages, int64_t length, int page_size,
                    int top_pages, int keep_sink, int32_t *out_tokens,
                    int64_t out_capacity, int32_t *out_count, void *workspace,
                    size_t workspace_bytes, int32_t *device_status, hs_stream stream);

/* Batched over `batch` requests of one layer. query is [batch, q_heads,
 * head_dim] with `query_batch_stride` elements between requests;
 * minimum_ptrs/maximum_ptrs are device arrays of `batch` pointers to each
 * request's [pages, kv_heads, head_dim] metadata (pages >= ceil(length / page_size) of
 * that request; max_pages >= every request's pages), each 16-byte aligned
 * (bulk copies read them; a misaligned request raises HS_DEV_MISALIGNED and
 * is skipped); lengths is a device int32[batch]. out_tokens is
 * [batch, out_capacity], out_counts int32[batch]. */
HS_API int hs_quest_select_batched(int batch, const void *query, int64_t query_batch_stride,
                            int query_dtype, const uint64_t *minimum_ptrs,
                            const uint64_t *maximum_ptrs, int kv_dtype,
                            const int32_t *lengths, int q_heads, int kv_heads,
                            int head_dim, int64_t max_pages, int page_size,
                            int top_pages, int keep_sink, int32_t *out_tokens,
                            int64_t out_capacity, int32_t *out_counts, void *workspace,
                            size_t workspace_bytes, int32_t *device_status,
                            hs_stream stream);

/* Head-sharded selection (configuration 5: one long request whose KV heads
 * are split over ranks). Replaces quest_selection (selection.py:69-91) when
 * each rank holds a slice of the heads: every rank runs
 * hs_quest_partial_scores_batched on its slice, the ranks exchange the
 * [batch, max_pages] partials (an all-gather), and every rank runs
 * hs_quest_select_partials on all of them, which yields the same tokens on
 * every rank.
 *
 * hs_quest_partial_scores_batched: arguments as hs_quest_select_batched for
 * this rank's q_heads / kv_heads; out_partial [batch, max_pages] fp32
 * receives, for pages p < ceil(length / page_size), the head sum of this
 * slice in the fixed order above (the xor tree over lanes of the per-lane
 * head sums, local head indices) WITHOUT the division by q_heads. Pages past
 * a request's length are not written. Needs no workspace. */
HS_API int hs_quest_partial_scores_batched(int batch, const void *query,
                                           int64_t query_batch_stride, int query_dtype,
                                           const uint64_t *minimum_ptrs,
                                           const uint64_t *maximum_ptrs, int kv_dtype,
                                           const int32_t *lengths, int q_heads, int kv_heads,
                                           int head_dim, int64_t max_pages, int page_size,
                                           float *out_partial, int32_t *device_status,
                                           hs_stream stream);

/* partials: [shards, batch, max_pages] fp32 (shard-major, as an all-gather
 * leaves them). score_p = (((0 + partial[0][b][p]) + partial[1][b][p]) + ...)
 * / q_heads (q_heads = the query heads of all shards), then the forced pages,
 * top-k and expansion of hs_quest_select. With shards = 1 the tokens equal
 * hs_quest_select's. Workspace: hs_quest_workspace_bytes(batch, max_pages),
 * no initialisation needed. */
HS_API int hs_quest_select_partials(int shards, const float *partials, int batch,
                                    const int32_t *lengths, int q_heads, int64_t max_pages,
                                    int page_size, int top_pages, int keep_sink,
                                    int32_t *out_tokens, int64_t out_capacity,
                                    int32_t *out_counts, void *workspace,
                                    size_t workspace_bytes, int32_t *device_status,
                                    hs_stream stream);

/* ---- (2) row resolver ------------------------------------------------------
 * Replaces resolve_rows (nano_hisparse/row_index.py:62-140) with identical
 * results: physical rows in input order (duplicates after their first
 * occurrence, negative and non-causal inputs -> -1), the compact miss plan in
 * sorted logical order (-1 padded to `count`), counts = {resident hits, hot
 * hits, misses}, and the in-place update of `tags` and `lru`.
 * Tables use the reference cache's dtypes: source/resident/hot/tags int32,
 * lru int64 (a permutation of [0, hot_rows)). positions are int32 or int64.
 * Optional legacy per-head columns (row_index.py:132-136): when head_columns
 * ([head_count, head_width] int64) is non-NULL, out_head_physical receives
 * physical[column] (or -1 for columns outside [0, count)).
 */
HS_API size_t hs_resolve_workspace_bytes(int batch, int64_t count, int64_t hot_rows);

HS_API int hs_resolve_rows(const void *positions, int positions_dtype, int64_t count,
                    const int32_t *source_table, const int32_t *resident_table,
                    int64_t table_pages, const int32_t *hot_table, int64_t hot_blocks,
                    int32_t *tags, int64_t *lru, int64_t hot_rows, int64_t length,
                    int page_size, int64_t *out_physical, int64_t *out_miss_host,
                    int64_t *out_miss_device, int64_t *out_counts,
                    const int64_t *head_columns, int64_t head_count, int64_t head_width,
                    int64_t *out_head_physical, void *workspace, size_t workspace_bytes,
                    int32_t *device_status, hs_stream stream);

/* Batched: positions int32 [batch, count]; per-request tables as device
 * pointer arrays; lengths device int32[batch]; outputs [batch, count] and
 * out_counts [batch, 3]. Each request's source/resident tables cover its own
 * ceil(length / page_size) pages; table_pages bounds every request's pages.
 * out_ready (optional, [batch, count]) receives
 * the physical rows that need no gather (resident and hot hits), compact in
 * sorted logical order and -1 padded: out_counts[b][0] + out_counts[b][1] of
 * them; with miss_device (out_counts[b][2] rows) it lets attention over the
 * ready rows run while the misses are gathered. */
HS_API int hs_resolve_rows_batched(int batch, const int32_t *positions, int64_t count,
                            const uint64_t *source_ptrs, const uint64_t *resident_ptrs,
                            int64_t table_pages, const uint64_t *hot_ptrs,
                            int64_t hot_blocks, const uint64_t *tags_ptrs,
                            const uint64_t *lru_ptrs, int64_t hot_rows,
                            const int32_t *lengths, int page_size, int64_t *out_physical,
                            int64_t *out_miss_host, int64_t *out_miss_device,
                            int64_t *out_counts, int64_t *out_ready, void *workspace,
                            size_t workspace_bytes, int32_t *device_status,
                            hs_stream stream);

/* ---- (3) miss gather --------------------------------------------------------
 * Replaces gather_rows (nano_hisparse/row_kernels.py:35-70): for every i with
 * miss_host[i] >= 0 and miss_device[i] >= 0 copies the K-plane and V-plane
 * rows (row_bytes = kv_heads * head_dim * element size, each) from the
 * mapped host store to the pool. The plans are `count` entries, organised as
 * segments of `segment` entries whose -1 entries form a suffix (the
 * resolver's compact prefix); segment = count for a single request.
 * host_alias is the device alias from hs_host_device_pointer().
 */
HS_API int hs_gather_rows(const void *host_alias, int64_t host_blocks, void *pool,
                   int64_t pool_blocks, const int64_t *miss_host,
                   const int64_t *miss_device, int64_t count, int64_t segment,
                   int page_size, int64_t row_bytes, int32_t *device_status,
                   hs_stream stream);

/* ---- (4) physical-row attention ---------------------------------------------
 * Replaces attend_rows (nano_hisparse/row_kernels.py:116-135) and the torch
 * path of row_attention (attention.py:26-35): for every batch item b and
 * query head h,
 *   out[b,h] = softmax_r(q[b,h] . K[r, h/g] / sqrt(head_dim)) V[r, h/g]
 * over the rows r = rows[b*rows_batch_stride + h*rows_head_stride + i] >= 0
 * (i < count), in fp32; zero when no row is valid. rows_head_stride = 0 for
 * the shared selection. out has the query dtype and layout [batch, q_heads,
 * head_dim] with out_batch_stride elements between batch items.
 */
HS_API size_t hs_attend_workspace_bytes(int batch, int q_heads, int kv_heads, int head_dim,
                                 int64_t count);

HS_API int hs_attend_rows(int batch, const void *query, int64_t query_batch_stride,
                   int query_dtype, const void *pool, int64_t pool_blocks, int kv_dtype,
                   const int64_t *rows, int64_t rows_batch_stride,
                   int64_t rows_head_stride, int64_t count, void *out,
                   int64_t out_batch_stride, int q_heads, int kv_heads, int head_dim,
                   int page_size, void *workspace, size_t workspace_bytes,
                   int32_t *device_status, hs_stream stream);

/* Two-phase form, for overlapping attention with the miss gather. A phase
 * launch attends over the leading valid rows of `rows` ([batch, count],
 * shared by all heads of a request) and leaves (max, sum, O) partials in the
 * workspace under `phase` (0 or 1); hs_attend_merge combines phases 0..phases-1
 * into `out`. The valid rows of batch item b are its first
 * sum(valid_counts[b*counts_stride + counts_first + i], i < counts_n) entries
 * (all `count` when valid_counts is NULL) — e.g. the resolver's counts select
 * the ready list (components 0-1) and the miss plan (component 2). Both calls
 * use the workspace sized by hs_attend_workspace_bytes for the same arguments
 * and must run in stream order. */
HS_API int hs_attend_rows_phase(int batch, const void *query, int64_t query_batch_stride,
                                int query_dtype, const void *pool, int64_t pool_blocks,
                                int kv_dtype, const int64_t *rows, int64_t rows_batch_stride,
                                int64_t count, const int64_t *valid_counts, int counts_stride,
                                int counts_first, int counts_n, int phase, int q_heads,
                                int kv_heads, int head_dim, int page_size, void *workspace,
                                size_t workspace_bytes, int32_t *device_status,
                                hs_stream stream);

HS_API int hs_attend_merge(int batch, int phases, void *out, int64_t out_batch_stride,
                           int query_dtype, int q_heads, int kv_heads, int head_dim,
                           int64_t count, void *workspace, size_t workspace_bytes,
                           int32_t *device_status, hs_stream stream);

/* ---- (5) KV append: pool rows, host mirror, page metadata ---------------------
 * Replaces the tensor work of HostStore.append (nano_hisparse/storage.py:
 * 296-321) for one page chunk per batch item b with count[b] > 0:
 *   rows within[b] .. within[b]+count[b]-1 of the K and V planes of pool block
 *   pool_block[b] take rows 0 .. count[b]-1 of k and v (batch item b starts
 *   kv_batch_stride elements after b-1; a row is kv_heads*head_dim elements);
 *   when host_block[b] >= 0 the same rows of host block host_block[b] (through
 *   host_alias, the hs_host_device_pointer alias) take the same values — the
 *   host mirror, written by the kernel itself. pool_block[b] < 0 makes the
 *   chunk host-only (a page that holds no pool block): it then needs a
 *   host block, and its earlier rows for the summary are read there;
 *   minimum_ptrs[b] / maximum_ptrs[b] point to the page's [kv_heads, head_dim]
 *   bounds in the KV dtype: min/max of the new K rows folded in exactly as
 *   torch.minimum(old, new) / torch.maximum(old, new) (NaN propagates, an equal
 *   new value replaces the old);
 *   summary_ptrs[b] points to the page's fp32 [kv_heads, head_dim] mean-K
 *   summary: the K rows 0 .. within[b]+count[b]-1 of the block added in row
 *   order in fp32, then divided by their number (bit-identical to the
 *   reference's CPU mean).
 * within/count are device int32[batch]; pool_block/host_block device
 * int64[batch]; the pointer arrays device uint64[batch]. A chunk that leaves
 * its page or addresses a block out of range is skipped and raises
 * HS_DEV_ROW_OUT_OF_RANGE. Chunks of one launch must touch distinct pages. */
HS_API int hs_append_rows(int batch, const void *k, const void *v, int64_t kv_batch_stride,
                          int kv_dtype, const int32_t *within, const int32_t *count,
                          const int64_t *pool_block, void *pool, int64_t pool_blocks,
                          const int64_t *host_block, void *host_alias, int64_t host_blocks,
                          const uint64_t *minimum_ptrs, const uint64_t *maximum_ptrs,
                          const uint64_t *summary_ptrs, int kv_heads, int head_dim,
                          int page_size, int32_t *device_status, hs_stream stream);

/* hs_attend_rows without a caller workspace: no counterpart in the reference
 * (whose Triton attention needs no scratch). For callers with no device
 * allocator at hand — a bare FFI binding of this library, or a process whose
 * device memory is all committed to its pools — the split partials live in a
 * fixed 16 MiB array in the library's device memory, one per device, and the
 * call allocates nothing. A call needing more scratch than that
 * (hs_attend_workspace_bytes > 16 MiB) returns HS_ERR_WORKSPACE. The first
 * call on a device looks up the array's address (make it before capturing a
 * stream). All calls on a device share the array: calls that can overlap on
 * the GPU race and must be ordered by the caller. Nothing in the array needs
 * to start at zero. Arguments and results are those of hs_attend_rows. */
HS_API int hs_attend_rows_static(int batch, const void *query, int64_t query_batch_stride,
                                 int query_dtype, const void *pool, int64_t pool_blocks,
                                 int kv_dtype, const int64_t *rows, int64_t rows_batch_stride,
                                 int64_t rows_head_stride, int64_t count, void *out,
                                 int64_t out_batch_stride, int q_heads, int kv_heads,
                                 int head_dim, int page_size, int32_t *device_status,
                                 hs_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* HISPARSE_H */
