/*
 * v1x.h -- C ABI of the B200 (sm_100a) kernels for the SGLang V1 sparse-attention
 * query-side selection path.
 *
 * Conventions shared by every entry point:
 *   - Kernels of the query path (metadata, staging, scoring, route, topk) are
 *     launched at the device's greatest stream priority, the gather at the
 *     default priority, so that independent batches on separate streams
 *     overlap (one batch's gather fills the SMs the next batch's selection
 *     leaves free).
 *   - All tensor arguments are raw DEVICE pointers of the dtype named in the
 *     comment; sizes and strides are in ELEMENTS unless the name says bytes.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call only
 *     enqueues work on that stream: no allocation, no host<->device copy, no
 *     synchronisation, so every call can be captured in a CUDA graph.
 *   - Return value: V1X_OK (0) or a negative V1X_ERR_* code; on error nothing was
 *     launched and v1x_last_error() returns a message (per calling thread).
 *   - Kernels never trap.  Conditions the reference turns into device asserts are
 *     reported through a caller-owned int32 device status word (see
 *     v1x_allocate), leaving the guarded state untouched.
 *   - Packed page: 8448 bytes = 64 tokens x 128 FP8 e4m3 bytes, then 64 fp32
 *     scales (reference: sglang/srt/layers/attention/v1_deepseek/kernels.py:1-3).
 *
 * Reference paths below are relative to the reference checkout:
 *   DS = sglang/srt/layers/attention/v1_deepseek
 *   NA = sglang/srt/layers/attention/v1_native
 *   VQ = sglang/kernels/jit/csrc/deepseek_v4/v1_query.cuh
 */
#ifndef V1X_H
#define V1X_H

#include <stdint.h>

#if defined(__GNUC__)
#define V1X_API __attribute__((visibility("default")))
#else
#define V1X_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define V1X_OK 0
#define V1X_ERR_INVALID (-1)     /* argument / shape / dtype check failed      */
#define V1X_ERR_CUDA (-2)        /* CUDA runtime error while launching         */
#define V1X_ERR_UNSUPPORTED (-3) /* valid request outside what is implemented  */

/* device status word values (written by kernels, read by the host) */
#define V1X_STATUS_OK 0
#define V1X_STATUS_ARENA_EXHAUSTED 1 /* allocate: free stack smaller than needed */
#define V1X_STATUS_TIMEOUT 2         /* a bounded device-side wait gave up          */
#define V1X_STATUS_BAD_PAGE 3        /* build: a source page id outside the native pool */
#define V1X_STATUS_CAPACITY 4        /* stage_union: the union needs more pages than dst holds */

/* Library identity: returns 0x010000 * major + 0x100 * minor + patch. */
V1X_API int v1x_version(void);

/* Message of the last failed call on this thread ("" if none). */
V1X_API const char* v1x_last_error(void);

/* ------------------------------------------------------------------------ */
/* fused.route -- replaces V1QueryKernel::route (VQ:155-180, kernel VQ:7-49).
 * scores  f32 [batch, score_cols] with row stride score_stride (% 4 == 0)
 * lens, takes, tail_rows  i32 [batch]
 * selected  i32 or i64 [batch, take_stride] (selected_is_i64 selects)
 * rt  i32 [batch, pages];  ft  i32 [batch, fine_pages]
 * Checks as the reference: 64 <= pages <= 4096, score_cols >= 8*pages,
 * take_stride <= pages, score_stride % 4 == 0, capacity > 0,
 * fine_pages >= take_stride. */
V1X_API int v1x_route(const float* scores, int64_t score_stride, int64_t score_cols,
              const int32_t* lens, const int32_t* takes, void* selected, int selected_is_i64,
              int64_t take_stride, int64_t pages, const int32_t* rt, int32_t* ft,
              int64_t fine_pages, const int32_t* tail_rows, int64_t capacity, int fill_table,
              int64_t batch, void* stream);

/* Extension (no reference counterpart): fused.route taking per-page scores
 * (the maxima of each page's 8 centre logits, e.g. v1x_score_fp8's page_max)
 * instead of centre logits.  page_scores f32 [batch, >= pages] with row stride
 * page_stride.  Selection, fine-table fill and checks are those of v1x_route. */
V1X_API int v1x_route_pages(const float* page_scores, int64_t page_stride, const int32_t* lens,
              const int32_t* takes, void* selected, int selected_is_i64, int64_t take_stride,
              int64_t pages, const int32_t* rt, int32_t* ft, int64_t fine_pages,
              const int32_t* tail_rows, int64_t capacity, int fill_table, int64_t batch,
              void* stream);

/* ------------------------------------------------------------------------ */
/* fused.topk -- replaces V1QueryKernel::topk (VQ:181-220, kernel VQ:62-153).
 * scores f32 [batch, cols] row stride score_stride (% 4 == 0); mutated in place
 *   when mask != 0 (boundary-bucket members outside [sink, tail) -> -inf).
 * fine_lens, lens, takes i32 [batch]; members i32 [member_rows, 64];
 * rt, nt i32 [batch, pages]; selected i32/i64 [batch, take_stride];
 * physical, logical, raw i32 [batch, topk]; expanded i32 [batch,
 * expansion_stride] with expansion_stride 0 or 4*topk+64; fine_table i32
 * [batch, fine_table_cols] (read when direct_fine).
 * Selection: the topk largest scores of scores[row, :fine_lens[row]] ordered
 * by (value desc, index asc); outputs in ascending raw-index order.
 * Checks: 0 < topk <= 2048, 0 <= window <= 4096, expansion stride, and
 * fine_table_cols >= take_stride when direct_fine.  Unlike the reference, any
 * batch >= 1 is accepted (the reference requires batch > 512). */
V1X_API int v1x_topk(float* scores, int64_t score_stride, int64_t cols, const int32_t* fine_lens,
             const int32_t* members, int64_t member_rows, const int32_t* rt, const int32_t* nt,
             int64_t pages, const void* selected, int selected_is_i64, int64_t take_stride,
             const int32_t* lens, const int32_t* takes, int32_t* physical, int32_t* logical,
             int32_t* raw, int64_t topk, int64_t window, int mask, int32_t* expanded,
             int64_t expansion_stride, int physical_output, int bucket_from_rank,
             const int32_t* fine_table, int64_t fine_table_cols, int direct_fine, int64_t batch,
             void* stream);

/* TopK-v2's transform -- replaces TopKKernel::transform of the vendored
 * topk_v2.cuh that NA/deps/topk2048.py:15-32 (identity page table) and
 * NA/deps/topk2048_mapped_20261012.py:13-21 (with original ids) call.  For row
 * b: the topk largest of scores[b, :seq_lens[b]] (cols columns at most),
 * ordered by (value desc, index asc); out[b, t] = -1 for an empty slot, else
 * idx = page_table[b*table_stride + (raw >> log2(page_size))] * page_size + raw %
 * page_size, or original_ids[idx] when original_ids is not NULL; raw[b, t] = raw
 * (raw may be NULL).  A row with seq_lens[b] <= topk lists raw = t for t <
 * seq_lens[b] and -1 after, as the reference's trivial transform.  Outputs in
 * ascending raw order (the reference leaves the order unspecified).
 * table_stride may be 0 (one shared row).  Checks: 0 < topk <= 2048,
 * score_stride % 4 == 0 and >= cols, page_size a power of two. */
V1X_API int v1x_topk_transform(const float* scores, int64_t score_stride, int64_t cols, const int32_t* seq_lens,
                       const int32_t* page_table, int64_t table_stride, int64_t page_size,
                       const int32_t* original_ids, int32_t* out, int32_t* raw, int64_t topk, int64_t batch,
                       void* stream);

/* ------------------------------------------------------------------------ */
/* Extension (no reference counterpart): the query selection of one row per CTA
 * -- query metadata (DS/kernels.py:568-591, fixed budget of
 * bench_v1_dynamic_budget_metadata.py:5-28 or the ratio rule), fused.route over
 * page maxima (VQ:7-49), fine_table_shared (DS/kernels.py:488-514), the FP8
 * fine logits of the row's candidates (DeepGEMM contract, runtime.py:538-548,
 * formula DS/kernels.py:310-313, ReLU scoring), the in-kernel boundary mask
 * (bucket from rank) and fused.topk with physical output (VQ:62-153) -- in one
 * launch.  The sink and tail candidates are scored from the native pool
 * directly (stage_tail_shared's copies into the fine pool, DS/kernels.py:
 * 518-564, are not made; the fine-table entries that name those staging pages
 * are still written).
 * q e4m3 [batch, heads, 128]; w f32 [batch, heads]; lens i32 [batch];
 * budget: i32 device word (take = min(built pages, *budget)) or NULL with
 * ratio_num/ratio_den > 0 (take = min(pages, max(ceil(pages*num/den),
 * ceil(topk/64)))); take is clamped to take_stride.  native_table,
 * reordered_table i32 [batch, pages]; page_scores f32 [batch, page_stride] (the
 * max of each built page's 8 centre logits, -inf past them; v1x_score_fp8's
 * page_max).  fine u8 [fine_pages, 8448] reordered pages; members i32
 * [member_rows, 64]; native u8 [native_pages, 8448].
 * Outputs: fine_lens, takes, dg_lens, center_lens, tail_rows i32 [batch];
 * selected i32 [batch, take_stride]; fine_table i32 [batch, fine_cols];
 * physical, logical, raw i32 [batch, topk]; expanded i32 [batch,
 * expansion_stride] (stride 0 or 4*topk+64); scores_out f32 [batch,
 * score_stride] or NULL: the masked fine logits of columns < fine_lens (for
 * checks; score_stride >= take_stride*64 + 64 + max(window, 1024)).
 * Selection and outputs equal those of v1x_query_metadata + v1x_route_pages +
 * v1x_score_fp8 + v1x_topk(mask, bucket_from_rank, physical_output) on the
 * same inputs.  Checks: heads 1 or a multiple of 32 <= 128, 0 < topk <= 2048,
 * 0 <= window <= 4096, 64 <= pages <= 4096, 0 < take_stride <= min(pages, 128),
 * fine_cols >= take_stride; q, pools and members 16-byte aligned.  status: a
 * bounded wait that expires writes V1X_STATUS_TIMEOUT (may be NULL). */
V1X_API int v1x_select_fused(const uint8_t* q, const float* w, int64_t heads, const int32_t* lens,
                     const int32_t* budget, int64_t ratio_num, int64_t ratio_den,
                     const int32_t* native_table, const int32_t* reordered_table, int64_t pages,
                     const float* page_scores, int64_t page_stride, const uint8_t* fine,
                     int64_t fine_pages, const int32_t* members, int64_t member_rows,
                     const uint8_t* native, int64_t native_pages, int64_t capacity, int64_t topk,
                     int64_t window, int64_t take_stride, int64_t fine_cols, int32_t* fine_lens,
                     int32_t* takes, int32_t* dg_lens, int32_t* center_lens, int32_t* tail_rows,
                     int32_t* selected, int32_t* fine_table, int32_t* physical, int32_t* logical,
                     int32_t* raw, int32_t* expanded, int64_t expansion_stride, float* scores_out,
                     int64_t score_stride, int64_t batch, int32_t* status, void* stream);

/* ------------------------------------------------------------------------ */
/* _sort -- replaces the Triton kernel NA/fused_grouping.py:64-76.
 * P (i32), S (f32), O (i32) are [heads, 4096]; segment (g, h) is the N
 * entries at h*4096 + g*N.  flag i32 scalar: the call is a no-op unless
 * *flag < 0 (read on the device).  N is a power of two in [2, 4096] and
 * groups*N <= 4096.  Output: stable sort by score desc, ties by position,
 * +0 == -0. */
V1X_API int v1x_sort_segments(const int32_t* P, int32_t* O, const float* S, const int32_t* flag,
                      int64_t N, int64_t groups, int64_t heads, void* stream);

/* Extension (no reference counterpart): per-segment group offsets for integer
 * keys in [0, key_range) stored as float scores: offsets[seg, j] = number of
 * records of the segment whose key > key_range-1-j, j in [0, key_range].
 * offsets i32 [heads*groups, key_range+1]; key_range <= 12288. */
V1X_API int v1x_group_offsets(const float* S, int32_t* offsets, int64_t N, int64_t groups,
                      int64_t heads, int64_t key_range, void* stream);

/* Extension (no reference counterpart): _sort and v1x_group_offsets in one pass
 * for N in {256, ..., 4096}: O as v1x_sort_segments, offsets [heads*groups,
 * key_range+1] as v1x_group_offsets (key_range <= 2^20), derived from the sorted
 * keys.  S, P and O 16-byte aligned. */
V1X_API int v1x_sort_segments_grouped(const int32_t* P, int32_t* O, const float* S, const int32_t* flag,
                      int32_t* offsets, int64_t N, int64_t groups, int64_t heads, int64_t key_range,
                      void* stream);

/* ------------------------------------------------------------------------ */
/* Index build of 1024-token buckets -- replaces Build.compute's first stages
 * (DS/runtime.py:170-233): initialize (DS/kernels.py:9-29), the seven grouping
 * levels of _dots / _anchor / _sort (NA/fused_grouping.py:39-76) and assemble
 * (DS/kernels.py:32-54).  Native pool: u8 [native_pages, 8448] packed pages; a
 * source page id outside [0, native_pages) reads as zeros and writes
 * V1X_STATUS_BAD_PAGE to *status (may be NULL). */

/* Workspace bytes v1x_build_buckets needs for `buckets` buckets. */
V1X_API int64_t v1x_build_workspace_bytes(int64_t buckets);

/* Whole build of `buckets` buckets in one launch (one 8-CTA cluster each): the
 * 44 launches of the reference's per-bucket sequence.  source i32 [buckets, 16]
 * (native page of each bucket page), starts i32 [buckets] (the bucket's first
 * logical token) -> tmp u8 [buckets, 16, 8448], centers u8 [buckets, 2, 8448],
 * mapping i32 [buckets, 16, 64] (Build.tmp / .centers / .mapping), perm i32
 * [buckets, 1024] (the final member order, Build.perm[current]; may be NULL).
 * work: v1x_build_workspace_bytes(buckets) bytes, 16-byte aligned; native and
 * tmp 16-byte aligned. */
V1X_API int v1x_build_buckets(const uint8_t* native, int64_t native_pages, const int32_t* source,
                      const int32_t* starts, uint8_t* tmp, uint8_t* centers, int32_t* mapping,
                      int32_t* perm, void* work, int32_t* status, int64_t buckets, void* stream);

/* No counterpart in the reference.  v1x_build_buckets without a workspace
 * argument, for callers that cannot allocate device memory when they call: an
 * engine that has handed all free device memory to its own pool, or a plain
 * C / FFI host with no device allocator at hand.  The workspace is a fixed 4 MB
 * array inside the library (8 buckets' worth); more than 8 buckets per call is
 * rejected with V1X_ERR_INVALID.  The call allocates nothing.  Nothing in the
 * scratch has to start at zero: every word the kernel reads was written earlier
 * in the same launch.  The scratch is shared by every call on a device, so
 * calls that can overlap (other streams, other host threads) race on it and must
 * be serialised by the caller.  Its address is looked up once per device, with
 * that device current, on the first call there; make that first call before any
 * stream capture on the device. */
V1X_API int v1x_build_buckets_noalloc(const uint8_t* native, int64_t native_pages, const int32_t* source,
                              const int32_t* starts, uint8_t* tmp, uint8_t* centers, int32_t* mapping,
                              int32_t* perm, int32_t* status, int64_t buckets, void* stream);

/* DS/kernels.py:9-29 (initialize, grid (64,)).  table i32 [16], meta i32 [3]
 * {start, lease, active} -> unit f32 [1024, 128], perm i32 [1024], flag i32
 * (-1 when active, else 0). */
V1X_API int v1x_initialize(const uint8_t* native, int64_t native_pages, const int32_t* table,
                   const int32_t* meta, float* unit, int32_t* perm, int32_t* flag, int32_t* status,
                   void* stream);

/* NA/fused_grouping.py:27-37 (_init, grid (256, heads)).  k: [slots, heads, 128]
 * bf16 (k_is_f32 = 0) or f32 with element strides ks0, ks1; req i32 slot map ->
 * u f32 [heads, 4096, 128], p i32 [heads, 4096] = start + i.  No-op unless *flag < 0. */
V1X_API int v1x_group_init(const void* k, int k_is_f32, const int32_t* req, float* u, int32_t* p,
                   const int32_t* flag, int64_t start, int64_t ks0, int64_t ks1, int64_t heads,
                   void* stream);

/* NA/fused_grouping.py:39-54 (_dots, grid (count/16, heads)).  u f32 [heads, 4096,
 * 128] (heads = 1: [count, 128]), p i32 and s f32 [heads, 4096], anchor i32
 * [heads, 256, 2]; count positions per head (a multiple of 4 and of n). */
V1X_API int v1x_group_dots(const float* u, const int32_t* p, const int32_t* anchor, float* s,
                   const int32_t* flag, int64_t n, int64_t start, int mode, int64_t count,
                   int64_t heads, void* stream);

/* NA/fused_grouping.py:56-63 (_anchor, grid (count/n, heads)): the leftmost
 * minimum of each group of n -> anchor[h, group, slot] = p[...]. */
V1X_API int v1x_group_anchor(const int32_t* p, int32_t* anchor, const float* s, const int32_t* flag,
                     int64_t n, int slot, int64_t count, int64_t heads, void* stream);

/* DS/kernels.py:32-54 (assemble, grid (16, 8)).  table i32 [16], meta i32 [3],
 * ids i32 [1024] (the member order) -> tmp u8 [16, 8448], centers u8 [2, 8448],
 * mapping i32 [16, 64]. */
V1X_API int v1x_assemble(const uint8_t* native, int64_t native_pages, const int32_t* table,
                 const int32_t* meta, const int32_t* ids, uint8_t* tmp, uint8_t* centers,
                 int32_t* mapping, void* stream);

/* ------------------------------------------------------------------------ */
/* Published-end shared-tail variant: one request's chunk of query rows with
 * non-decreasing lengths shares one staged copy of its sink and tail pages.
 * experiments/tail_union_lab_20261021/union.py:10-40 and
 * experiments/fine_pool_shared_20261021/{kernels.py:8-76, route_shared.cu:12-54}.
 * A row's tail starts at the published index end indexed_end[0] (device word):
 * s = min(n, sink), t = max(s, min(min(max(end, 0), n), max(s, n - window))),
 * count = s + n - t. */

/* union.py:16-40 (stage_union).  src / dst u8 [pages, 8448]; nt i32 [nt_len]
 * (the request's logical -> physical page table); lens i32 [rows] -> dst pages
 * [0, total) = the sink pages [0, sp) then the tail pages [tp, ep) of nt,
 * meta i32 [rows, 3] = (s, t, count), desc i32 [4] = (sp, tp, ep, total).  A union
 * larger than dst_pages copies what fits and writes V1X_STATUS_CAPACITY. */
V1X_API int v1x_stage_union(const uint8_t* src, int64_t src_pages, const int32_t* nt, int64_t nt_len,
                    const int32_t* lens, int64_t rows, const int32_t* indexed_end, uint8_t* dst,
                    int64_t dst_pages, int32_t* meta, int32_t* desc, int64_t sink, int64_t window,
                    int32_t* status, void* stream);

/* kernels.py:13-41 (tables): ft i32 [rows, fp] (selected pages, then the staged
 * pages: shared -> cap + union page, else cap + row*scratch + k), dglens i32
 * [rows] = max(take*64 + scored span, 1), clens i32 [rows] = take*64 + count. */
V1X_API int v1x_shared_tables(const int32_t* lens, const int32_t* indexed_end, const int32_t* takes,
                      const int32_t* selected, const int32_t* desc, int32_t* ft, int32_t* dglens,
                      int32_t* clens, int64_t cap, int64_t max_take, int64_t scratch, int64_t fp,
                      int64_t sink, int64_t window, int shared, int64_t rows, void* stream);

/* kernels.py:43-63 (normalize): out f32 [rows, width] = the canonical candidate
 * order [selected members | sink | tail] read from raw f32 [rows, stride], masked
 * (-inf) before Top-K; members i32 [member_rows, 64]. */
V1X_API int v1x_shared_normalize(const float* raw, int64_t stride, const int32_t* lens,
                         const int32_t* indexed_end, const int32_t* takes, const int32_t* selected,
                         const int32_t* members, int64_t member_rows, float* out, int64_t max_take,
                         int64_t width, int64_t sink, int64_t window, int shared, int64_t rows,
                         void* stream);

/* kernels.py:65-76 (map_topk): Top-K ids i64 / values f32 [rows, top] ->
 * logical and physical slot ids i32 [rows, top] (-1 for -inf picks and
 * positions outside [0, n)); nt = the request's page table. */
V1X_API int v1x_shared_map_topk(const int64_t* ids, const float* values, const int32_t* lens,
                        const int32_t* indexed_end, const int32_t* takes, const int32_t* selected,
                        const int32_t* members, int64_t member_rows, const int32_t* nt, int64_t nt_len,
                        int32_t* logical, int32_t* slots, int64_t max_take, int64_t top, int64_t sink,
                        int64_t window, int64_t rows, void* stream);

/* route_shared.cu:12-54 (route_physical): per row the top take = min(max(budget,
 * 0), clamp(published, 0, pages), take_stride) published pages by the max of
 * their 8 centre scores (stable, ties by the blocked rank of a 128-thread
 * layout) written as physical ids rt[row, page] into selected i32 [rows,
 * take_stride] (0 past take); takes i32 [rows]. */
V1X_API int v1x_route_physical(const float* scores, int64_t score_stride, const int32_t* published,
                       const int32_t* budgets, const int32_t* rt, int32_t* selected, int32_t* takes,
                       int64_t pages, int64_t take_stride, int64_t rows, void* stream);

/* ------------------------------------------------------------------------ */
/* Page lifecycle -- replace DS/kernels.py:57-179.  meta i32[3] =
 * {bucket start, lease, active}; every op is a no-op when meta[2] == 0
 * (release has no meta, as in the reference). */

/* DS/kernels.py:57-69. tmp u8 [n_pages, 8448], map i32 [n_pages, 64] -> hash i64 [n_pages, 2] */
V1X_API int v1x_fingerprint(const uint8_t* tmp, const int32_t* map, const int32_t* meta, int64_t* hash,
                    int64_t n_pages, void* stream);

/* DS/kernels.py:72-113. For each tmp page: the lowest live (refs > 0) arena page
 * whose two hashes, 8448 bytes and 64 members are equal, else -1.
 * fine u8 [cap, 8448], members i32 [cap, 64], hashes i64 [cap, 2], refs i32 [cap],
 * match i32 [n_pages]. */
V1X_API int v1x_match_pages(const uint8_t* tmp, const int32_t* map, const int64_t* hash,
                    const int32_t* meta, const uint8_t* fine, const int32_t* members,
                    const int64_t* hashes, const int32_t* refs, int32_t* match, int64_t cap,
                    int64_t n_pages, void* stream);

/* DS/kernels.py:116-131. 16 lanes. free i32 [cap], count i32 scalar, refs i32
 * [cap], tables i32 [leases, 16], new_flags u8 (torch.bool) [16].  If the free
 * stack holds fewer pages than needed, *status = V1X_STATUS_ARENA_EXHAUSTED,
 * every new_flags entry is set to 2 ("bucket not allocated", so that
 * v1x_publish skips the bucket), the lease's table row is set to -1 (no page;
 * v1x_release and v1x_release_many skip -1 entries) and nothing else is written
 * (the reference traps).  The exhaustion is sticky: while *status holds it,
 * every later call on the same word aborts the same way, as nothing runs after
 * the reference's trap; the host reads and clears the word.  status may be
 * NULL. */
V1X_API int v1x_allocate(const int32_t* meta, const int32_t* match, int32_t* free_stack,
                 int32_t* count, int32_t* refs, int32_t* tables, uint8_t* new_flags,
                 int32_t* status, void* stream);

/* DS/kernels.py:134-167. tmp u8 [16, 8448]; tc_bytes u8 / tc_scales f32 = the
 * bucket's 2 centre pages (byte and float views); fine u8 [cap, 8448];
 * centers u8 / center_scales f32 = centre pool views; members i32; hashes i64.
 * A bucket whose new_flags hold 2 (allocation failed) writes nothing. */
V1X_API int v1x_publish(const uint8_t* tmp, const uint8_t* tc_bytes, const float* tc_scales,
                const int32_t* map, const int64_t* hash, const int32_t* meta,
                const int32_t* tables, const uint8_t* new_flags, uint8_t* fine,
                uint8_t* centers, float* center_scales, int32_t* members, int64_t* hashes,
                void* stream);

/* DS/kernels.py:170-179. table i32 [16] (one lease's row).  Entries of -1 (a
 * lease whose allocation aborted) are skipped. */
V1X_API int v1x_release(const int32_t* table, int32_t* refs, int32_t* free_stack, int32_t* count,
                void* stream);

/* Scratch of v1x_prepare_buckets, in int32 words: 4 counters/flags, two lists of
 * 4096 fingerprint-equal pairs (int32 x 2 each), 1024 earliest-equal entries,
 * the call's 64 meta records and source ids. */
#define V1X_PREPARE_WORK_INTS (4 + 4 * 4096 + 1024 + 64 * 5)

/* Extension (no reference counterpart): the page part of Build.compute
 * (DS/runtime.py:230-270: fingerprint -> match_pages -> allocate -> publish,
 * DS/kernels.py:57-167) for up to 64 buckets in canonical order, in five
 * launches instead of six per bucket.  The arena state afterwards equals that
 * of the per-bucket calls in the same order.
 * tmp u8 [*, 16, 8448]; tc_bytes u8 / tc_scales f32 [*, 2, 8448] (byte and
 * float views); map i32 [*, 16, 64]; bucket b reads entry src[b] of these
 * (src: a HOST i32 array [buckets], each id checked to lie in [0,
 * src_buckets)) or entry b when src is NULL, so a caller holding bucket
 * contents in a pool passes their ids instead of copying them; meta: a HOST
 * i32 array [buckets, 4] = (token start, lease, active, state row).  meta and
 * src travel in the launch parameters (no host -> device copy precedes the
 * call).  Scratch: hash i64 [buckets*16, 2],
 * match i32 [buckets*16], new_flags u8 [buckets*16], work i32
 * [V1X_PREPARE_WORK_INTS] (no initial contents needed).  Arena arrays as in
 * v1x_match_pages / v1x_allocate / v1x_publish; center_pages i32 [leases, 2].
 * state_tables i32 [rows, state_table_stride] and state_centers i32 [rows,
 * state_center_stride] (may be NULL together): the request page-table rows,
 * receiving tables[lease] at columns start/1024*16 and center_pages[lease] at
 * start/1024*2 of the bucket's state row.  The first bucket that finds the
 * free stack too short writes V1X_STATUS_ARENA_EXHAUSTED to *status; it and
 * every later bucket of the call change nothing (new_flags 2, lease table rows
 * -1, state rows untouched); a status word that already holds the exhaustion
 * aborts the whole call (sticky, as v1x_allocate).  Precondition: a bucket's 16
 * pages are distinct (their members are disjoint token positions, as every
 * index build produces); two identical pages in one bucket would both be
 * published, and a later bucket of the same call could then take the other
 * copy than the per-bucket sequence's lowest one. */
/* Extension (no reference counterpart): Indexer._release (DS/runtime.py:771-780,
 * kernel DS/kernels.py:170-179) for several requests in one launch.  leases i32
 * = the requests' lease ids, request after request, each request's in order;
 * offsets i32 [requests + 1] = where each request's leases start (CSR).  The
 * refcounts, free stack and count afterwards equal those of v1x_release called
 * for every lease in that order, provided a request's leases hold distinct
 * pages (true of every arena state the prepare paths build: a request's
 * buckets cover disjoint token positions, which are part of a page's
 * identity). */
V1X_API int v1x_release_many(const int32_t* tables, const int32_t* leases, const int32_t* offsets,
                     int64_t requests, int32_t* refs, int32_t* free_stack, int32_t* count,
                     void* stream);

V1X_API int v1x_prepare_buckets(const uint8_t* tmp, const uint8_t* tc_bytes, const float* tc_scales,
                        const int32_t* map, const int32_t* meta, const int32_t* src, int64_t src_buckets,
                        int64_t buckets, int64_t* hash,
                        int32_t* match, uint8_t* new_flags, uint8_t* fine, uint8_t* centers,
                        float* center_scales, int32_t* members, int64_t* hashes, int32_t* refs,
                        int32_t* free_stack, int32_t* count, int32_t* tables,
                        const int32_t* center_pages, int32_t* state_tables, int64_t state_table_stride,
                        int32_t* state_centers, int64_t state_center_stride, int64_t cap,
                        int32_t* work, int32_t* status, void* stream);

/* ------------------------------------------------------------------------ */
/* Per-row query metadata and staging. */

/* DS/kernels.py:568-591 (budget == NULL) or bench_v1_dynamic_budget_metadata.py:5-27
 * (budget = i32 device scalar, take = min(pages, *budget)). lens i32 [batch];
 * nt i32 [batch, np] (row stride np); outputs i32 [batch]. */
V1X_API int v1x_query_metadata(const int32_t* lens, const int32_t* nt, int32_t* fine_lens,
                       int32_t* takes, int32_t* dg_lens, int32_t* center_lens,
                       int32_t* tail_rows, int64_t np, int64_t topk, int64_t num, int64_t den,
                       int64_t sink, int64_t window, const int32_t* budget, int64_t batch,
                       void* stream);

/* Extension (no reference counterpart): v1x_query_metadata followed by
 * v1x_stage_tail_shared (grid form rows_bound = group-of-1 = batch, grid_pages =
 * scratch) in one launch.  Outputs are identical to the two calls; the reference
 * runs them as two kernels (DS/runtime.py:364-368, :492-509). */
V1X_API int v1x_query_prepare(const int32_t* lens, const int32_t* nt, int32_t* fine_lens, int32_t* takes,
                      int32_t* dg_lens, int32_t* center_lens, int32_t* tail_rows, int64_t np,
                      int64_t topk, int64_t num, int64_t den, int64_t sink, int64_t window,
                      const int32_t* budget, const uint8_t* native_bytes, const float* native_scales,
                      uint8_t* fine_bytes, float* fine_scales, int64_t cap, int64_t scratch,
                      int64_t batch, void* stream);

/* DS/kernels.py:224-245. */
V1X_API int v1x_query_lengths(const int32_t* lens, int32_t* fine_lens, int32_t* takes, int64_t topk,
                      int64_t num, int64_t den, int64_t sink, int64_t window, int64_t batch,
                      void* stream);

/* DS/kernels.py:488-514. rt i32 (row stride maxp), selected i32/i64 (row stride
 * take), ft i32 [batch, fp]. */
V1X_API int v1x_fine_table_shared(const int32_t* rt, const void* selected, int selected_is_i64,
                          const int32_t* takes, int32_t* ft, const int32_t* tail_rows,
                          int64_t cap, int64_t maxp, int64_t take, int64_t fp, int64_t scratch,
                          int64_t batch, void* stream);

/* DS/kernels.py:518-564. native_bytes u8 / native_scales f32 and fine_bytes /
 * fine_scales are byte and float views of packed pools; nt row stride np.
 * Programs (g, p) for g < grid_groups, p < grid_pages; rows g*group + [0, group)
 * bounded by rows_bound when rows_bound > 0. */
V1X_API int v1x_stage_tail_shared(const uint8_t* native_bytes, const float* native_scales,
                          const int32_t* nt, const int32_t* lens, uint8_t* fine_bytes,
                          float* fine_scales, const int32_t* tail_rows, int64_t cap,
                          int64_t np, int64_t scratch, int64_t sink, int64_t window,
                          int64_t rows_bound, int64_t group, int64_t grid_groups,
                          int64_t grid_pages, void* stream);

/* DS/kernels.py:444-472 (non-fused mask). scores row stride `stride`, WIDTH cols. */
V1X_API int v1x_mask_fine(float* scores, const void* selected, int selected_is_i64, const int32_t* rt,
                  const int32_t* members, const int32_t* lens, const int32_t* takes,
                  int64_t maxp, int64_t take, int64_t stride, int64_t width, int64_t sink,
                  int64_t window, int64_t batch, void* stream);

/* DS/kernels.py:475-486. logits row stride `stride`; out f32 [batch, maxp];
 * pages p < min(maxp, pcount) are written (pcount = programs x 32 in the reference). */
V1X_API int v1x_reduce_centers(const float* logits, const int32_t* lens, float* out, int64_t maxp,
                       int64_t pcount, int64_t stride, int64_t batch, void* stream);

/* DS/kernels.py:323-376 (non-fused mapping). raw/out/logical i32 [batch, topk];
 * scores row stride width. */
V1X_API int v1x_output_ids(const int32_t* raw, const float* scores, const int32_t* members,
                   const int32_t* rt, const int32_t* nt, const void* selected,
                   int selected_is_i64, const int32_t* lens, const int32_t* takes, int32_t* out,
                   int32_t* logical, const int32_t* ft, int64_t maxp, int64_t np, int64_t take,
                   int64_t width, int64_t topk, int64_t sink, int64_t window, int map_physical,
                   int direct_fine, int64_t fp, int64_t batch, void* stream);

/* Extension (no reference counterpart): the row staging of the reference's
 * Query.run (DS/runtime.py:643-666) in one launch (the reference issues a copy per tensor and per run of equal owners).
 * For rows i < n: q_out[i] = q[i] (heads*128 bytes), w_out[i] = w[i] (heads
 * floats), lens_out[i] = lens[i], nt_out[i] = native_tables[i] (width entries,
 * zeros up to pages), rt_out[i] = state_tables[rows[i]] (pages entries),
 * ct_out[i] = state_centers[rows[i]] (pages/8 entries).  Rows n <= i < filled
 * of every output are zeroed.  rows is a HOST array of n arena row ids, each in
 * [0, state_rows) (checked; it travels in the launch parameters).  Outputs are
 * dense [*, heads*128] / [*, heads] / [*] / [*, pages] / [*, pages] / [*, pages/8]. */
V1X_API int v1x_query_stage(const uint8_t* q, const float* w, const int32_t* lens, const int32_t* native_tables,
                    int64_t width, const int32_t* rows, const int32_t* state_tables,
                    const int32_t* state_centers, int64_t state_rows, uint8_t* q_out, float* w_out,
                    int32_t* lens_out, int32_t* nt_out, int32_t* rt_out, int32_t* ct_out, int64_t heads,
                    int64_t pages, int64_t n, int64_t filled, void* stream);

/* pack_q of the signed-score path -- replaces qwen_gqa_probe_kernels.py:15-20 and
 * the Scorer's quantize + head padding (NA/scoring.py:66-71, NA/grouping.py:41-44).
 * q [rows, qheads, 128] of dtype 0 = f32, 1 = bf16, 2 = f16 with element strides
 * qs0 (row) and qs1 (head), unit inner stride; q8 u8 (e4m3) [out_rows, out_heads,
 * 128]; w f32 [out_rows, out_heads].  For row < rows and head < qheads: scale = the
 * power of two >= max(max|q|, 1e-4) / 448 (exactly; the reference's
 * exp2(ceil(log2(.))) agrees except a few ulps above a power of two), q8 =
 * e4m3(q / scale) (round to nearest even), w = scale * w_mul (the reference's
 * softmax scale / 4); every other entry of q8 and w is 0. */
V1X_API int v1x_pack_q(const void* q, int dtype, int64_t qs0, int64_t qs1, int64_t rows, int64_t out_rows,
                  int64_t qheads, int64_t out_heads, float w_mul, uint8_t* q8, float* w, void* stream);

/* NA/kernels.py:47-59 (mask_scores of the v1_native backend).  scores f32
 * [rows, width] row stride score_stride; table i32 row stride table_stride (fine
 * page of each 64 columns); mapping i32 [pages, 64] logical tokens; positions
 * i32 [rows].  Column c of row r becomes -inf when its logical token l is < 0,
 * > positions[r], or (c < dedup_cols and (l < 64 or l >= fixed_start)).  A table
 * entry outside [0, mapping_pages) reads as l = -1 (the reference reads past the
 * mapping there). */
V1X_API int v1x_mask_scores(float* scores, int64_t score_stride, int64_t width, const int32_t* table,
                    int64_t table_stride, const int32_t* mapping, int64_t mapping_pages,
                    const int32_t* positions, int64_t dedup_cols, int64_t fixed_start, int64_t rows,
                    void* stream);

/* DS/kernels.py:594-600. logical i32 [batch, topk] -> out i32 [batch, stride]. */
V1X_API int v1x_expand_logical(const int32_t* logical, int32_t* out, int64_t topk, int64_t stride,
                       int64_t batch, void* stream);

/* ------------------------------------------------------------------------ */
/* FP8 paged scoring -- the DeepGEMM fp8_paged_mqa_logits contract the reference
 * calls at DS/runtime.py:434-444 and :538-548 (next_n = 1), with the formula of
 * DS/kernels.py:310-313: out[b, j] = sum_h w[b,h] * relu(q[b,h,:] . k_j) * s_j for
 * j < lens[b]; when clean != 0 also -inf for lens[b] <= j < max_len.
 * q u8 (e4m3) [batch, heads, 128]; w f32 [batch, heads]; pool u8 [pool_pages, 8448];
 * table i32 [batch, table_stride]; out f32 [batch, out_stride] (may be NULL).
 * page_max (extension, may be NULL): f32 [batch, page_stride], entries
 * p < ceil(max_len/8) = max over keys 8p..8p+7 (-inf for keys >= lens[b]) -- the
 * per-page centre maximum that fused.route computes (VQ:26-41), produced in the
 * scoring epilogue.
 * relu = 0 gives the signed variant.  impl: 0 = automatic (tensor cores when
 * heads is 1 or a multiple of 32 up to 128 and batch <= 8192, else SIMT), 1 = SIMT (fixed fp32
 * evaluation order, bit-identical to a sequential fp32 restatement, heads <= 64),
 * 2 = tensor cores (heads in {1, 32, 64, 96, 128}; batch <= 8192).  status: optional i32 device
 * word receiving V1X_STATUS_TIMEOUT if a bounded device wait gave up. */
V1X_API int v1x_score_fp8(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages,
                  const int32_t* lens, const int32_t* table, int64_t table_stride, float* out,
                  int64_t out_stride, int64_t max_len, float* page_max, int64_t page_stride,
                  int64_t heads, int relu, int clean, int impl, int32_t* status, int64_t batch,
                  void* stream);

/* Extension (no reference counterpart): v1x_score_fp8 with the scored length of
 * row b derived from lens[b] by lens_kind: 0 = lens[b] (v1x_score_fp8 itself);
 * 1 = the centre count of a token length n, max(8 * ((n-1)/1024*16), 1) -- the
 * center_lens of DS/kernels.py:589 -- so centre scoring can run on the raw token
 * lengths concurrently with the query-metadata kernel.  max_ctas > 0 caps the
 * tensor-core scorer's persistent grid (0: up to two CTAs per SM): small batches
 * stepped many at a time on separate streams finish sooner together when each
 * takes a share of the SMs. */
V1X_API int v1x_score_fp8_ex(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages,
                  const int32_t* lens, const int32_t* table, int64_t table_stride, float* out,
                  int64_t out_stride, int64_t max_len, float* page_max, int64_t page_stride,
                  int64_t heads, int relu, int clean, int impl, int lens_kind, int64_t max_ctas,
                  int32_t* status, int64_t batch, void* stream);

/* Extension (no reference counterpart): the signed-score Scorer's paged logits
 * (NA/scoring.py:48-53, DeepGEMM over q padded to 32 heads, four of them live)
 * for groups of query rows that share one key table.  A group of group_rows
 * rows x 4 heads is one tensor-core MMA operand (N = 4 * group_rows), so a key
 * tile is read once per group instead of once per row.  Keys j < keys are
 * (table[j / 64], j % 64) of the pool.  Without row_tables: out[r, j] = the
 * logit of row r for key j (j < keys).  With row_tables (i32 [rows,
 * row_table_stride], pool pages): out[r, c] for c < row_table_cols * 64 = the
 * logit of row r for key (row_tables[r, c / 64], c % 64) -- the shared table
 * then lists the pool pages any row uses (every page a row table names must be
 * in it); columns of a page outside the pool are 0.  The logits equal the
 * per-row tensor-core scorer's (v1x_score_fp8, heads padded with zero weights).
 * q u8 (e4m3) [ceil(rows / group_rows) * group_rows, 4, 128] and w f32 [same, 4],
 * zero past `rows`, both 16-byte aligned; group_rows in {8, 16, 32}; workspace
 * i32 [ceil(rows / group_rows) * group_rows * pool_pages + 1 + 3 * rows *
 * row_table_cols] (row tables only).  key_valid (u8 [keys], may be NULL; without
 * row tables only): the logits of key j are -inf where key_valid[j] == 0 (the
 * Scorer's masked_fill of invalid centres, NA/scoring.py:86).  mask_map (i32
 * [pool_pages * 64], may be NULL; with row tables only) and mask_pos (i32
 * [rows]): mask_scores fused (NA/kernels.py:47-59 without dedup columns) -- the
 * logit of row r for a key whose logical token l = mask_map[page * 64 + slot]
 * is < 0 or > mask_pos[r] is -inf (so are the columns of a page outside the
 * pool, which are 0 without the mask). */
V1X_API int v1x_score_fp8_grouped(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages,
                  int64_t keys, const int32_t* table, const int32_t* row_tables, int64_t row_table_stride,
                  int64_t row_table_cols, const uint8_t* key_valid, const int32_t* mask_map,
                  const int32_t* mask_pos, int32_t* workspace, float* out, int64_t out_stride, int64_t heads,
                  int64_t group_rows, int64_t rows, int relu, int32_t* status, void* stream);

/* Extension (no reference counterpart): v1x_mqa_logits_fp8 with clean = 1 for
 * query rows of four heads (the signed-score Scorer's dsa mode), on the tensor
 * cores: group_rows rows x 4 heads form one MMA operand, so a tile of 128 keys is
 * read once per group.  q u8 (e4m3) [ceil(rows / group_rows) * group_rows, 4,
 * 128] and w f32 [same, 4], zero past `rows`; k and k_scale 16-byte aligned;
 * group_rows in {8, 16, 32}.  Logits equal v1x_score_fp8's per-row tensor-core
 * order of accumulation, not the SIMT order of v1x_mqa_logits_fp8. */
V1X_API int v1x_mqa_logits_fp8_grouped(const uint8_t* q, const float* w, const uint8_t* k, const float* k_scale,
                  int64_t kv_len, const int32_t* starts, const int32_t* ends, float* out, int64_t out_stride,
                  int64_t heads, int64_t group_rows, int64_t rows, int relu, int32_t* status, void* stream);

/* FP8 MQA logits over a flat key array -- the DeepGEMM fp8_mqa_logits contract
 * the signed-score Scorer calls in its `dsa` mode (NA/scoring.py:74-78) and the
 * probe backend at qwen_gqa_probe_backend.py:184: out[b, j] = sum_h w[b,h] *
 * relu(q[b,h,:] . k_j) * k_scale[j] for starts[b] <= j < ends[b] (ends clamped to
 * kv_len); with clean != 0 every other column j < kv_len is -inf, else untouched.
 * q u8 (e4m3) [batch, heads, 128], 16-byte aligned; w f32 [batch, heads]; k u8
 * (e4m3) [kv_len, 128], 16-byte aligned; k_scale f32 [kv_len]; out f32 [batch,
 * out_stride >= kv_len].  relu = 0 gives the signed variant.  heads <= 64, the
 * SIMT scorer's fixed fp32 evaluation order; heads of weight 0 are skipped (their
 * terms are +-0 for finite inputs). */
V1X_API int v1x_mqa_logits_fp8(const uint8_t* q, const float* w, const uint8_t* k, const float* k_scale,
                  int64_t kv_len, const int32_t* starts, const int32_t* ends, float* out,
                  int64_t out_stride, int64_t heads, int relu, int clean, int64_t batch, void* stream);

/* ------------------------------------------------------------------------ */
/* _gather_slots -- replaces NA/kernels.py:62-77 (GatherWorkspace.gather, :102-111).
 * For t < rows*top: id = ids[(t/top)*ids_stride + t%top]; if id >= 0 the slot
 * p = req ? req[id] : id and kg[t, :] = k[p*ks0 + head*ks1 + d*ks2] (d < dim), same
 * for v; else zero rows.  Element size elem_bytes in {1, 2, 4}; kg/vg contiguous
 * [rows*top, dim]; v/vg may both be NULL (single-output gather). */
V1X_API int v1x_gather_slots(const void* k, const void* v, const int32_t* req, const int32_t* ids,
                     void* kg, void* vg, int64_t rows, int64_t top, int64_t head, int64_t ks0,
                     int64_t ks1, int64_t ks2, int64_t vs0, int64_t vs1, int64_t vs2,
                     int64_t ids_stride, int64_t dim, int64_t elem_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Extension (no reference counterpart): failure-detection self test.  Launches
 * one kernel that waits, with the same bounded mbarrier wait the pipelined
 * kernels use, on a barrier nothing arrives at; after limit_ns (plus at most
 * ~64 ms of polling granularity) it writes V1X_STATUS_TIMEOUT to *status and,
 * if elapsed_ns is not NULL, the measured wait (u64 ns).  The context remains
 * usable.  0 < limit_ns <= 10 s. */
V1X_API int v1x_selftest_wait_timeout(int64_t limit_ns, int32_t* status, uint64_t* elapsed_ns, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* V1X_H */
