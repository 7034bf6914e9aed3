/*
 * fi8.h -- C ABI of libfi8_b200.so, the B200 (sm_100a) backend for aikit's
 * exact int8 nearest-neighbour scan (ann.FlatI8) and its FlatBinary -> FlatI8
 * two-stage path.
 *
 * The ABI is what a Go adapter registered through ann.RegisterBackend
 * (ann/backend.go:139) binds, cgo-free through a purego-style dlopen (as the
 * reference's gocudrv binds libcuda, gpu/cuda.go:11,54) or with cgo. Plain
 * pointers and sizes only, no exceptions across the
 * boundary, integer status codes, and no CPU fallback: a call either runs on
 * the GPU or returns an error, which the Go seam already treats as "decline,
 * use the next tier" (ann/flat_i8.go:191-198, ann/backend.go:86-122).
 *
 * Threading: every index serializes its own calls with an internal mutex, so an
 * index may be shared by concurrent callers (FlatI8.Query is called
 * concurrently, ann/flat_i8.go:29-30). Different indexes run concurrently.
 */
#ifndef FI8_H
#define FI8_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define FI8_OK 0
#define FI8_ERR_ARG 1      /* bad argument (shape mismatch, null pointer) */
#define FI8_ERR_DECLINED 2 /* outside what the device path answers; caller falls back
                              (the decline contract of gpu/anncuda/backend.go:577-579) */
#define FI8_ERR_CUDA 3     /* a CUDA runtime call failed */
#define FI8_ERR_OOM 4      /* device allocation failed (gpu/anncuda/backend.go:131-139) */
#define FI8_ERR_DEVICE 5   /* a kernel reported an error (e.g. a bounded wait expired) */

typedef struct fi8_ctx fi8_ctx;     /* one CUDA device */
typedef struct fi8_index fi8_index; /* a device-resident FlatI8 shard */
typedef struct fi8_bin fi8_bin;     /* a device-resident FlatBinaryI8 shard */

/* Message for the last failing call on this thread ("" if none). */
const char* fi8_last_error(void);

/* Number of visible CUDA devices. */
int fi8_device_count(int* out);

/* Open / close a device context. Replaces the device bring-up of
 * gpu/anncuda/backend.go:67-116 (CreateSystemDefaultDevice + module loads). */
int fi8_ctx_create(int device, fi8_ctx** out);
int fi8_ctx_destroy(fi8_ctx* ctx);
/* Streaming-multiprocessor count of the context's device. */
int fi8_ctx_sm_count(fi8_ctx* ctx, int* out);

/* Measurement aid with no counterpart in the reference: the device's int8
 * tensor-pipe rate. One CTA per SM issues iters x 4 back-to-back
 * tcgen05.mma.kind::i8 (M=128, N=256, K=32) on shared-memory operands (no
 * global traffic), timed with CUDA events: *ops_per_s (2 ops per
 * multiply-add) and *ms. The roofline denominator for tensor-bound batches. */
int fi8_probe_tensor_i8(fi8_ctx* ctx, int64_t iters, double* ops_per_s, double* ms);

/* ann.Backend.NewI8Index (ann/backend.go:20; gpu/anncuda/backend.go:124-154).
 * Copies codes [n*dim] int8 row-major and scales [n] f32 to the device; the host
 * arrays are not retained (they may alias an mmap, ann/flat_i8_mmap.go:157-180).
 * id_base is the global index of row 0: a row shard of a larger corpus reports
 * global indices (0 for a whole corpus). Rows are stored with a pitch of
 * dim rounded up to 16 bytes, zero padded. */
int fi8_index_create(fi8_ctx* ctx, const int8_t* codes, const float* scales, int64_t n,
                     int32_t dim, int64_t id_base, fi8_index** out);

/* NewFlatI8 on the device (ann/flat_i8.go:74-109): vecs [n*dim] f32 host rows
 * are copied in chunks and quantized on the GPU exactly as QuantizeRowInt8
 * does (linalg/quant.go:43-71; an all-zero row gets scale 1). Ragged input is
 * the caller's to pad or truncate to dim, as NewFlatI8 does. The result is
 * the index fi8_index_create would build from NewFlatI8's own codes. No
 * counterpart on the reference's device seam (its build is CPU-only). */
int fi8_index_create_f32(fi8_ctx* ctx, const float* vecs, int64_t n, int32_t dim, int64_t id_base,
                         fi8_index** out);

/* Paged and streamed sources: the device path of a paged FlatI8
 * (LoadFlatI8MmapPaged, ann/flat_i8_mmap.go:75-102), whose codes may exceed
 * host RAM and which the reference refuses to put on a device
 * (ann/backend.go:162, errPagedGPU at :366). The adapter creates an empty
 * index, then walks the pager's blocks in order -- Touch a block, upload its
 * rows, let the pager evict it -- so only a block or two is resident on the
 * host at a time, and the device ends up holding the whole corpus.
 * fi8_index_create_empty: n rows of dim, all zero (a row not yet uploaded
 * scores 0). fi8_index_upload_rows: rows [row0, row0 + rows) from host codes
 * [rows*dim] and scales [rows]; the host memory may be released as soon as the
 * call returns (the rows are already in pinned staging buffers), and the copies
 * drain on the index's stream, overlapping the caller's next block.
 * fi8_index_upload_finish: wait for every upload and free the staging buffers
 * (two 64 MB pinned buffers, allocated by the first upload_rows). Call it
 * before device-resident queries on other streams; the host-pointer entry
 * points are ordered after the uploads anyway. Uploading every row gives the
 * index fi8_index_create would build from the same rows. */
int fi8_index_create_empty(fi8_ctx* ctx, int64_t n, int32_t dim, int64_t id_base, fi8_index** out);
int fi8_index_upload_rows(fi8_index* idx, int64_t row0, const int8_t* codes, const float* scales, int64_t rows);
int fi8_index_upload_finish(fi8_index* idx);

/* Copy an index's rows back to the host: codes [n*dim] int8 and scales [n]
 * (e.g. to fill FlatI8's bq and scales after a device build). */
int fi8_index_read_rows(fi8_index* idx, int8_t* codes, float* scales);

/* I8Index.Close (ann/backend.go:31; gpu/anncuda/backend.go:238-246). */
int fi8_index_destroy(fi8_index* idx);

int fi8_index_info(fi8_index* idx, int64_t* n, int32_t* dim);

/* I8Index.Score (ann/backend.go:30; gpu/anncuda/backend.go:181-205): q [dim] f32
 * on the host, dst [n] f32 on the host. dst[j] is bit-identical to
 * linalg.MatmulBTW8A8's value for row j (linalg/quant.go:290-296). */
int fi8_score(fi8_index* idx, const float* q, float* dst);

/* I8BatchIndex.ScoreBatch (ann/backend.go:43; gpu/anncuda/backend.go:212-236):
 * q [M*dim], dst [M*n] row-major, every element assigned. */
int fi8_score_batch(fi8_index* idx, const float* q, int32_t M, float* dst);

/* I8TopKIndex.TopKBatch (ann/backend.go:54; gpu/anncuda/backend.go:568-667):
 * q [M*dim] host f32; out_idx [M*k] int32 global indices, out_score [M*k] f32,
 * each row sorted (score desc, index asc), padded with index -1 when fewer than
 * k rows have a non-NaN score. Declines (FI8_ERR_DECLINED) when k <= 0 or
 * k >= n, like the reference; also when k is beyond the device top-K: above
 * fi8_topk_max_k() for a batch that runs the scan (M below
 * FI8_OPT_GEMM_MIN_BATCH), above 4096 for one that runs the GEMM. */
int fi8_topk_batch(fi8_index* idx, const float* q, int32_t M, int32_t k, int32_t* out_idx,
                   float* out_score);

/* FlatI8.QueryFilter (ann/flat_i8.go:136) for a batch: fi8_topk_batch over
 * the rows whose keep bit is set. keep is a host bitmap over GLOBAL row ids
 * (bit id%64 of word id/64; ids at or past nbits are not kept), shared by the
 * M queries, in place of the reference's keep(id) callback. The reference
 * runs filtered queries on the CPU (flat_i8.go:176-198 only offers the
 * device the unfiltered case); this is additive. Same declines as
 * fi8_topk_batch; fewer than k kept rows pad with index -1. */
int fi8_topk_batch_keep(fi8_index* idx, const float* q, int32_t M, int32_t k, const uint64_t* keep,
                        int64_t nbits, int32_t* out_idx, float* out_score);

/* Largest k the scan path answers for this index (single queries and
 * batches below FI8_OPT_GEMM_MIN_BATCH); batches on the GEMM take k <= 4096. */
int fi8_topk_max_k(fi8_index* idx, int32_t* out);

/* The row ranges a batched top-k of M queries at k over n rows runs as (one
 * GEMM launch and one select each; plan_ranges in fi8_api.cu): *count ranges,
 * written as count + 1 ascending row offsets to out_bounds, 0 first and n
 * last. Host-only, no device work; FI8_ERR_ARG (with *count set) when
 * max_bounds < count + 1. No counterpart in the reference. */
int fi8_gemm_plan(int64_t n, int32_t M, int32_t k, int64_t* out_bounds, int32_t max_bounds, int32_t* count);

/* Stream-ordered, device-resident form of fi8_topk_batch for callers that keep
 * queries and results in HBM (multi-GPU merge, benchmarks): d_q [M*dim] f32 and
 * d_keys [M*k] packed uint64 keys (decode with fi8_keys_unpack), both device
 * pointers; stream is a cudaStream_t (NULL = the legacy default stream, as in
 * CUDA). Does not synchronize; device-side errors surface at the next
 * fi8_index_sync. The answer is exact: a batch on the GEMM path whose row
 * range admitted more candidates than its per-query buffer holds (a corpus
 * ordered against the query) is recomputed on the device, in stream order,
 * by the per-query scan -- launches gated on the batch's own overflow flag,
 * which return at once when nothing was dropped. d_q is read until the
 * call's work completes on the stream. Unlike fi8_topk_batch it accepts
 * k >= n (a row shard smaller than k yields all of its
 * rows, then empty keys). Calls on one index must not overlap on the GPU (they
 * share the index's scratch); issue them on one stream. */
int fi8_topk_batch_async(fi8_index* idx, const float* d_q, int32_t M, int32_t k, uint64_t* d_keys,
                         void* stream);
/* fi8_topk_batch_async restricted by a device keep bitmap d_keep (as
 * fi8_topk_batch_keep; NULL = every row). */
int fi8_topk_batch_async_keep(fi8_index* idx, const float* d_q, int32_t M, int32_t k, const uint64_t* d_keep,
                              int64_t nbits, uint64_t* d_keys, void* stream);

/* Tuning knobs of an index. FI8_OPT_GEMM_MIN_BATCH: batches of at least this
 * many queries take the tcgen05 GEMM path, smaller ones the per-query scan
 * (default 2). Both return identical results. */
#define FI8_OPT_GEMM_MIN_BATCH 1
/* FI8_OPT_KERNEL_TIMING: 1 records a CUDA event pair around every kernel the
 * index launches (on the launch stream), read back by fi8_index_kernel_times;
 * 0 (default) records nothing. A measurement aid with no counterpart in the
 * reference. */
#define FI8_OPT_KERNEL_TIMING 2
/* FI8_OPT_GEMM_CTAS: the batched GEMM's persistent grid uses at most this many
 * CTAs, one per SM (0, the default: every SM). For rows of at most 256 bytes
 * the launch may use fewer, down to the largest multiple of the batch's
 * 128-query tiles when that keeps 90 % of the cap, so that each CTA stays on
 * one query tile. No counterpart in the reference. A multi-GPU caller that
 * overlaps the NCCL all-gather of one batch with the next batch's GEMM leaves
 * a few SMs free for the collective's kernel; results are identical. */
#define FI8_OPT_GEMM_CTAS 3
/* FI8_OPT_GEMM_PAIR: 1 runs batches of more than 128 queries on pairs of
 * CTAs (tcgen05 cta_group::2: 256-query x 256-row tiles, each SM loading 2/3
 * of the operand bytes of a single-CTA tile); 0 (default) keeps one CTA per
 * tile, which measured faster on B200 (at the full C3 shape under the power
 * cap, 154.5 against 194 ms of GEMM per batch of 4096): a pair waits for the
 * slower of two epilogues, and it ran at a lower clock for the same power.
 * Results are identical. No counterpart in the reference. */
#define FI8_OPT_GEMM_PAIR 4
int fi8_index_set_option(fi8_index* idx, int option, int64_t value);

/* Kernel classes reported by fi8_index_kernel_times. */
#define FI8_KERNEL_SCAN 0     /* fused W8A8 scan + top-K (or scores) */
#define FI8_KERNEL_GEMM 1     /* tcgen05 GEMM with threshold-filter epilogue */
#define FI8_KERNEL_SELECT 2   /* per-query exact select of the candidates */
#define FI8_KERNEL_QUANTIZE 3 /* query quantization / sign-bit packing */
#define FI8_KERNEL_RERANK 4   /* FlatBinaryI8 shortlist rerank */
#define FI8_KERNEL_REDO 5     /* the batched path's gated exact redo (see fi8_topk_batch_async) */
#define FI8_KERNEL_KINDS 6

/* Totals over the launches timed since the last reset, per kernel class:
 * launches[i], ms[i] (sum of per-launch device durations) and bytes[i]
 * (algorithmic bytes: corpus codes + scales of the rows each launch covers,
 * times the passes it makes, plus its query bytes). Each array holds
 * FI8_KERNEL_KINDS entries. Waits for the timed launches to finish; reset != 0
 * then clears the totals. */
int fi8_index_kernel_times(fi8_index* idx, int64_t* launches, double* ms, double* bytes, int reset);

/* The timed launches themselves, in launch order (up to cap of them, *count
 * set): kernel class, device ms and algorithmic bytes of each. Does not reset;
 * read it before fi8_index_kernel_times(..., reset = 1). */
int fi8_index_kernel_log(fi8_index* idx, int32_t cap, int32_t* count, int32_t* kinds, double* ms, double* bytes);

/* Number of kernels the index's last query call launched (scan: one per 64
 * queries; batched: quantize + a GEMM and a select per row range, then the
 * gated redo -- a latch and one scan launch per up to 32 MB of its per-query
 * scratch (one launch for a batch of 4096 at k = 100), or the popcount
 * prefilter's launches for a tensor-core shortlist -- which return at once
 * unless a candidate was dropped). */
int fi8_index_last_launch_count(fi8_index* idx, int32_t* out);

/* Wait for the index's stream and report any device-side error flag. */
int fi8_index_sync(fi8_index* idx);

/* Decode packed keys (host memory): index -1 / score 0 for empty slots. */
int fi8_keys_unpack(const uint64_t* keys, int64_t count, int32_t* out_idx, float* out_score);

/* Merge per-shard candidate keys: d_in [nsrc][M][k] (device, 0 = empty) ->
 * d_out [M][k], the top k per query under (score desc, index asc). The
 * N-way form of queryBatchSharded's merge (ann/backend.go:262-277). */
int fi8_merge_keys_async(fi8_ctx* ctx, const uint64_t* d_in, int32_t nsrc, int32_t M, int32_t k,
                         uint64_t* d_out, void* stream);

/* Allocation-free single-query top-K. No counterpart in the reference: it is
 * for callers that must not allocate device memory while serving (HBM fully
 * reserved at start-up, so a cudaMalloc on the query path could fail or
 * stall the device). Same result as fi8_topk_batch_async with M = 1: d_q [dim]
 * f32 and d_keys [k] packed keys, both device pointers supplied by the caller;
 * stream is a cudaStream_t (NULL = the legacy default stream). It allocates
 * nothing: its scratch is a fixed 368,896-byte array in the library (one per
 * device, held until the process exits), so k is limited to 256 (a clear
 * FI8_ERR_ARG above that). The first call on each device resolves that array's
 * address (set-up; make that first call before any stream capture). Calls
 * share the array, so two calls that overlap on the GPU race: serialize them.
 * Does not synchronize; device errors surface at fi8_index_sync. */
int fi8_topk1_noalloc(fi8_index* idx, const float* d_q, int32_t k, uint64_t* d_keys, void* stream);

/* ---------------------------------------------------------------------------
 * FlatBinaryI8 (ann/flat_binary_i8.go): the sign-bit Hamming prefilter over a
 * FlatI8 shard, then an int8 W8A8 rerank of the shortlist. The reference has
 * no device seam for this type (it always runs on the CPU); these entry points
 * are additive surface for an optional BinaryI8Index interface, detected by
 * type assertion the way I8TopKIndex is (ann/backend.go:50-55).
 * ------------------------------------------------------------------------- */

/* Build from the prefilter's packed codes [n*words] (binaryPrefilter.codes,
 * ann/flat_binary_prefilter.go:87-95; words = ceil(dim/64)), its center [dim]
 * (NULL for an uncentred prefilter, prefilter.go:79-84) and the FlatI8 rows
 * i8 [n*dim] / scales [n] (ann/flat_i8.go:31-66). overquery below 1 is taken
 * as 1 (prefilter.go:58). id_base as for fi8_index_create. All host arrays are
 * copied. */
int fi8_bin_index_create(fi8_ctx* ctx, const uint64_t* codes, int32_t words, const float* center,
                         const int8_t* i8, const float* scales, int64_t n, int32_t dim, int32_t overquery,
                         int64_t id_base, fi8_bin** out);
int fi8_bin_index_destroy(fi8_bin* b);

/* Streamed and paged sources for a FlatBinaryI8, as fi8_index_create_empty /
 * fi8_index_upload_rows / fi8_index_upload_finish are for a FlatI8: the
 * prefilter's codes and the FlatI8 rows of a corpus larger than host RAM
 * (an FI8 file walked block by block, or rows generated block by block) reach
 * the device without the whole corpus ever being resident on the host.
 * fi8_bin_index_create_empty: n rows of dim, all zero, with the prefilter's
 * centre [dim] (NULL: uncentred; copied). fi8_bin_upload_rows: rows
 * [row0, row0 + rows) from host codes [rows*words], i8 [rows*dim] and scales
 * [rows]; the host memory may be reused when the call returns.
 * fi8_bin_upload_finish: wait for every upload and free the staging buffers.
 * Uploading every row gives the index fi8_bin_index_create builds from the
 * same arrays. Upload before fi8_bin_set_tensor_prefilter (it unpacks the
 * codes already on the device). No counterpart in the reference. */
int fi8_bin_index_create_empty(fi8_ctx* ctx, int64_t n, int32_t dim, int32_t words, const float* center,
                               int32_t overquery, int64_t id_base, fi8_bin** out);
int fi8_bin_upload_rows(fi8_bin* b, int64_t row0, const uint64_t* codes, const int8_t* i8, const float* scales,
                        int64_t rows);
int fi8_bin_upload_finish(fi8_bin* b);

/* newFlatBinaryI8 on the device (ann/flat_binary_i8.go:57-62): from f32 rows
 * vecs [n*dim], the FlatI8 rows (quantized as fi8_index_create_f32) and the
 * prefilter's sign codes. valid [n] (NULL = all) marks the rows of the
 * reference's full dim; the others (ragged input) are left out of the centre
 * and keep all-zero codes (prefilter.go:70-95). centered = 0 builds an
 * uncentred prefilter. center (NULL = compute) supplies the centre, e.g. the
 * whole corpus's for a row shard; computed, it is float32(float64 sum of the
 * valid rows in row order / their count), bit-identical to the reference,
 * and none when no row is valid. */
int fi8_bin_index_create_f32(fi8_ctx* ctx, const float* vecs, const uint8_t* valid, int64_t n, int32_t dim,
                             int32_t overquery, int32_t centered, const float* center, int64_t id_base,
                             fi8_bin** out);

/* The prefilter's centre [dim] (*has_center = 0 when uncentred) and its
 * packed codes [n*words], copied back to the host. */
int fi8_bin_center(fi8_bin* b, float* out, int32_t* has_center);
int fi8_bin_read_codes(fi8_bin* b, uint64_t* codes);

/* The FlatI8 index inside b (owned by b): for fi8_index_* options, timing and
 * launch counts. */
int fi8_bin_index_handle(fi8_bin* b, fi8_index** out);

/* Tensor-core prefilter for query batches (no reference counterpart; the
 * result is the same shortlist). min_batch > 0 unpacks the codes on the
 * device into +1/-1 int8 rows (n x dim bytes, rounded up to 16, held until
 * min_batch = 0 or destroy; built once) and sends every prefilter of at least
 * min_batch queries through the tcgen05 kind::i8 GEMM: the dot of two sign
 * rows is dim - 2 * distance, so the batch's distances are one matrix
 * product, and the epilogue selects each query's cand nearest rows under
 * (distance, id) exactly. Smaller batches keep the popcount pass. */
int fi8_bin_set_tensor_prefilter(fi8_bin* b, int32_t min_batch);

/* FlatBinaryI8.Query for M queries (ann/flat_binary_i8.go:86-109): q [M*dim]
 * host f32; out_idx/out_score [M*k], as fi8_topk_batch. With cand = k *
 * overquery: when cand >= n this is FlatI8's exact top-k (:95-97); otherwise
 * the cand rows nearest the centred query's sign bits in Hamming distance,
 * ties by ascending id (prefilterHist, prefilter.go:145-216), reranked by
 * W8A8 score (rerank, :122-153). Declines k <= 0 and k >= n (the reference
 * returns the whole corpus there), and cand above the device limit (2048).
 * A batch on the tensor-core prefilter whose row range admits more candidates
 * than its buffer holds is redone on the device with the popcount pass, so the
 * answer stays exact (as for fi8_bin_prefilter_async). */
int fi8_bin_query_topk(fi8_bin* b, const float* q, int32_t M, int32_t k, int32_t* out_idx, float* out_score);

/* FlatBinaryI8.QueryFilter (flat_binary_i8.go:83): the keep filter applies in
 * the prefilter, as prefilterHeap does (prefilter.go:227-313): the shortlist
 * is the cand nearest KEPT rows under (distance, id). keep as for
 * fi8_topk_batch_keep. */
int fi8_bin_query_topk_keep(fi8_bin* b, const float* q, int32_t M, int32_t k, const uint64_t* keep, int64_t nbits,
                            int32_t* out_idx, float* out_score);

/* Device-resident halves, for sharded use: every rank prefilters its shard,
 * the M x cand keys are all-gathered and merged (fi8_merge_keys_async) into the
 * global shortlist -- the global cand nearest by (distance, id), as the
 * reference computes it over the whole corpus -- then every rank reranks the
 * shortlist rows it holds and the M x k results are merged again.
 * fi8_bin_prefilter_async: d_q [M*dim] f32 -> d_keys [M*cand] packed keys of
 * (-distance, global id), 0-padded; sorted != 0 sorts each query's keys
 * descending, which the key merge needs (the rerank takes any order).
 * fi8_bin_rerank_async: d_short
 * [M*cand] keys (rows of other shards are skipped) -> d_keys [M*k] W8A8 keys,
 * sorted, 0-padded. Stream semantics as fi8_topk_batch_async: a tensor-core
 * shortlist that dropped candidates is recomputed by the popcount pass in
 * stream order (launches gated on that batch's overflow flag), so the keys
 * are exact. */
int fi8_bin_prefilter_async(fi8_bin* b, const float* d_q, int32_t M, int32_t cand, uint64_t* d_keys, int32_t sorted,
                            void* stream);
int fi8_bin_rerank_async(fi8_bin* b, const float* d_q, int32_t M, const uint64_t* d_short, int32_t cand, int32_t k,
                         uint64_t* d_keys, void* stream);
/* fi8_bin_prefilter_async over the rows of a device keep bitmap (NULL = all). */
int fi8_bin_prefilter_async_keep(fi8_bin* b, const float* d_q, int32_t M, int32_t cand, const uint64_t* d_keep,
                                 int64_t nbits, uint64_t* d_keys, int32_t sorted, void* stream);

#ifdef __cplusplus
}
#endif
#endif
