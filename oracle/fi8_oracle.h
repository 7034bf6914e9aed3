/*
 * fi8_oracle.h -- CPU restatement of the reference's FlatI8 / FlatBinaryI8
 * exact-scan path (github.com/townsendmerino/aikit). TEST INFRASTRUCTURE ONLY.
 *
 * This library is the checker the parity tests and the CPU-baseline leg of
 * bench.py compare the CUDA path against. Nothing in the product links it, and
 * the product never falls back to it. Every function cites the reference
 * file:line it restates; floating point is IEEE binary32 with no contraction
 * (built with -ffp-contract=off, no fast-math), matching Go's amd64 semantics.
 *
 * Parity pinning: the reference's own tests hold no golden top-K numbers (their
 * inputs come from Go's math/rand streams, and no Go toolchain exists on this
 * machine). The restatement is pinned by the reference's literal vectors
 * (sign-bit order, linalg/hamming_test.go:12-48), its known-answer relations
 * (all-ties -> ids 0..k-1, topk tie/NaN rules, exact-fallback boundaries) and
 * its real-data fixtures (an FI8 v1 blob and a d=256 embedding set).
 */
#ifndef FI8_ORACLE_H
#define FI8_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* quantizeRowInt8Core (linalg/quant.go:43-71). zero_scale is 1 for corpus rows
 * (QuantizeRowInt8, linalg/quant.go:83) and 0 for activations/queries
 * (quantizeRowInt8, linalg/quant.go:171). Returns the row scale. */
float or_quantize_row(const float* row, int64_t d, int8_t* q, float zero_scale);

/* QuantizeRowsInt8 / NewFlatI8's per-row loop (linalg/quant.go:21-31,
 * ann/flat_i8.go:96-107) over a dense, already padded/truncated [n][d] block. */
void or_quantize_rows(const float* v, int64_t n, int64_t d, int8_t* q,
                      float* scales, float zero_scale);

/* dotI8Scalar (linalg/quant.go:150-156). */
int32_t or_dot_i8_scalar(const int8_t* a, const int8_t* b, int64_t d);

/* dotI8 (linalg/quant_i8_amd64.go:10-21): AVX2 bulk restating dotI8AVX2
 * (linalg/dot_amd64.s:323-387) plus the scalar tail. Integer-exact. */
int32_t or_dot_i8(const int8_t* a, const int8_t* b, int64_t d);

/* MatmulBTW8A8Pre/w8a8Span (linalg/quant.go:220-298) for M already-quantized
 * rows against N corpus rows: dst[i*N+j] = float32(dot)*aScale[i]*bScale[j],
 * left to right, 0 when aScale[i]==0. Column-sharded over nthreads exactly like
 * parallelSpawnCols (linalg/linalg.go:208-233); nthreads<=1 runs serially. */
void or_w8a8(const int8_t* aq, const float* ascales, int64_t M,
             const int8_t* bq, const float* bscales, int64_t N, int64_t d,
             float* dst, int nthreads);

/* topHits (ann/flat_i8.go:214-246) over topk.Selector (topk/topk.go:61-186) and
 * topk.ItemCmp (topk/cmp.go:15-34). keep is a live-set mask (nonzero = keep) or
 * NULL. Returns the hit count; writes up to max(k, n) hits. */
int64_t or_top_hits(const float* scores, int64_t n, int64_t k,
                    const uint8_t* keep, int64_t* out_idx, double* out_score);

/* FlatI8.query's CPU path (ann/flat_i8.go:140-206): quantize q (zero scale 0),
 * W8A8 over all n rows, topHits. Returns -1 for the reference's nil (n==0). */
int64_t or_flat_i8_query(const int8_t* bq, const float* scales, int64_t n,
                         int64_t d, const float* q, int64_t k,
                         const uint8_t* keep, int64_t* out_idx,
                         double* out_score, int nthreads);

/* The shard merge of queryBatchSharded / Flat.queryShards (ann/backend.go:
 * 262-277, ann/flat.go:201-229, hitCmp ann/flat.go:298): concatenate, sort by
 * (score desc, index asc), truncate to k. Returns the merged count. */
int64_t or_merge_hits(const int64_t* idx, const double* score, int64_t total,
                      int64_t k, int64_t* out_idx, double* out_score);

/* newBinaryPrefilter centering (ann/flat_binary_prefilter.go:64-85): float64
 * running sums in row order over rows with valid[i]!=0 (valid NULL = all). */
int64_t or_center(const float* v, int64_t n, int64_t d, const uint8_t* valid,
                  float* center);

/* PackSignBitsRow (linalg/hamming.go:28-36) of (v - center) (centered,
 * ann/flat_binary_prefilter.go:100-108); center may be NULL. */
void or_pack_row(const float* v, const float* center, int64_t d, uint64_t* dst);

/* newBinaryPrefilter code build (ann/flat_binary_prefilter.go:87-95): invalid
 * (ragged) rows keep all-zero codes. */
void or_pack_codes(const float* v, const float* center, int64_t n, int64_t d,
                   const uint8_t* valid, uint64_t* codes);

/* hammingRowsGeneric (linalg/hamming.go:64-73). */
void or_hamming_rows(const uint64_t* q, const uint64_t* codes, int64_t words,
                     int64_t n, uint16_t* dst);

/* prefilterHist (ann/flat_binary_prefilter.go:145-216): ids out ascending.
 * Returns the id count. */
int64_t or_prefilter_hist(const uint64_t* qc, const uint64_t* codes, int64_t n,
                          int64_t dim, int64_t cand, int32_t* ids_out);
/* or_prefilter_hist with the reference's worker split over nthreads host
 * threads (identical results). */
int64_t or_prefilter_hist_mt(const uint64_t* qc, const uint64_t* codes, int64_t n,
                             int64_t dim, int64_t cand, int32_t* ids_out, int nthreads);

/* prefilterHeap/scanShard/finishCandidates (ann/flat_binary_prefilter.go:
 * 227-313) with nshards shards (binQueryWorkers' fan-out, :330-335). */
int64_t or_prefilter_heap(const uint64_t* qc, const uint64_t* codes, int64_t n,
                          int64_t dim, int64_t cand, const uint8_t* keep,
                          int nshards, int32_t* ids_out);

/* FlatBinaryI8.query (ann/flat_binary_i8.go:86-153): exact FlatI8 fallback when
 * k<=0, k>=n, cand>=n or cand overflows; otherwise pack the centered query,
 * prefilter (hist without keep, heap with keep), gather + W8A8 rerank, topk.
 * Returns -1 for the reference's nil. */
int64_t or_flat_binary_i8_query(const uint64_t* codes, const float* center,
                                int64_t words, const int8_t* bq,
                                const float* scales, int64_t n, int64_t d,
                                int64_t over, const float* q, int64_t k,
                                const uint8_t* keep, int64_t* out_idx,
                                double* out_score, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
