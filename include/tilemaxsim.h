/*
 * tilemaxsim.h -- C ABI of libtilemaxsim_b200.so, the B200 (sm_100a) MaxSim scoring library.
 *
 * Late-interaction MaxSim:  score(q, doc) = sum_i max_j <Q[q,i,:], D[doc,j,:]>
 *
 * Every entry point is stream-ordered and asynchronous on `stream` (a cudaStream_t passed as
 * void*), never allocates or frees device memory, and never synchronises the host. The caller
 * owns every buffer, including outputs and workspace. All pointers are device pointers unless
 * a comment says otherwise. Return value: TMS_OK or a TMS_ERR_* code (see tms_strerror).
 *
 * Reference interfaces replaced (ashutoshuiuc/tilemaxsim, paths inside that project):
 *   tms_dense_maxsim   <- src/flash_maxsim_v2.py:227-289 flash_maxsim_v2_multiquery (kernels :73-190),
 *                         src/flash_maxsim_v2.py:193-224 flash_maxsim_v2 (kernel :19-70),
 *                         src/flash_maxsim_kernel.py:167-273 flash_maxsim_single / _batch / _multi_doc
 *                         (kernels :25-164; TMS_OUT_TOKEN_MAX is the V1 per-query-token output)
 *   tms_pq_table       <- src/flash_pqsim_kernel.py:190-211 TileMaxSimPQ.build_distance_table (kernel :31-67)
 *   tms_pq_maxsim      <- src/flash_pqsim_kernel.py:213-280 TileMaxSimPQ.score_batch / score_single
 *                         (kernels :70-173)
 *   tms_topk           <- torch.topk after scoring, src/cycle3_experiments.py:215 (with ids_in it
 *                         also merges per-shard top-k lists; the reference has no sharded search)
 */
#ifndef TILEMAXSIM_B200_H
#define TILEMAXSIM_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TMS_API __attribute__((visibility("default")))
#else
#define TMS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define TMS_OK 0
#define TMS_ERR_INVALID 1     /* bad argument: shape, null pointer, misalignment */
#define TMS_ERR_UNSUPPORTED 2 /* valid but not implemented (e.g. d not a multiple of 8) */
#define TMS_ERR_CUDA 3        /* a CUDA runtime/driver call failed */
#define TMS_ERR_TIMEOUT 4     /* a bounded device-side wait gave up (reported by tms_last_device_error) */
#define TMS_ERR_WORKSPACE 5   /* workspace smaller than the *_workspace_size query */
#define TMS_ERR_TOO_LARGE 6   /* problem needs more scratch than tms_dense_maxsim_noalloc holds */
#define TMS_ERR_BAD_OFFSETS 7 /* document offsets negative, decreasing or past n_tokens
                                 (found by tms_validate_offsets, reported by tms_last_device_error) */

/* element types */
#define TMS_F16 0
#define TMS_BF16 1
#define TMS_F32 2 /* multiplied as TF32 on the tensor cores, like the reference's tl.dot on fp32 */

/* PQ modes */
#define TMS_PQ_FAST 0  /* tensor cores where the shape allows (fp16 codebook) */
#define TMS_PQ_EXACT 1 /* fp32 table lookups, the reference precision */
#define TMS_PQ_PRECISE 2 /* the reference precision, by the fastest kernel that keeps it (Python
                            default): fp16 queries of up to 128 rows on the tensor cores with the
                            codebook split into fp16 hi + lo (|codebook| < 65504, the caller's
                            guarantee), in passes of up to four 32-row chunks; batches of <= 8-row
                            queries needing several passes, and other shapes, by the fp32 table
                            lookups */

/* dense output modes */
#define TMS_OUT_SCORE 0     /* out[q * n_docs + doc] = sum_i max_j <Q_qi, D_j>                 */
#define TMS_OUT_TOKEN_MAX 1 /* out[(q * n_docs + doc) * nq + i] = max_j <Q_qi, D_j> (V1 output) */

TMS_API const char* tms_strerror(int code);
TMS_API const char* tms_version(void);

/* Reads and clears the device-side error word (bit 31: a bounded wait timed out, low bits = the
 * wait's site; bit 30: tms_validate_offsets found a bad entry, low bits = its index). Synchronises
 * `stream`. Returns TMS_OK, TMS_ERR_TIMEOUT or TMS_ERR_BAD_OFFSETS; *detail (may be NULL)
 * receives the raw word. */
TMS_API int tms_last_device_error(void* stream, uint32_t* detail);

/* Checks a document offsets array on the device, asynchronously on `stream`: every entry of
 * offsets[0..n_docs] must be >= 0 and <= n_tokens and the array non-decreasing. A violation sets
 * the device error word (read it with tms_last_device_error). The scoring calls do not run this
 * check themselves (it would cost a host synchronisation per call); whatever the offsets, they
 * never read outside D or the codes array. */
TMS_API int tms_validate_offsets(const int64_t* doc_offsets, int64_t n_docs, int64_t n_tokens,
                                 void* stream);

/* ---------------------------------------------------------------- dense MaxSim (tcgen05 + TMA) */

/* Workspace bytes tms_dense_maxsim needs for this problem (packed query tiles, and partial sums
 * when nq > 32 in TMS_OUT_SCORE mode). */
TMS_API size_t tms_dense_workspace_size(int dtype, int64_t n_queries, int64_t nq, int64_t d,
                                int64_t n_docs, int out_mode);

/* Q: (n_queries, nq, d) contiguous, dtype.
 * D: (n_tokens, d) contiguous, dtype: all documents' tokens concatenated.
 * Documents: if doc_offsets != NULL, doc i owns tokens [doc_offsets[i], doc_offsets[i+1]) (int64,
 *   n_docs+1 entries, non-decreasing, doc_offsets[n_docs] <= n_tokens; an empty document scores
 *   -inf, as the reference's running max starts at -inf). Otherwise every document has
 *   nd_uniform tokens and doc i owns [i*nd_uniform, (i+1)*nd_uniform) (the padded (B,Nd,d) layout:
 *   every row participates, zero padding included).
 * out: fp32, TMS_OUT_SCORE -> (n_queries, n_docs); TMS_OUT_TOKEN_MAX -> (n_queries, n_docs, nq).
 * Requirements: d % 8 == 0 (16-bit) or d % 4 == 0 (fp32); Q, D 16-byte aligned; n_tokens < 2^31. */
TMS_API int tms_dense_maxsim(const void* Q, int dtype, int64_t n_queries, int64_t nq, int64_t d,
                     const void* D, int64_t n_tokens, const int64_t* doc_offsets, int64_t n_docs,
                     int64_t nd_uniform, float* out, int out_mode, void* workspace,
                     size_t workspace_bytes, void* stream);

/* No-allocation variant of tms_dense_maxsim. It has no counterpart in the reference.
 * For callers that cannot hand the library any device memory -- e.g. a serving engine that
 * reserves the whole GPU for its own memory pool at start-up, or a host plug-in that must not call
 * cudaMalloc (which can synchronise the device and fail under memory pressure) -- the kernel's
 * scratch lives in a fixed 4 MiB static device array that every GPU loading the library holds
 * until exit. Same arguments and results as tms_dense_maxsim without the workspace; returns
 * TMS_ERR_TOO_LARGE when tms_dense_workspace_size() for the problem exceeds 4 MiB (e.g. more than
 * 512 queries of <= 32 tokens at d = 128 fp16). The first call on each device (and again in each
 * new CUDA context on it, e.g. after cudaDeviceReset) looks up the array's device address
 * (cudaGetSymbolAddress, with that device current) and caches it: make that first call before any
 * stream capture. All calls share the one array, so two calls whose kernels
 * overlap on the GPU race with each other; issue them on one stream (or otherwise order them).
 * Nothing in the array has to start at zero. It allocates nothing and calls no allocator. */
TMS_API int tms_dense_maxsim_noalloc(const void* Q, int dtype, int64_t n_queries, int64_t nq,
                                     int64_t d, const void* D, int64_t n_tokens,
                                     const int64_t* doc_offsets, int64_t n_docs, int64_t nd_uniform,
                                     float* out, int out_mode, void* stream);

/* ---------------------------------------------------------------- PQ asymmetric distance (ADC) */

/* table[(q*nq + i) * M*K + m*K + k] = <Q[q,i, m*dsub:(m+1)*dsub], codebook[m,k,:]> in fp32.
 * Q dtype: TMS_F16/BF16/F32; codebook dtype: TMS_F16/BF16/F32, (M, K, dsub) contiguous. */
TMS_API int tms_pq_table(const void* Q, int q_dtype, int64_t n_queries, int64_t nq, const void* codebook,
                 int cb_dtype, int64_t M, int64_t K, int64_t dsub, float* table, void* stream);

TMS_API size_t tms_pq_workspace_size(int64_t n_queries, int64_t nq, int64_t M, int64_t K,
                                     int64_t dsub, int64_t n_docs);

/* codes: (n_tokens, M) uint8, doc layout as in tms_dense_maxsim (offsets or nd_uniform).
 * out[q * n_docs + doc] = sum_i max_j sum_m table[q,i,m,codes[j,m]] (K <= 256).
 * mode TMS_PQ_FAST: fp16 queries with dsub % 8 == 0, M*dsub % 64 == 0 and a codebook of <= 96 KB
 * in fp16 run on the tensor cores (codes decoded on chip through the codebook rounded to fp16,
 * never written to HBM; |error| <= 1e-3*|score| + 5e-3): up to four 32-row query chunks
 * (n_queries * ceil(nq / 32) <= 4, d <= 256) with the decoded tokens written to tensor memory,
 * larger batches with the tokens decoded into shared memory; other shapes fall back to:
 * mode TMS_PQ_EXACT: the fp32 distance table of eight query tokens is built in shared memory and
 * table entries are summed straight from the codes (the reference's arithmetic; M = 8 or 16 with
 * code rows aligned to M bytes take a bank-conflict-free layout that sums the subspaces in groups
 * of four, other shapes sum in m order). The workspace must be 1024-byte aligned. */
TMS_API int tms_pq_maxsim(const void* Q, int q_dtype, int64_t n_queries, int64_t nq,
                          const void* codebook, int cb_dtype, int64_t M, int64_t K, int64_t dsub,
                          const uint8_t* codes, int64_t n_tokens, const int64_t* doc_offsets,
                          int64_t n_docs, int64_t nd_uniform, float* out, int mode,
                          void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- scoring + top-k, bounded memory */

/* Workspace for tms_dense_maxsim_topk with the same arguments (0 = unsupported shape). */
TMS_API size_t tms_dense_topk_workspace_size(int dtype, int64_t n_queries, int64_t nq, int64_t d,
                                             int64_t n_docs, int64_t k, int64_t chunk_docs);

/* Scores the corpus as tms_dense_maxsim does and writes each query's k best documents
 * (score descending, id ascending, NaN last; ids = document index + id_base) to out_vals
 * (n_queries, k) fp32 and out_ids (n_queries, k) int64, never holding more than chunk_docs
 * documents' scores (chunk_docs <= 0: a 1 GiB score buffer). The result equals tms_topk over the
 * full score matrix. k <= 2048 and k <= n_docs. The workspace must be 1024-byte aligned.
 * Replaces torch.topk over the full score matrix (reference src/cycle3_experiments.py:215). */
TMS_API int tms_dense_maxsim_topk(const void* Q, int dtype, int64_t n_queries, int64_t nq,
                                  int64_t d, const void* D, int64_t n_tokens,
                                  const int64_t* doc_offsets, int64_t n_docs, int64_t nd_uniform,
                                  int64_t k, int64_t chunk_docs, int64_t id_base, float* out_vals,
                                  int64_t* out_ids, void* workspace, size_t workspace_bytes,
                                  void* stream);

/* ---------------------------------------------------------------- residual-compressed corpora */

/* Workspace for tms_residual_maxsim (0 = unsupported shape: d must be 64 or 128). */
TMS_API size_t tms_residual_workspace_size(int64_t n_queries, int64_t nq, int64_t d, int64_t n_docs);

/* MaxSim over a corpus stored as ColBERTv2-style residual codes: token t is
 *   x = centroids[codes[t], :] + bucket_weights[b_j]   (j = 0..d-1),
 * optionally scaled to unit length (normalize != 0), where b_j is dimension j's nbits-bit bucket
 * index: bit k of b_j is bit (j*nbits + k) of the token's residual row, bits numbered from the most
 * significant bit of byte 0 (residuals: n_tokens x d*nbits/8 bytes; nbits 1, 2 or 4). Tokens are
 * decoded on chip, rounded once to fp16 and scored like tms_dense_maxsim (fp16 queries, fp32
 * accumulation; offsets or nd_uniform as there): out[q * n_docs + doc]. Up to four 32-row query
 * chunks run on the token-rows kernel, which rounds the unscaled token to fp16 and applies the
 * unit-length scale to the token's fp32 products; larger batches scale before rounding. centroids: (n_centroids, d)
 * fp16, 16-byte aligned; codes int32 (clamped to [0, n_centroids)); bucket_weights: 2^nbits fp32.
 * d = 64 or 128. The workspace must be 1024-byte aligned. */
TMS_API int tms_residual_maxsim(const void* Q, int64_t n_queries, int64_t nq, int64_t d,
                                const void* centroids, int64_t n_centroids, const int32_t* codes,
                                const uint8_t* residuals, const float* bucket_weights, int nbits,
                                int normalize, int64_t n_tokens, const int64_t* doc_offsets,
                                int64_t n_docs, int64_t nd_uniform, float* out, void* workspace,
                                size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- top-k */

TMS_API size_t tms_topk_workspace_size(int64_t rows, int64_t n, int64_t k);

/* Per row r of scores (rows, n) fp32 with row stride ld: the k best (score descending, then id
 * ascending; NaN ranks last) -> out_vals (rows, k), out_ids (rows, k) int64. The id of column c is
 * ids_in[r*ld_ids + c] when ids_in != NULL, else c + id_base. k <= 2048 and k <= n. */
TMS_API int tms_topk(const float* scores, int64_t rows, int64_t n, int64_t ld, int64_t k,
             const int64_t* ids_in, int64_t ld_ids, int64_t id_base, float* out_vals,
             int64_t* out_ids, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- candidate generation (IVF probe) */
/* No reference function: the reference reaches a candidate stage only through external searchers
 * (PLAID's dense_search, src/plaid_integration_benchmark.py:186-211; WARP, baselines/bench_warp.py).
 * Python: tilemaxsim_b200.IVFIndex. */

/* probe: (n_queries, n_probe) centroid ids (each query's tokens' nprobe best centroids, any order,
 * ids outside [0, n_centroids) ignored); ivf_offsets (n_centroids + 1) / ivf_docs: inverted lists
 * (the documents holding a token of each centroid; ids outside [0, n_docs) ignored). Writes
 * bitmaps ((n_queries + 1) rows of ceil(n_docs / 32) words; row q = query q's candidates, row
 * n_queries = their union), the union's documents in increasing order into cand_ids (at most
 * cand_capacity of them) and their number into *cand_count (device). */
TMS_API int tms_ivf_candidates(const int64_t* probe, int64_t n_queries, int64_t n_probe,
                               const int64_t* ivf_offsets, const int32_t* ivf_docs,
                               int64_t n_centroids, int64_t n_docs, uint32_t* bitmaps,
                               int64_t* cand_ids, int64_t cand_capacity, int64_t* cand_count,
                               void* stream);

/* out_offsets (n_ids + 1): running token counts of the documents ids[0..n_ids) of a ragged corpus
 * (ids outside [0, n_docs) count 0 tokens). */
TMS_API int tms_gather_offsets(const int64_t* doc_offsets, int64_t n_docs, const int64_t* ids,
                               int64_t n_ids, int64_t* out_offsets, void* stream);

/* Copies the token rows (row_bytes each, a multiple of 16; 16-byte aligned buffers) of documents
 * ids[0..n_ids) into out, document i at rows [out_offsets[i], out_offsets[i+1]). */
TMS_API int tms_gather_docs(const void* D, int64_t row_bytes, const int64_t* doc_offsets,
                            int64_t n_docs, int64_t n_tokens, const int64_t* ids, int64_t n_ids,
                            const int64_t* out_offsets, int64_t out_tokens, void* out, void* stream);

/* scores (n_queries, n_cand) with row stride ld: entries whose document ids[c] is not set in row
 * q of bitmaps (as written by tms_ivf_candidates) become `fill`. */
TMS_API int tms_mask_candidates(float* scores, int64_t n_queries, int64_t n_cand, int64_t ld,
                                const int64_t* ids, const uint32_t* bitmaps, int64_t n_docs,
                                float fill, void* stream);

/* Sharded search merge (no reference function: the reference has no distributed path). Each rank
 * packs its (rows, k) list into packed (rows, 2k) int64: k ids, then the k scores' fp32 bit
 * patterns; after an all-gather of the packed rows (rank-major: (world * rows, 2k)),
 * tms_topk_merge_packed writes the global top-k of every row by the tms_topk rule (score
 * descending, id ascending, NaN last). world * k <= 16384. */
TMS_API int tms_topk_pack(const float* vals, const int64_t* ids, int64_t rows, int64_t k,
                          int64_t* packed, void* stream);
TMS_API int tms_topk_merge_packed(const int64_t* gathered, int64_t world, int64_t rows, int64_t k,
                                  float* out_vals, int64_t* out_ids, void* stream);

/* ---------------------------------------------------------------- introspection and test hooks */

/* Launch plan the dense kernel would use (no reference counterpart): info[0..9] = tokens per tile,
 * query-resident flag, query tiles per CTA group, pipeline stages, groups, token ranges, query
 * tiles, 128-byte K chunks, dynamic shared memory bytes, CTAs. */
TMS_API int tms_dense_plan_info(int dtype, int64_t n_queries, int64_t nq, int64_t d, int64_t n_docs,
                                int64_t n_tokens, int out_mode, int num_sms, int64_t* info);

/* Test hook (no reference counterpart): wait limit of the bounded device waits in ns (0 keeps the
 * current limit) and fault flags (bit 0: the dense kernel's producer issues no load, so the
 * consumers' waits run out and tms_last_device_error reports TMS_ERR_TIMEOUT). */
TMS_API void tms_set_debug(uint64_t timeout_ns, int flags);

#ifdef __cplusplus
}
#endif
#endif /* TILEMAXSIM_B200_H */
