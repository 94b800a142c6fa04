// maxsim_topk.cu -- scoring + per-query top-k in bounded memory.
//
// The reference ranks with torch.topk over the full (B_q, n) score matrix
// (src/cycle3_experiments.py:215). Here the corpus is scored in document chunks into one reused
// (B_q, chunk) buffer; each chunk's top-k (global ids) is sort-merged into a running list. A
// global top-k entry is always in its chunk's top-k, and every merge ranks by (score descending,
// id ascending, NaN last), so the result equals the top-k of the full matrix exactly. Short lists
// are padded with (NaN, INT64_MAX), which ranks after every real entry, NaN scores included.
//
// The top-k is not folded into the scoring kernel's epilogue: that kernel sits at its register
// limit, and extra epilogue code measured slower than the separate passes cost (the score chunk
// is written once and read by the top-k while it is still in L2 for typical chunk sizes).
#include <cmath>
#include <cstdint>

#include "tms_internal.h"

namespace tms {
namespace {

constexpr int64_t kDefaultChunkBytes = int64_t(1) << 30;  // score buffer bound when not given

__global__ void pad_topk_kernel(float* vals, int64_t* ids, int64_t rows, int64_t ld, int64_t c0,
                                int64_t c1) {
  const int64_t w = c1 - c0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < rows * w;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / w, c = c0 + (i - r * w);
    vals[r * ld + c] = __int_as_float(0x7fc00000);  // NaN: ranks last
    ids[r * ld + c] = INT64_MAX;
  }
}

int64_t resolve_chunk(int64_t n_queries, int64_t n_docs, int64_t chunk_docs) {
  int64_t c = chunk_docs;
  if (c <= 0) c = kDefaultChunkBytes / (4 * (n_queries > 0 ? n_queries : 1));
  if (c > n_docs) c = n_docs;
  return c < 1 ? 1 : c;
}

struct TopkWs {
  size_t dense, scores, topk, tmp, cand, total;
};
TopkWs topk_ws_layout(int dtype, int64_t n_queries, int64_t nq, int64_t d, int64_t chunk,
                      int64_t k) {
  TopkWs w;
  w.dense = align_up(tms_dense_workspace_size(dtype, n_queries, nq, d, chunk, TMS_OUT_SCORE), 1024);
  w.scores = align_up(static_cast<size_t>(n_queries * chunk) * 4, 1024);
  size_t t1 = tms_topk_workspace_size(n_queries, chunk, k);
  const size_t t2 = tms_topk_workspace_size(n_queries, 2 * k, k);
  w.topk = align_up(t1 > t2 ? t1 : t2, 1024);
  w.tmp = align_up(static_cast<size_t>(n_queries * k) * 12, 1024);
  w.cand = align_up(static_cast<size_t>(n_queries * 2 * k) * 12, 1024);
  w.total = w.dense + w.scores + w.topk + w.tmp + w.cand;
  return w;
}

// rows x width elements of `esize` bytes, row pitches in elements
int copy2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t rows,
           size_t esize, cudaStream_t st) {
  return cuda_status(cudaMemcpy2DAsync(dst, static_cast<size_t>(dpitch) * esize, src,
                                       static_cast<size_t>(spitch) * esize,
                                       static_cast<size_t>(width) * esize,
                                       static_cast<size_t>(rows), cudaMemcpyDeviceToDevice, st));
}

int pad(float* vals, int64_t* ids, int64_t rows, int64_t ld, int64_t c0, int64_t c1,
        cudaStream_t st) {
  if (c1 <= c0) return TMS_OK;
  const int64_t n = rows * (c1 - c0);
  const int blocks = static_cast<int>(n / 256 + 1 < 1024 ? n / 256 + 1 : 1024);
  pad_topk_kernel<<<blocks, 256, 0, st>>>(vals, ids, rows, ld, c0, c1);
  return cuda_status(cudaGetLastError());
}

}  // namespace
}  // namespace tms

using namespace tms;

extern "C" size_t tms_dense_topk_workspace_size(int dtype, int64_t n_queries, int64_t nq,
                                                int64_t d, int64_t n_docs, int64_t k,
                                                int64_t chunk_docs) {
  if (n_queries <= 0 || nq <= 0 || d <= 0 || n_docs <= 0 || k <= 0) return 0;
  if (tms_dense_workspace_size(dtype, n_queries, nq, d, 1, TMS_OUT_SCORE) == 0) return 0;
  const int64_t chunk = resolve_chunk(n_queries, n_docs, chunk_docs);
  return topk_ws_layout(dtype, n_queries, nq, d, chunk, k).total;
}

extern "C" int tms_dense_maxsim_topk(const void* Q, int dtype, int64_t n_queries, int64_t nq,
                                     int64_t d, const void* D, int64_t n_tokens,
                                     const int64_t* doc_offsets, int64_t n_docs,
                                     int64_t nd_uniform, int64_t k, int64_t chunk_docs,
                                     int64_t id_base, float* out_vals, int64_t* out_ids,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  NvtxRange nvtx_range("tms_dense_maxsim_topk");
  if (n_queries < 0 || nq <= 0 || d <= 0 || n_docs < 0 || k < 0) return TMS_ERR_INVALID;
  if (n_queries == 0 || k == 0) return TMS_OK;
  if (k > n_docs || !out_vals || !out_ids) return TMS_ERR_INVALID;
  if (!doc_offsets && nd_uniform < 0) return TMS_ERR_INVALID;
  const int64_t chunk = resolve_chunk(n_queries, n_docs, chunk_docs);
  const TopkWs L = topk_ws_layout(dtype, n_queries, nq, d, chunk, k);
  if (L.total == 0 || !workspace || workspace_bytes < L.total) return TMS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 1023) return TMS_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  void* ws_dense = base;
  float* scores = reinterpret_cast<float*>(base + L.dense);
  void* ws_topk = base + L.dense + L.scores;
  // ids first in each region: the regions are 1024-aligned, so both arrays stay aligned
  int64_t* tmp_ids = reinterpret_cast<int64_t*>(base + L.dense + L.scores + L.topk);
  float* tmp_vals = reinterpret_cast<float*>(tmp_ids + n_queries * k);
  int64_t* cand_ids = reinterpret_cast<int64_t*>(base + L.dense + L.scores + L.topk + L.tmp);
  float* cand_vals = reinterpret_cast<float*>(cand_ids + n_queries * 2 * k);
  const size_t esize = dtype == TMS_F32 ? 4 : 2;
  const int64_t rows = n_queries;
  int rc = TMS_OK;
  for (int64_t c0 = 0; c0 < n_docs; c0 += chunk) {
    const int64_t nc = n_docs - c0 < chunk ? n_docs - c0 : chunk;
    const void* Dc = D;
    int64_t tok = n_tokens;
    if (!doc_offsets) {  // uniform documents: the chunk is a contiguous block of tokens
      Dc = static_cast<const uint8_t*>(D) + static_cast<size_t>(c0 * nd_uniform * d) * esize;
      tok = nc * nd_uniform;
    }
    rc = tms_dense_maxsim(Q, dtype, n_queries, nq, d, Dc, tok, doc_offsets ? doc_offsets + c0 : nullptr,
                          nc, nd_uniform, scores, TMS_OUT_SCORE, ws_dense, L.dense, stream);
    if (rc != TMS_OK) return rc;
    const int64_t kc = k < nc ? k : nc;
    const bool first = c0 == 0;
    // the chunk's top-kc: straight into the output when it is the whole answer
    float* dv = (first && kc == k) ? out_vals : tmp_vals;
    int64_t* di = (first && kc == k) ? out_ids : tmp_ids;
    rc = tms_topk(scores, rows, nc, nc, kc, nullptr, 0, id_base + c0, dv, di, ws_topk, L.topk, stream);
    if (rc != TMS_OK) return rc;
    if (first) {
      if (kc < k) {
        if ((rc = copy2d(out_vals, k, tmp_vals, kc, kc, rows, 4, st)) != TMS_OK) return rc;
        if ((rc = copy2d(out_ids, k, tmp_ids, kc, kc, rows, 8, st)) != TMS_OK) return rc;
        if ((rc = pad(out_vals, out_ids, rows, k, kc, k, st)) != TMS_OK) return rc;
      }
      continue;
    }
    // candidates (rows, 2k): the running list, then this chunk's list padded to k
    if ((rc = copy2d(cand_vals, 2 * k, out_vals, k, k, rows, 4, st)) != TMS_OK) return rc;
    if ((rc = copy2d(cand_ids, 2 * k, out_ids, k, k, rows, 8, st)) != TMS_OK) return rc;
    if ((rc = copy2d(cand_vals + k, 2 * k, tmp_vals, kc, kc, rows, 4, st)) != TMS_OK) return rc;
    if ((rc = copy2d(cand_ids + k, 2 * k, tmp_ids, kc, kc, rows, 8, st)) != TMS_OK) return rc;
    if ((rc = pad(cand_vals, cand_ids, rows, 2 * k, k + kc, 2 * k, st)) != TMS_OK) return rc;
    rc = tms_topk(cand_vals, rows, 2 * k, 2 * k, k, cand_ids, 2 * k, 0, out_vals, out_ids, ws_topk,
                  L.topk, stream);
    if (rc != TMS_OK) return rc;
  }
  return TMS_OK;
}
