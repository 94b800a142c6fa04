// ivf.cu -- candidate generation upstream of MaxSim: an inverted-file (IVF) probe over the token
// centroids, the first stage of PLAID-style late-interaction search.
//
// The reference has no candidate stage of its own: it reaches one only through external searchers
// (PLAID's dense_search, src/plaid_integration_benchmark.py:186-211 and :309-317; WARP,
// baselines/bench_warp.py). The stage implemented here: every query token probes its nprobe best
// centroids (scores Q . C^T, top-nprobe per token by the library's top-k); a document is a
// candidate of a query when one of its tokens is assigned to a probed centroid (the inverted list
// of a centroid = the sorted ids of the documents holding a token of that centroid). Candidates
// are then scored exactly by the dense MaxSim kernel.
//
// Kernels (all bounds-checked against the caller's sizes, no atomics on scores):
//  * ivf_mark_kernel: one warp per (query, probed centroid) ORs the centroid's documents into the
//    query's candidate bitmap and into a union bitmap (row n_queries) -- 32 documents per word.
//  * bitmap_compact_kernel: one CTA turns the union bitmap into the sorted list of its documents
//    (block-wide exclusive scan of per-thread popcounts over 1024-word windows).
//  * gather_offsets_kernel / gather_docs_kernel: the candidates' token rows are copied into one
//    contiguous ragged corpus (16-byte vectors, one warp per document), so the candidates of the
//    whole query batch are scored by ONE multi-query launch.
//  * mask_candidates_kernel: a query's score of a candidate that is not in its own bitmap (it was
//    probed by another query of the batch) is set to `fill` (-inf), so every query ranks exactly
//    its own candidate set.
#include "tms_device.cuh"
#include "tms_internal.h"

namespace tms {
namespace {

constexpr int kCompactThreads = 1024;

__global__ void zero_words_kernel(uint32_t* __restrict__ w, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    w[i] = 0u;
}

// bitmaps: (n_queries + 1, words) -- row q = query q's candidates, row n_queries = their union.
__global__ void ivf_mark_kernel(const int64_t* __restrict__ probe, int64_t n_queries,
                                int64_t n_probe, const int64_t* __restrict__ ivf_offsets,
                                const int32_t* __restrict__ ivf_docs, int64_t n_centroids,
                                int64_t n_docs, uint32_t* __restrict__ bitmaps, int64_t words) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  uint32_t* const uni = bitmaps + n_queries * words;
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
       w < n_queries * n_probe; w += warps) {
    const int64_t q = w / n_probe;
    const int64_t c = __ldg(probe + w);
    if (c < 0 || c >= n_centroids) continue;  // an id outside the centroid table probes nothing
    const int64_t lo = __ldg(ivf_offsets + c), hi = __ldg(ivf_offsets + c + 1);
    uint32_t* const row = bitmaps + q * words;
    for (int64_t i = lo + lane; i < hi; i += 32) {
      const int64_t doc = __ldg(ivf_docs + i);
      if (doc < 0 || doc >= n_docs) continue;
      const uint32_t bit = 1u << (doc & 31);
      const int64_t wi = doc >> 5;
      // most bits are already set by an earlier centroid: read before writing
      if (!(row[wi] & bit)) atomicOr(row + wi, bit);
      if (!(uni[wi] & bit)) atomicOr(uni + wi, bit);
    }
  }
}

// Block-wide exclusive scan of one value per thread; returns the block total in *total.
__device__ __forceinline__ int64_t block_exclusive_scan(int64_t v, int64_t* total, int64_t* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t s = (lane < static_cast<int>(blockDim.x >> 5)) ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    sh[lane] = s;  // inclusive prefix of the warp totals
  }
  __syncthreads();
  const int64_t before = (warp > 0 ? sh[warp - 1] : 0) + x - v;
  *total = sh[(blockDim.x >> 5) - 1];
  __syncthreads();
  return before;
}

// One CTA: the set bits of `bitmap` (words words, bits past n_bits ignored) in increasing order.
__global__ void __launch_bounds__(kCompactThreads) bitmap_compact_kernel(
    const uint32_t* __restrict__ bitmap, int64_t words, int64_t n_bits, int64_t* __restrict__ ids,
    int64_t capacity, int64_t* __restrict__ count) {
  __shared__ int64_t sh[32];
  int64_t base = 0;
  for (int64_t w0 = 0; w0 < words; w0 += kCompactThreads) {
    const int64_t w = w0 + threadIdx.x;
    uint32_t bits = (w < words) ? bitmap[w] : 0u;
    if (w == words - 1 && (n_bits & 31)) bits &= (1u << (n_bits & 31)) - 1u;
    int64_t total;
    int64_t pos = base + block_exclusive_scan(__popc(bits), &total, sh);
    while (bits) {
      const int b = __ffs(bits) - 1;
      bits &= bits - 1u;
      if (pos < capacity) ids[pos] = w * 32 + b;
      ++pos;
    }
    base += total;
  }
  if (threadIdx.x == 0) *count = base;
}

// out_offsets[i] = sum of the lengths of documents ids[0..i) (n_ids + 1 entries), one CTA.
__global__ void __launch_bounds__(kCompactThreads) gather_offsets_kernel(
    const int64_t* __restrict__ doc_offsets, int64_t n_docs, const int64_t* __restrict__ ids,
    int64_t n_ids, int64_t* __restrict__ out_offsets) {
  __shared__ int64_t sh[32];
  int64_t base = 0;
  for (int64_t i0 = 0; i0 < n_ids; i0 += kCompactThreads) {
    const int64_t i = i0 + threadIdx.x;
    int64_t len = 0;
    if (i < n_ids) {
      const int64_t doc = ids[i];
      if (doc >= 0 && doc < n_docs) {
        len = __ldg(doc_offsets + doc + 1) - __ldg(doc_offsets + doc);
        if (len < 0) len = 0;
      }
    }
    int64_t total;
    const int64_t pos = base + block_exclusive_scan(len, &total, sh);
    if (i < n_ids) out_offsets[i] = pos;
    base += total;
  }
  if (threadIdx.x == 0) out_offsets[n_ids] = base;
}

// One warp per selected document copies its rows (row_bytes, a multiple of 16) into `out`.
__global__ void gather_docs_kernel(const uint4* __restrict__ D, int64_t row_vecs,
                                   const int64_t* __restrict__ doc_offsets, int64_t n_docs,
                                   int64_t n_tokens, const int64_t* __restrict__ ids, int64_t n_ids,
                                   const int64_t* __restrict__ out_offsets, int64_t out_tokens,
                                   uint4* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
       i < n_ids; i += warps) {
    const int64_t doc = ids[i];
    if (doc < 0 || doc >= n_docs) continue;
    const int64_t src0 = __ldg(doc_offsets + doc);
    const int64_t o0 = out_offsets[i], o1 = out_offsets[i + 1];
    const int64_t n = o1 - o0;
    for (int64_t e = lane; e < n * row_vecs; e += 32) {
      const int64_t r = e / row_vecs, v = e - r * row_vecs;
      const int64_t src = src0 + r, dst = o0 + r;
      if (src >= 0 && src < n_tokens && dst < out_tokens) out[dst * row_vecs + v] = __ldg(D + src * row_vecs + v);
    }
  }
}

__global__ void mask_candidates_kernel(float* __restrict__ scores, int64_t n_queries, int64_t n_cand,
                                       int64_t ld, const int64_t* __restrict__ ids,
                                       const uint32_t* __restrict__ bitmaps, int64_t words,
                                       int64_t n_docs, float fill) {
  const int64_t total = n_queries * n_cand;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t q = e / n_cand, c = e - q * n_cand;
    const int64_t doc = ids[c];
    const bool in = doc >= 0 && doc < n_docs &&
                    ((bitmaps[q * words + (doc >> 5)] >> (doc & 31)) & 1u);
    if (!in) scores[q * ld + c] = fill;
  }
}

int grid_for(const DeviceInfo* dev, int64_t work, int per_block) {
  int64_t b = (work + per_block - 1) / per_block;
  if (b > dev->num_sms * 8) b = dev->num_sms * 8;
  return b < 1 ? 1 : static_cast<int>(b);
}

}  // namespace
}  // namespace tms

using namespace tms;

extern "C" int tms_ivf_candidates(const int64_t* probe, int64_t n_queries, int64_t n_probe,
                                  const int64_t* ivf_offsets, const int32_t* ivf_docs,
                                  int64_t n_centroids, int64_t n_docs, uint32_t* bitmaps,
                                  int64_t* cand_ids, int64_t cand_capacity, int64_t* cand_count,
                                  void* stream) {
  NvtxRange nvtx_range("tms_ivf_candidates");
  if (n_queries < 0 || n_probe < 0 || n_centroids < 0 || n_docs < 0 || cand_capacity < 0)
    return TMS_ERR_INVALID;
  if (!bitmaps || !cand_count || (n_queries * n_probe > 0 && (!probe || !ivf_offsets)) ||
      (cand_capacity > 0 && !cand_ids))
    return TMS_ERR_INVALID;
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t words = (n_docs + 31) / 32;
  const int64_t all_words = (n_queries + 1) * words;
  zero_words_kernel<<<grid_for(dev, all_words, 256), 256, 0, st>>>(bitmaps, all_words);
  if (n_queries * n_probe > 0 && words > 0)
    ivf_mark_kernel<<<grid_for(dev, n_queries * n_probe * 32, 256), 256, 0, st>>>(
        probe, n_queries, n_probe, ivf_offsets, ivf_docs, n_centroids, n_docs, bitmaps, words);
  bitmap_compact_kernel<<<1, kCompactThreads, 0, st>>>(bitmaps + n_queries * words, words, n_docs,
                                                       cand_ids, cand_capacity, cand_count);
  return cuda_status(cudaGetLastError());
}

extern "C" int tms_gather_offsets(const int64_t* doc_offsets, int64_t n_docs, const int64_t* ids,
                                  int64_t n_ids, int64_t* out_offsets, void* stream) {
  NvtxRange nvtx_range("tms_gather_offsets");
  if (n_docs < 0 || n_ids < 0 || !out_offsets || (n_ids > 0 && (!ids || !doc_offsets)))
    return TMS_ERR_INVALID;
  gather_offsets_kernel<<<1, kCompactThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      doc_offsets, n_docs, ids, n_ids, out_offsets);
  return cuda_status(cudaGetLastError());
}

extern "C" int tms_gather_docs(const void* D, int64_t row_bytes, const int64_t* doc_offsets,
                               int64_t n_docs, int64_t n_tokens, const int64_t* ids, int64_t n_ids,
                               const int64_t* out_offsets, int64_t out_tokens, void* out,
                               void* stream) {
  NvtxRange nvtx_range("tms_gather_docs");
  if (row_bytes <= 0 || row_bytes % 16 || n_docs < 0 || n_tokens < 0 || n_ids < 0 || out_tokens < 0)
    return TMS_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(D) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return TMS_ERR_INVALID;
  if (n_ids == 0 || out_tokens == 0) return TMS_OK;
  if (!D || !doc_offsets || !ids || !out_offsets || !out) return TMS_ERR_INVALID;
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;
  gather_docs_kernel<<<grid_for(dev, n_ids * 32, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(D), row_bytes / 16, doc_offsets, n_docs, n_tokens, ids, n_ids,
      out_offsets, out_tokens, static_cast<uint4*>(out));
  return cuda_status(cudaGetLastError());
}

extern "C" int tms_mask_candidates(float* scores, int64_t n_queries, int64_t n_cand, int64_t ld,
                                   const int64_t* ids, const uint32_t* bitmaps, int64_t n_docs,
                                   float fill, void* stream) {
  NvtxRange nvtx_range("tms_mask_candidates");
  if (n_queries < 0 || n_cand < 0 || ld < n_cand || n_docs < 0) return TMS_ERR_INVALID;
  if (n_queries * n_cand == 0) return TMS_OK;
  if (!scores || !ids || !bitmaps) return TMS_ERR_INVALID;
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;
  mask_candidates_kernel<<<grid_for(dev, n_queries * n_cand, 256), 256, 0,
                           static_cast<cudaStream_t>(stream)>>>(
      scores, n_queries, n_cand, ld, ids, bitmaps, (n_docs + 31) / 32, n_docs, fill);
  return cuda_status(cudaGetLastError());
}
