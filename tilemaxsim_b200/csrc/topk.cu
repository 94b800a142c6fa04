// topk.cu -- deterministic per-row top-k of fp32 scores: score descending, then id ascending,
// NaN last. Replaces torch.topk after scoring (reference: src/cycle3_experiments.py:215) and merges
// the per-shard (score, id) lists of the sharded search.
//
// One CTA (1024 threads) per row.
//  * Rows of at most kSortMax elements (always the case for shard merges, which carry ids):
//    the whole row is sorted in shared memory by a bitonic network on (key, id).
//  * Longer rows: 4-pass MSB radix select over order-preserving 32-bit keys finds the k-th key K*
//    and how many of its ties are needed; one more pass gathers every key > K* and, through an
//    ordered block scan, the lowest-index ties; the k candidates are then bitonic-sorted.
// Each pass reads the row once (the rows of a score matrix stay L2-resident between passes).
#include "tms_device.cuh"
#include "tms_internal.h"

namespace tms {
namespace {

constexpr int kTopkThreads = 1024;
constexpr int kSortMax = 16384;  // elements sorted whole in shared memory (12 B each)
constexpr int kMaxK = 2048;

// Order-preserving key: larger float -> larger key; every NaN -> 0 (ranks last).
__device__ __forceinline__ uint32_t f2key(float f) {
  const uint32_t b = __float_as_uint(f);
  if (f != f) return 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);  // key 0 decodes to 0xffffffff, a NaN
}

// true if (ka, ia) ranks before (kb, ib)
__device__ __forceinline__ bool before(uint32_t ka, int64_t ia, uint32_t kb, int64_t ib) {
  return ka > kb || (ka == kb && ia < ib);
}

// Bitonic sort of P (power of two) pairs in shared memory into "before" order.
__device__ void bitonic_sort(uint32_t* keys, int64_t* ids, int P) {
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < (P >> 1); i += blockDim.x) {
        const int lo = 2 * stride * (i / stride) + (i % stride);
        const int hi = lo + stride;
        const bool asc = (lo & size) == 0;
        const uint32_t kl = keys[lo], kh = keys[hi];
        const int64_t il = ids[lo], ih = ids[hi];
        const bool swap = asc ? before(kh, ih, kl, il) : before(kl, il, kh, ih);
        if (swap) {
          keys[lo] = kh;
          keys[hi] = kl;
          ids[lo] = ih;
          ids[hi] = il;
        }
      }
      __syncthreads();
    }
  }
}

__device__ __forceinline__ int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

__global__ void __launch_bounds__(kTopkThreads)
    topk_sort_kernel(const float* __restrict__ scores, int64_t n, int64_t ld, int k,
                     const int64_t* __restrict__ ids_in, int64_t ld_ids, int64_t id_base,
                     float* __restrict__ out_vals, int64_t* __restrict__ out_ids) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int P = next_pow2(static_cast<int>(n));
  int64_t* ids = reinterpret_cast<int64_t*>(sm);
  uint32_t* keys = reinterpret_cast<uint32_t*>(sm + static_cast<size_t>(P) * 8);
  const int64_t row = blockIdx.x;
  const float* s = scores + row * ld;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    if (i < n) {
      keys[i] = f2key(s[i]);
      ids[i] = ids_in ? ids_in[row * ld_ids + i] : id_base + i;
    } else {
      keys[i] = 0u;
      ids[i] = INT64_MAX;
    }
  }
  __syncthreads();
  bitonic_sort(keys, ids, P);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    out_vals[row * k + i] = key2f(keys[i]);
    out_ids[row * k + i] = ids[i];
  }
}

// Shard merge without unpacking: every rank's (rows, k) list is packed as one int64 row of 2k
// entries (k ids, then the k scores' fp32 bit patterns), all-gathered rank-major, and merged here:
// one CTA per query row reads its world * k candidates straight from the gathered buffer.
__global__ void pack_topk_kernel(const float* __restrict__ vals, const int64_t* __restrict__ ids,
                                 int64_t rows, int64_t k, int64_t* __restrict__ packed) {
  const int64_t total = rows * k;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = e / k, j = e - r * k;
    packed[r * 2 * k + j] = ids[e];
    packed[r * 2 * k + k + j] = static_cast<int64_t>(__float_as_uint(vals[e]));
  }
}

__global__ void __launch_bounds__(kTopkThreads)
    merge_packed_topk_kernel(const int64_t* __restrict__ gathered, int world, int64_t rows, int k,
                             float* __restrict__ out_vals, int64_t* __restrict__ out_ids) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int n = world * k;
  const int P = next_pow2(n);
  int64_t* ids = reinterpret_cast<int64_t*>(sm);
  uint32_t* keys = reinterpret_cast<uint32_t*>(sm + static_cast<size_t>(P) * 8);
  const int64_t row = blockIdx.x;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    if (i < n) {
      const int r = i / k, j = i - r * k;
      const int64_t* src = gathered + (static_cast<int64_t>(r) * rows + row) * 2 * k;
      keys[i] = f2key(__uint_as_float(static_cast<uint32_t>(src[k + j])));
      ids[i] = src[j];
    } else {
      keys[i] = 0u;
      ids[i] = INT64_MAX;
    }
  }
  __syncthreads();
  bitonic_sort(keys, ids, P);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    out_vals[row * k + i] = key2f(keys[i]);
    out_ids[row * k + i] = ids[i];
  }
}

__global__ void __launch_bounds__(kTopkThreads)
    topk_select_kernel(const float* __restrict__ scores, int64_t n, int64_t ld, int k,
                       int64_t id_base, float* __restrict__ out_vals,
                       int64_t* __restrict__ out_ids, int64_t chunk, int n_chunks) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_mask, s_remaining;
  __shared__ uint32_t s_gt_pos, s_taken;
  __shared__ uint32_t warp_cnt[32];
  __shared__ int64_t cand_ids[kMaxK];
  __shared__ uint32_t cand_keys[kMaxK];
  // Virtual row blockIdx.x = chunk c of row r: columns [c*chunk, c*chunk + chunk) of that row,
  // whose own top-k (ids offset by c*chunk) lands in output row blockIdx.x; a row that is shorter
  // than k is padded with (NaN, INT64_MAX), which ranks after everything.
  const int64_t row = blockIdx.x;
  const int64_t r = row / n_chunks, c = row - r * n_chunks;
  const float* s = scores + r * ld + c * chunk;
  const int64_t n_all = n;
  n = (n_all - c * chunk < chunk) ? n_all - c * chunk : chunk;
  id_base += c * chunk;
  const int k_out = k;
  if (k > n) k = static_cast<int>(n);
  const int tid = threadIdx.x;
  if (n <= 0) {  // empty slice: padding only
    for (int i = tid; i < k_out; i += blockDim.x) {
      out_vals[row * k_out + i] = key2f(0u);
      out_ids[row * k_out + i] = INT64_MAX;
    }
    return;
  }
  const int lane = tid & 31, wid = tid >> 5;

  if (tid == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_remaining = static_cast<uint32_t>(k);
  }
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int64_t i = tid; i < n; i += blockDim.x) {
      const uint32_t key = f2key(__ldg(s + i));
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t rem = s_remaining, cum = 0;
      int b = 255;
      for (; b > 0; --b) {
        if (cum + hist[b] >= rem) break;
        cum += hist[b];
      }
      s_remaining = rem - cum;
      s_prefix = prefix | (static_cast<uint32_t>(b) << shift);
      s_mask = mask | (255u << shift);
    }
    __syncthreads();
  }
  const uint32_t kth = s_prefix;          // key of the k-th best element
  const uint32_t need_ties = s_remaining;  // how many elements equal to kth are taken
  const uint32_t n_gt = static_cast<uint32_t>(k) - need_ties;
  if (tid == 0) {
    s_gt_pos = 0;
    s_taken = 0;
  }
  __syncthreads();
  for (int64_t base = 0; base < n; base += blockDim.x) {
    const int64_t i = base + tid;
    uint32_t key = 0;
    bool gt = false, eq = false;
    if (i < n) {
      key = f2key(__ldg(s + i));
      gt = key > kth;
      eq = key == kth;
    }
    if (gt) {
      const uint32_t p = atomicAdd(&s_gt_pos, 1u);
      cand_keys[p] = key;
      cand_ids[p] = i;
    }
    // Ordered compaction of ties: the lowest indices win.
    const uint32_t bal = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) warp_cnt[wid] = __popc(bal);
    __syncthreads();
    if (wid == 0) {
      const uint32_t c = warp_cnt[lane];
      uint32_t incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      warp_cnt[lane] = incl - c;  // exclusive prefix
    }
    __syncthreads();
    const uint32_t taken = s_taken;
    if (eq) {
      const uint32_t pos = taken + warp_cnt[wid] + __popc(bal & ((1u << lane) - 1u));
      if (pos < need_ties) {
        cand_keys[n_gt + pos] = key;
        cand_ids[n_gt + pos] = i;
      }
    }
    __syncthreads();
    // ties in this step = exclusive prefix of the last warp + the last warp's own count
    if (wid == 31 && lane == 0) s_taken = taken + warp_cnt[31] + __popc(bal);
    __syncthreads();
  }
  const int P = next_pow2(k);
  for (int i = k + tid; i < P; i += blockDim.x) {
    cand_keys[i] = 0u;
    cand_ids[i] = INT64_MAX;
  }
  __syncthreads();
  bitonic_sort(cand_keys, cand_ids, P);
  for (int i = tid; i < k_out; i += blockDim.x) {
    out_vals[row * k_out + i] = i < k ? key2f(cand_keys[i]) : key2f(0u);
    out_ids[row * k_out + i] = i < k ? cand_ids[i] + id_base : INT64_MAX;
  }
}

}  // namespace
}  // namespace tms

using namespace tms;

namespace {
// Long rows with few of them: split each row into n_chunks slices selected by separate CTAs, then
// sort-merge the n_chunks * k candidates per row. Depends on the shape only.
int topk_chunks(int64_t rows, int64_t n, int64_t k) {
  if (n <= kSortMax || rows <= 0 || k <= 0) return 1;
  int64_t c = (n + 16383) / 16384;      // slices of at least ~16k scores
  const int64_t by_merge = kSortMax / k;  // the merge sorts at most kSortMax candidates
  const int64_t by_grid = rows >= 296 ? 1 : 296 / rows;
  if (c > by_merge) c = by_merge;
  if (c > by_grid) c = by_grid;
  return c < 2 ? 1 : static_cast<int>(c);
}
}  // namespace

extern "C" size_t tms_topk_workspace_size(int64_t rows, int64_t n, int64_t k) {
  const int c = topk_chunks(rows, n, k);
  return c > 1 ? static_cast<size_t>(rows * c * k) * 12 + 256 : 0;
}

extern "C" int tms_topk(const float* scores, int64_t rows, int64_t n, int64_t ld, int64_t k,
                        const int64_t* ids_in, int64_t ld_ids, int64_t id_base, float* out_vals,
                        int64_t* out_ids, void* workspace, size_t workspace_bytes, void* stream) {
  NvtxRange nvtx_range("tms_topk");
  if (rows < 0 || n < 0 || k < 0 || ld < n) return TMS_ERR_INVALID;
  if (rows == 0 || k == 0) return TMS_OK;
  if (k > n || !scores || !out_vals || !out_ids) return TMS_ERR_INVALID;
  if (k > kMaxK || rows > 0x7fffffffLL) return TMS_ERR_UNSUPPORTED;
  if (ids_in && ld_ids < n) return TMS_ERR_INVALID;
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n <= kSortMax) {
    int P = 1;
    while (P < n) P <<= 1;
    const size_t smem = static_cast<size_t>(P) * 12;
    if (cudaFuncSetAttribute(topk_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return TMS_ERR_CUDA;
    topk_sort_kernel<<<static_cast<unsigned>(rows), kTopkThreads, smem, st>>>(
        scores, n, ld, static_cast<int>(k), ids_in, ld_ids, id_base, out_vals, out_ids);
    return cuda_status(cudaGetLastError());
  }
  if (ids_in) return TMS_ERR_UNSUPPORTED;  // explicit ids are for shard merges (short rows)
  const int c = topk_chunks(rows, n, k);
  if (c > 1 && workspace && workspace_bytes >= tms_topk_workspace_size(rows, n, k) &&
      rows * c <= 0x7fffffffLL) {
    // slice top-k into the workspace, then one sort-merge per row (ids carried explicitly)
    int64_t* cand_ids = reinterpret_cast<int64_t*>(
        (reinterpret_cast<uintptr_t>(workspace) + 15) & ~static_cast<uintptr_t>(15));
    float* cand_vals = reinterpret_cast<float*>(cand_ids + rows * c * k);
    const int64_t chunk = (n + c - 1) / c;
    topk_select_kernel<<<static_cast<unsigned>(rows * c), kTopkThreads, 0, st>>>(
        scores, n, ld, static_cast<int>(k), id_base, cand_vals, cand_ids, chunk, c);
    if (cudaGetLastError() != cudaSuccess) return TMS_ERR_CUDA;
    const int64_t m = static_cast<int64_t>(c) * k;
    int P = 1;
    while (P < m) P <<= 1;
    const size_t smem = static_cast<size_t>(P) * 12;
    if (cudaFuncSetAttribute(topk_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return TMS_ERR_CUDA;
    topk_sort_kernel<<<static_cast<unsigned>(rows), kTopkThreads, smem, st>>>(
        cand_vals, m, m, static_cast<int>(k), cand_ids, m, 0, out_vals, out_ids);
    return cuda_status(cudaGetLastError());
  }
  topk_select_kernel<<<static_cast<unsigned>(rows), kTopkThreads, 0, st>>>(
      scores, n, ld, static_cast<int>(k), id_base, out_vals, out_ids, n, 1);
  return cuda_status(cudaGetLastError());
}

extern "C" int tms_topk_pack(const float* vals, const int64_t* ids, int64_t rows, int64_t k,
                             int64_t* packed, void* stream) {
  NvtxRange nvtx_range("tms_topk_pack");
  if (rows < 0 || k < 0) return TMS_ERR_INVALID;
  if (rows * k == 0) return TMS_OK;
  if (!vals || !ids || !packed) return TMS_ERR_INVALID;
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;
  int blocks = static_cast<int>((rows * k + 255) / 256);
  if (blocks > dev->num_sms * 8) blocks = dev->num_sms * 8;
  pack_topk_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(vals, ids, rows, k, packed);
  return cuda_status(cudaGetLastError());
}

extern "C" int tms_topk_merge_packed(const int64_t* gathered, int64_t world, int64_t rows, int64_t k,
                                     float* out_vals, int64_t* out_ids, void* stream) {
  NvtxRange nvtx_range("tms_topk_merge_packed");
  if (world < 1 || rows < 0 || k < 0) return TMS_ERR_INVALID;
  if (rows * k == 0) return TMS_OK;
  if (!gathered || !out_vals || !out_ids) return TMS_ERR_INVALID;
  if (world * k > kSortMax || rows > 0x7fffffffLL) return TMS_ERR_UNSUPPORTED;
  int P = 1;
  while (P < world * k) P <<= 1;
  const size_t smem = static_cast<size_t>(P) * 12;
  if (cudaFuncSetAttribute(merge_packed_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return TMS_ERR_CUDA;
  merge_packed_topk_kernel<<<static_cast<unsigned>(rows), kTopkThreads, smem,
                             static_cast<cudaStream_t>(stream)>>>(
      gathered, static_cast<int>(world), rows, static_cast<int>(k), out_vals, out_ids);
  return cuda_status(cudaGetLastError());
}
