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

__global__ void __launch_bounds__(kTopkThreads)
    topk_select_kernel(const float* __restrict__ scores, int64_t n, int64_t ld, int k,
                       int64_t id_base, float* __restrict__ out_vals,
                       int64_t* __restrict__ out_ids) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_mask, s_remaining;
  __shared__ uint32_t s_gt_pos, s_taken;
  __shared__ uint32_t warp_cnt[32];
  __shared__ int64_t cand_ids[kMaxK];
  __shared__ uint32_t cand_keys[kMaxK];
  const int64_t row = blockIdx.x;
  const float* s = scores + row * ld;
  const int tid = threadIdx.x;
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
  for (int i = tid; i < k; i += blockDim.x) {
    out_vals[row * k + i] = key2f(cand_keys[i]);
    out_ids[row * k + i] = cand_ids[i] + id_base;
  }
}

}  // namespace
}  // namespace tms

using namespace tms;

extern "C" size_t tms_topk_workspace_size(int64_t rows, int64_t n, int64_t k) {
  (void)rows;
  (void)n;
  (void)k;
  return 0;
}

extern "C" int tms_topk(const float* scores, int64_t rows, int64_t n, int64_t ld, int64_t k,
                        const int64_t* ids_in, int64_t ld_ids, int64_t id_base, float* out_vals,
                        int64_t* out_ids, void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
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
  topk_select_kernel<<<static_cast<unsigned>(rows), kTopkThreads, 0, st>>>(
      scores, n, ld, static_cast<int>(k), id_base, out_vals, out_ids);
  return cuda_status(cudaGetLastError());
}
