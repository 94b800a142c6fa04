// tms_internal.h -- host-side helpers shared by the library's translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <nvtx3/nvToolsExt.h>

#include <cstddef>
#include <cstdint>

#include "../../include/tilemaxsim.h"

namespace tms {

// Per-device facts and the address of the device error word (set up once per device).
struct DeviceInfo {
  int device = -1;
  void* ctx = nullptr;  // the CUcontext current when the entry was filled in
  int num_sms = 0;
  int max_smem_optin = 0;
  uint32_t* err_word = nullptr;
};
// Returns nullptr (and sets *status) when the current device cannot be queried.
const DeviceInfo* current_device_info(int* status);
// The calling thread's current CUcontext (nullptr when none): addresses of __device__ variables
// are only valid in the context they were looked up in.
void* current_cu_context();

// Wait limit for the bounded mbarrier waits, in nanoseconds (default 2 s; tms_set_debug changes it).
uint64_t wait_timeout_ns();
// Test hook flags (tms_set_debug); 0 in normal operation.
int debug_flags();

// Encodes a 2-D row-major tensor map: `rows` rows of `inner` elements, row stride in bytes, box of
// box_inner x box_rows elements, 128-byte swizzle, zero fill outside the tensor.
int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                   uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner,
                   uint32_t box_rows);

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? TMS_OK : TMS_ERR_CUDA; }

// NVTX range around an entry point (named in Nsight Systems / Compute timelines; a no-op costing a
// few nanoseconds when no tool is attached).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Tensor-core PQ path (dense kernel with decoder warps), defined in dense_maxsim.cu. Q is fp16.
// pq_mma_codebook_bytes returns 0 when the shape does not fit that path.
size_t pq_mma_codebook_bytes(int64_t M, int64_t K, int64_t dsub);
size_t pq_mma_workspace_size(int64_t n_queries, int64_t nq, int64_t d, int64_t n_docs);
int pq_mma_maxsim(const void* Q, int64_t n_queries, int64_t nq, const void* codebook, int cb_dtype,
                  int64_t M, int64_t K, int64_t dsub, const uint8_t* codes, int64_t n_tokens,
                  const int64_t* doc_offsets, int64_t n_docs, int64_t nd_uniform, float* out,
                  void* workspace, size_t workspace_bytes, cudaStream_t st);

// Tensor-core PQ path for small query batches (<= 2 chunks of 32 query rows), tokens on the TMEM
// lanes; defined in pq_tokrows.cu. Q is fp16. `split`: the codebook as fp16 hi + fp16 lo (about 22
// significant bits, the fp32 reference's precision) instead of rounded to fp16. Returns
// TMS_ERR_UNSUPPORTED for shapes it does not take.
size_t pq_tokrows_workspace_size(int64_t n_queries, int64_t nq, int64_t n_docs);
int pq_tokrows_maxsim(const void* Q, int64_t n_queries, int64_t nq, const void* codebook,
                      int cb_dtype, int64_t M, int64_t K, int64_t dsub, const uint8_t* codes,
                      int64_t n_tokens, const int64_t* doc_offsets, int64_t n_docs,
                      int64_t nd_uniform, float* out, void* workspace, size_t workspace_bytes,
                      cudaStream_t st, bool split);
// Residual-compressed corpora on the token-rows kernel (up to four 32-row query chunks, d = 64 or
// 128); TMS_ERR_UNSUPPORTED for other shapes (the caller then takes the dense decoder kernel).
int res_tokrows_maxsim(const void* Q, int64_t n_queries, int64_t nq, int64_t d,
                       const void* centroids, int64_t n_centroids, const int32_t* codes,
                       const uint8_t* residuals, const float* bucket_weights, int nbits,
                       int normalize, int64_t n_tokens, const int64_t* doc_offsets, int64_t n_docs,
                       int64_t nd_uniform, float* out, void* workspace, size_t workspace_bytes,
                       cudaStream_t st);

}  // namespace tms
