// api.cu -- library-wide host pieces of the C ABI: status strings, the per-device error word,
// device facts, TMA descriptor encoding and the test hooks.
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "tms_device.cuh"
#include "tms_internal.h"

namespace tms {

// One error word per device that loads the library; bounded waits that give up write here.
__device__ uint32_t g_tms_dev_error_word;

namespace {

constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
std::mutex g_dev_mutex;

uint64_t g_timeout_ns = 2000000000ull;  // 2 s
int g_debug_flags = 0;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn get_ctx_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

}  // namespace

void* current_cu_context() {
  CUcontext c = nullptr;
  const CtxGetCurrentFn fn = get_ctx_fn();
  if (fn) fn(&c);
  return c;
}

const DeviceInfo* current_device_info(int* status) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *status = TMS_ERR_CUDA;
    return nullptr;
  }
  // The cached error-word address belongs to the context the module was loaded in: a different
  // current context (after cudaDeviceReset, or a caller's own driver context) looks it up again.
  void* ctx = current_cu_context();
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  DeviceInfo& d = g_devices[dev];
  if (d.device != dev || d.ctx != ctx) {
    DeviceInfo n;
    n.device = dev;
    n.ctx = ctx;
    if (cudaDeviceGetAttribute(&n.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
            cudaSuccess) {
      *status = TMS_ERR_CUDA;
      return nullptr;
    }
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tms_dev_error_word) != cudaSuccess) {
      *status = TMS_ERR_CUDA;
      return nullptr;
    }
    n.err_word = static_cast<uint32_t*>(p);
    d = n;
  }
  *status = TMS_OK;
  return &d;
}

uint64_t wait_timeout_ns() { return g_timeout_ns; }
int debug_flags() { return g_debug_flags; }

int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                   uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner,
                   uint32_t box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return TMS_ERR_CUDA;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TMS_OK : TMS_ERR_CUDA;
}

}  // namespace tms

using namespace tms;

extern "C" const char* tms_strerror(int code) {
  switch (code) {
    case TMS_OK: return "ok";
    case TMS_ERR_INVALID: return "invalid argument";
    case TMS_ERR_UNSUPPORTED: return "unsupported shape or type";
    case TMS_ERR_CUDA: return "CUDA error";
    case TMS_ERR_TIMEOUT: return "device wait timed out";
    case TMS_ERR_WORKSPACE: return "workspace too small";
    case TMS_ERR_TOO_LARGE: return "problem exceeds the no-allocation entry point's static scratch";
    case TMS_ERR_BAD_OFFSETS: return "document offsets negative, decreasing or past the token count";
    default: return "unknown error";
  }
}

extern "C" const char* tms_version(void) { return "tilemaxsim_b200 0.1.0 (sm_100a)"; }

extern "C" int tms_last_device_error(void* stream, uint32_t* detail) {
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t word = 0;
  if (cudaMemcpyAsync(&word, dev->err_word, sizeof(word), cudaMemcpyDeviceToHost, st) !=
      cudaSuccess)
    return TMS_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return TMS_ERR_CUDA;
  if (word != 0) {
    const uint32_t zero = 0;
    if (cudaMemcpyAsync(dev->err_word, &zero, sizeof(zero), cudaMemcpyHostToDevice, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
      return TMS_ERR_CUDA;
  }
  if (detail) *detail = word;
  if (word & kDevErrTimeout) return TMS_ERR_TIMEOUT;
  return word ? TMS_ERR_BAD_OFFSETS : TMS_OK;
}

namespace tms {
namespace {
__global__ void validate_offsets_kernel(const int64_t* __restrict__ off, int64_t n_docs,
                                        int64_t n_tokens, uint32_t* err) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i <= n_docs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t v = off[i];
    const bool bad = v < 0 || v > n_tokens || (i > 0 && off[i - 1] > v);
    if (bad) atomicCAS(err, 0u, kDevErrBadInput | static_cast<uint32_t>(i < 0x3fffffff ? i : 0x3fffffff));
  }
}
}  // namespace
}  // namespace tms

extern "C" int tms_validate_offsets(const int64_t* doc_offsets, int64_t n_docs, int64_t n_tokens,
                                    void* stream) {
  if (n_docs < 0 || n_tokens < 0 || !doc_offsets) return TMS_ERR_INVALID;
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;
  NvtxRange range("tms_validate_offsets");
  const int64_t n = n_docs + 1;
  int blocks = static_cast<int>((n + 255) / 256);
  if (blocks > dev->num_sms * 8) blocks = dev->num_sms * 8;
  tms::validate_offsets_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      doc_offsets, n_docs, n_tokens, dev->err_word);
  return cuda_status(cudaGetLastError());
}

// Test hook: wait limit for the bounded device waits (0 keeps the current value) and fault flags
// (bit 0: the dense kernel's producer issues no load, so its consumers' waits run out).
extern "C" void tms_set_debug(uint64_t timeout_ns, int flags) {
  if (timeout_ns) g_timeout_ns = timeout_ns;
  g_debug_flags = flags;
}
