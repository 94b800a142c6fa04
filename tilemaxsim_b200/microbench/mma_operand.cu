// mma_operand.cu -- issue rate of tcgen05.mma (kind::f16, M = 128, K = 16) on one B200 SM with the
// A operand in shared memory (descriptor) or in TMEM, for N = 32 ... 256. The token-rows PQ kernel
// puts decoded tokens in TMEM as A with a small N (the query rows); this measures what that costs
// against the shared-memory form.
//
// One CTA per SM; one thread issues `iters` x 8 MMAs into a 256-column accumulator (operand values
// are whatever the buffers hold: only the timing matters), commits to an mbarrier and waits for it
// (bounded). Prints cycles per MMA and the operand bytes per cycle that rate implies.
#include <cstdint>
#include <cstdio>

#include "../csrc/tms_device.cuh"

using namespace tms;

__device__ int g_timeouts;

template <bool A_TMEM>
__global__ void mma_operand_kernel(long long* out, int iters, int N) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tslot;
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tslot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0 && lane == 0) {
    // operand buffers on a 1024-byte boundary (the 128-byte swizzle atoms need it)
    const uint32_t a_s = (smem_u32(smem) + 1023u) & ~1023u;  // 128 rows x 128 B (A)
    const uint32_t b_s = a_s + 128 * 128;           // 256 rows x 128 B (B)
    const uint32_t idesc = make_idesc(128, N, 0u);
    const uint32_t d_tmem = tslot;                  // columns [0, N)
    const uint32_t a_tmem = tslot + 256u;           // columns [256, 320): A, 2 fp16 per column
    const uint64_t ad0 = sw128_kmajor_desc(a_s), bd0 = sw128_kmajor_desc(b_s);
    const long long t0 = clock64();
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        // K steps 0-3 within the first 128-byte chunk, 4-7 repeat them (timing only)
        const uint32_t kk = static_cast<uint32_t>(k & 3);
        if (A_TMEM)
          mma_f16_ts(d_tmem, a_tmem + 8u * k, bd0 + 2u * kk, idesc, (it | k) != 0);
        else
          mma_f16(d_tmem, ad0 + 2u * kk, bd0 + 2u * kk, idesc, (it | k) != 0);
      }
    }
    mma_commit(smem_u32(&bar));
    if (!mbar_wait(smem_u32(&bar), 0, &abort_flag, 2000000000ull, reinterpret_cast<uint32_t*>(&g_timeouts), 1))
      atomicAdd(&g_timeouts, 1);
    const long long t1 = clock64();
    out[blockIdx.x] = t1 - t0;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tslot, 512);
  }
}

template <bool A_TMEM>
static int run(long long* d, int sms, int N) {
  const int iters = 2000;
  const size_t smem = 128 * 128 + 256 * 128 + 1024;
  cudaFuncSetAttribute(mma_operand_kernel<A_TMEM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  for (int rep = 0; rep < 2; ++rep) mma_operand_kernel<A_TMEM><<<sms, 128, smem>>>(d, iters, N);
  if (cudaDeviceSynchronize() != cudaSuccess) {
    printf("N=%d failed\n", N);
    return 1;
  }
  long long h = 0;
  cudaMemcpy(&h, d, sizeof(long long), cudaMemcpyDeviceToHost);
  const double per = static_cast<double>(h) / (iters * 8.0);
  const double a_bytes = 128 * 16 * 2, b_bytes = N * 16 * 2;
  printf("A in %-5s N=%3d: %6.1f cycles per MMA (ideal %5.1f at 8192 FLOP/clk); A %6.1f B/clk, B %6.1f B/clk\n",
         A_TMEM ? "TMEM" : "smem", N, per, 128.0 * N * 16 * 2 / 8192.0, a_bytes / per, b_bytes / per);
  return 0;
}

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  long long* d = nullptr;
  cudaMalloc(&d, sizeof(long long) * sms);
  int rc = 0;
  for (int N : {32, 64, 128, 256}) {
    rc |= run<false>(d, sms, N);
    rc |= run<true>(d, sms, N);
  }
  int timeouts = 0;
  cudaMemcpyFromSymbol(&timeouts, g_timeouts, sizeof(int));
  if (timeouts) printf("(%d waits timed out)\n", timeouts);
  cudaFree(d);
  return rc;
}
