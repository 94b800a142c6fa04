// tmem_read.cu -- measures the TMEM -> register read bandwidth of one B200 SM (tcgen05.ld), the
// resource that bounds the dense MaxSim epilogue: every fp32 similarity value the MMA writes to
// TMEM is read once by the epilogue warps.
//
// Each CTA (one per SM) allocates all 512 TMEM columns; `nwarps` warps (lane quarter = warp % 4)
// repeatedly load 4 KB (32 lanes x 32 columns, or 16 lanes x 64 columns) and wait, timed with
// clock64. Prints cycles per load and bytes per clock per SM for each load shape and warp count.
#include <cstdint>
#include <cstdio>

#include "../csrc/tms_device.cuh"

using namespace tms;

#define R32 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}"
#define O32(r)                                                                                  \
  "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), \
      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),    \
      "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),  \
      "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),  \
      "=r"(r[29]), "=r"(r[30]), "=r"(r[31])

template <int SHAPE>
__device__ __forceinline__ void ld_wait(uint32_t a, uint32_t (&r)[32]) {
  if (SHAPE == 0)
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 " R32 ", [%32];\n\ttcgen05.wait::ld.sync.aligned;"
                 : O32(r) : "r"(a) : "memory");
  else
    asm volatile("tcgen05.ld.sync.aligned.16x256b.x8.b32 " R32 ", [%32];\n\ttcgen05.wait::ld.sync.aligned;"
                 : O32(r) : "r"(a) : "memory");
}

template <int SHAPE>
__global__ void tmem_read_kernel(long long* out, int iters, int nwarps) {
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    tmem_alloc(smem_u32(&slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t base = slot + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  float acc = 0.f;
  const long long t0 = clock64();
  if (warp >= 2 && warp < 2 + nwarps) {
    for (int i = 0; i < iters; ++i) {
      uint32_t r[32];
      ld_wait<SHAPE>(base + (i * 32) % 256, r);
      acc += __uint_as_float(r[i & 31]);
    }
  }
  const long long t1 = clock64();
  if (lane == 0) out[blockIdx.x * 16 + warp] = t1 - t0;
  if (acc == 12345.f) out[0] = 0;  // keeps the loads live
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(slot, 512);
  }
}

template <int S>
static int run(long long* d, int sms, int nw, const char* name) {
  static long long h[1024 * 16];
  const int iters = 4096;
  for (int rep = 0; rep < 2; ++rep) tmem_read_kernel<S><<<sms, 320>>>(d, iters, nw);
  const cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    printf("%s: %s\n", name, cudaGetErrorString(e));
    return 1;
  }
  cudaMemcpy(h, d, sizeof(long long) * sms * 16, cudaMemcpyDeviceToHost);
  const double c = h[2] / static_cast<double>(iters);
  printf("%-12s warps=%d  %7.1f cycles per 4 KB load per warp  ->  %5.1f B/clk per SM\n", name, nw, c,
         nw * 4096.0 / c);
  return 0;
}

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  long long* d = nullptr;
  cudaMalloc(&d, sizeof(long long) * sms * 16);
  int rc = 0;
  for (int nw : {1, 4, 8}) {
    rc |= run<0>(d, sms, nw, "32x32b.x32");
    rc |= run<1>(d, sms, nw, "16x256b.x8");
  }
  cudaFree(d);
  return rc;
}
