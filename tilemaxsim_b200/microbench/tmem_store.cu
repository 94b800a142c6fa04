// tmem_store.cu -- measures the register -> TMEM write bandwidth of one B200 SM (tcgen05.st), the
// resource a kernel pays when it builds an MMA operand in TMEM from registers (the single-query PQ
// kernel writes every decoded token row there), alone and while other warps read TMEM.
//
// Each CTA (one per SM) allocates all 512 TMEM columns. `nst` warps store 4 KB each (32 lanes x
// 32 columns) per iteration and wait for the store; `nld` other warps read 4 KB per iteration at
// the same time. Timed with clock64; prints bytes per clock per SM for each direction.
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
#define I32(r)                                                                                  \
  "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),         \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),           \
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),         \
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),         \
      "r"(r[29]), "r"(r[30]), "r"(r[31])
#define S32 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32}"

__global__ void tmem_store_kernel(long long* out, int iters, int nst, int nld) {
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    tmem_alloc(smem_u32(&slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t q = static_cast<uint32_t>((warp & 3) * 32) << 16;
  float acc = 0.f;
  uint32_t v[32];
  for (int i = 0; i < 32; ++i) v[i] = static_cast<uint32_t>(lane * 32 + i + warp);
  const long long t0 = clock64();
  if (warp < nst) {
    // store warps write columns [0, 256) (their own column block per warp group of four)
    const uint32_t base = slot + q + static_cast<uint32_t>((warp >> 2) * 64);
    for (int i = 0; i < iters; ++i) {
      asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], " S32 ";\n\ttcgen05.wait::st.sync.aligned;"
                   ::"r"(base + (i & 1) * 32), I32(v) : "memory");
      v[i & 31] += 1u;
    }
  } else if (warp >= 8 && warp < 8 + nld) {
    // load warps read columns [256, 512)
    const uint32_t base = slot + q + 256u;
    for (int i = 0; i < iters; ++i) {
      uint32_t r[32];
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 " R32 ", [%32];\n\ttcgen05.wait::ld.sync.aligned;"
                   : O32(r) : "r"(base + (i * 32) % 256) : "memory");
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

static int run(long long* d, int sms, int nst, int nld) {
  static long long h[1024 * 16];
  const int iters = 4096;
  for (int rep = 0; rep < 2; ++rep) tmem_store_kernel<<<sms, 512>>>(d, iters, nst, nld);
  const cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    printf("st=%d ld=%d: %s\n", nst, nld, cudaGetErrorString(e));
    return 1;
  }
  cudaMemcpy(h, d, sizeof(long long) * sms * 16, cudaMemcpyDeviceToHost);
  double st_bpc = 0, ld_bpc = 0;
  if (nst) st_bpc = nst * 4096.0 / (h[0] / static_cast<double>(iters));
  if (nld) ld_bpc = nld * 4096.0 / (h[8] / static_cast<double>(iters));
  printf("store warps=%d load warps=%d  ->  store %5.1f B/clk per SM, load %5.1f B/clk per SM\n", nst, nld,
         st_bpc, ld_bpc);
  return 0;
}

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  long long* d = nullptr;
  cudaMalloc(&d, sizeof(long long) * sms * 16);
  int rc = 0;
  rc |= run(d, sms, 1, 0);
  rc |= run(d, sms, 4, 0);
  rc |= run(d, sms, 8, 0);
  rc |= run(d, sms, 0, 4);
  rc |= run(d, sms, 4, 4);
  rc |= run(d, sms, 8, 4);
  cudaFree(d);
  return rc;
}
