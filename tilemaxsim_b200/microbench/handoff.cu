// handoff.cu -- cost of one pipeline hand-off between warps on one B200 SM: a ring of 4 slots
// passed producer warp -> middle warp (one thread) -> consumer warp -> producer through mbarriers,
// the shape of a decode -> MMA -> epilogue pipeline. Variants add the pieces such a pipeline uses
// one at a time: tcgen05 thread-sync fences, tcgen05.commit as the middle stage's arrive, a TMEM
// load in the consumer, and the wait flavour (try_wait / test_wait spin). Prints cycles per slot.
#include <cstdint>
#include <cstdio>

#include "../csrc/tms_device.cuh"

using namespace tms;

constexpr int kSlots = 4;

// Bounded: gives up after 2^26 polls (far beyond any hand-off here) and counts the give-up.
__device__ int g_gave_up;
__device__ __forceinline__ void wait_bar(uint32_t bar, uint32_t parity, bool test) {
  for (int i = 0; i < (1 << 26); ++i)
    if (test ? mbar_test_wait(bar, parity) : mbar_try_wait(bar, parity)) return;
  atomicAdd(&g_gave_up, 1);
}

// flags: 1 = tcgen05 fences, 2 = commit in the middle stage, 4 = TMEM load in the consumer,
// 8 = test_wait spin instead of try_wait
__global__ void handoff_kernel(long long* out, int tiles, int flags) {
  __shared__ __align__(8) uint64_t bars[3 * kSlots];
  __shared__ uint32_t tslot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t b0 = smem_u32(bars);
  auto full = [&](int s) { return b0 + 8u * s; };
  auto mid = [&](int s) { return b0 + 8u * (kSlots + s); };
  auto empty = [&](int s) { return b0 + 8u * (2 * kSlots + s); };
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(full(s), 1);
      mbar_init(mid(s), 1);
      mbar_init(empty(s), 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tslot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const bool fences = flags & 1, commit = flags & 2, ld = flags & 4, test = flags & 8;
  const long long t0 = clock64();
  if (warp == 0) {  // producer (decoder)
    for (int j = 0; j < tiles; ++j) {
      const int s = j % kSlots;
      if (lane == 0) wait_bar(empty(s), ((j / kSlots) & 1u) ^ 1u, test);
      __syncwarp();
      if (fences) tc_fence_before();
      if (lane == 0) mbar_arrive(full(s));
    }
  } else if (warp == 1) {  // middle (MMA issuer)
    if (lane == 0) {
      for (int j = 0; j < tiles; ++j) {
        const int s = j % kSlots;
        wait_bar(full(s), (j / kSlots) & 1u, test);
        if (fences) tc_fence_after();
        if (commit) mma_commit(mid(s));
        else mbar_arrive(mid(s));
      }
    }
  } else if (warp == 2) {  // consumer (epilogue)
    float acc = 0.f;
    for (int j = 0; j < tiles; ++j) {
      const int s = j % kSlots;
      if (lane == 0) wait_bar(mid(s), (j / kSlots) & 1u, test);
      __syncwarp();
      if (fences) tc_fence_after();
      if (ld) {
        uint32_t r[32];
        tmem_ld32_async(tslot + (static_cast<uint32_t>(2 * 32) << 16) + 32u * s, r);
        tmem_wait_ld32(r);
        acc += __uint_as_float(r[j & 31]);
      }
      if (fences) tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(empty(s));
    }
    if (acc == 12345.f) out[1] = 0;
  }
  const long long t1 = clock64();
  if (threadIdx.x == 64) out[0] = t1 - t0;
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tslot, 512);
  }
}

int main() {
  long long* d = nullptr;
  cudaMalloc(&d, 2 * sizeof(long long));
  const int tiles = 20000;
  for (int threads : {96, 512}) {
    for (int flags : {0, 1, 2, 3, 7, 8, 15}) {
      long long h = 0;
      for (int rep = 0; rep < 2; ++rep) handoff_kernel<<<1, threads>>>(d, tiles, flags);
      if (cudaDeviceSynchronize() != cudaSuccess) {
        printf("flags %d: failed\n", flags);
        return 1;
      }
      cudaMemcpy(&h, d, sizeof(long long), cudaMemcpyDeviceToHost);
      int gave_up = 0;
      cudaMemcpyFromSymbol(&gave_up, g_gave_up, sizeof(int));
      if (gave_up) printf("(%d waits gave up)\n", gave_up);
      printf("threads %3d fences %d commit %d ld %d test_wait %d: %7.1f cycles per slot\n", threads,
             flags & 1, (flags >> 1) & 1, (flags >> 2) & 1, (flags >> 3) & 1,
             static_cast<double>(h) / tiles);
    }
  }
  cudaFree(d);
  return 0;
}
