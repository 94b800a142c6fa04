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

// Shared-memory flag hand-off: the signaller bumps a per-slot counter with a release store, the
// waiter polls it with acquire loads (bounded like wait_bar).
__device__ __forceinline__ void flag_signal(uint32_t* f) {
  asm volatile("red.release.cta.shared::cta.add.u32 [%0], 1;" ::"r"(smem_u32(f)) : "memory");
}
__device__ __forceinline__ void flag_wait(const uint32_t* f, uint32_t target) {
  for (int i = 0; i < (1 << 26); ++i) {
    uint32_t v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(f)) : "memory");
    if (static_cast<int32_t>(v - target) >= 0) return;
  }
  atomicAdd(&g_gave_up, 1);
}

// Relaxed variant: volatile store / volatile poll (ordering by the fences the caller adds).
__device__ __forceinline__ void vflag_signal(uint32_t* f) {
  __threadfence_block();
  *reinterpret_cast<volatile uint32_t*>(f) = *reinterpret_cast<volatile uint32_t*>(f) + 1u;
}
__device__ __forceinline__ void vflag_wait(const uint32_t* f, uint32_t target) {
  for (int i = 0; i < (1 << 26); ++i)
    if (static_cast<int32_t>(*reinterpret_cast<const volatile uint32_t*>(f) - target) >= 0) {
      __threadfence_block();
      return;
    }
  atomicAdd(&g_gave_up, 1);
}
// Named-barrier hand-off between two whole warps: the signaller arrives, the waiter syncs
// (64 threads). Only usable where both sides always reach the barrier.
__device__ __forceinline__ void nb_arrive(int id) {
  asm volatile("bar.arrive %0, 64;" ::"r"(id) : "memory");
}
__device__ __forceinline__ void nb_sync(int id) {
  asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}

// flags: 1 = tcgen05 fences, 2 = commit in the middle stage, 4 = TMEM load in the consumer,
// 8 = test_wait spin instead of try_wait, 16 = shared-memory flags instead of mbarriers for the
// warp-to-warp hand-offs (producer -> middle, consumer -> producer, and middle -> consumer unless
// the middle stage commits), 32 = relaxed volatile flags instead (with 16), 64 = named barriers
// for all three hand-offs (ids 1 + slot, 5 + slot, 9 + slot; the whole middle warp takes part)
__global__ void handoff_kernel(long long* out, int tiles, int flags) {
  __shared__ __align__(8) uint64_t bars[3 * kSlots];
  __shared__ uint32_t tslot;
  __shared__ uint32_t fl[3 * kSlots];
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
    for (int i = 0; i < 3 * kSlots; ++i) fl[i] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tslot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const bool fences = flags & 1, commit = flags & 2, ld = flags & 4, test = flags & 8, sf = flags & 16;
  const bool vf = flags & 32, nb = flags & 64;
  uint32_t* f_full = fl;
  uint32_t* f_mid = fl + kSlots;
  uint32_t* f_empty = fl + 2 * kSlots;
  const long long t0 = clock64();
  if (warp == 0) {  // producer (decoder)
    for (int j = 0; j < tiles; ++j) {
      const int s = j % kSlots;
      if (nb) {
        if (j >= kSlots) nb_sync(9 + s);
        if (fences) tc_fence_before();
        nb_arrive(1 + s);
        continue;
      }
      if (lane == 0) {
        if (sf && vf) vflag_wait(&f_empty[s], static_cast<uint32_t>(j / kSlots));
        else if (sf) flag_wait(&f_empty[s], static_cast<uint32_t>(j / kSlots));
        else wait_bar(empty(s), ((j / kSlots) & 1u) ^ 1u, test);
      }
      __syncwarp();
      if (fences) tc_fence_before();
      if (lane == 0) {
        if (sf && vf) vflag_signal(&f_full[s]);
        else if (sf) flag_signal(&f_full[s]);
        else mbar_arrive(full(s));
      }
    }
  } else if (warp == 1 && nb) {  // middle, named barriers: the whole warp
    for (int j = 0; j < tiles; ++j) {
      const int s = j % kSlots;
      nb_sync(1 + s);
      if (fences) tc_fence_after();
      nb_arrive(5 + s);
    }
  } else if (warp == 1) {  // middle (MMA issuer)
    if (lane == 0) {
      for (int j = 0; j < tiles; ++j) {
        const int s = j % kSlots;
        if (sf && vf) vflag_wait(&f_full[s], static_cast<uint32_t>(j / kSlots + 1));
        else if (sf) flag_wait(&f_full[s], static_cast<uint32_t>(j / kSlots + 1));
        else wait_bar(full(s), (j / kSlots) & 1u, test);
        if (fences) tc_fence_after();
        if (commit) mma_commit(mid(s));
        else if (sf && vf) vflag_signal(&f_mid[s]);
        else if (sf) flag_signal(&f_mid[s]);
        else mbar_arrive(mid(s));
      }
    }
  } else if (warp == 2) {  // consumer (epilogue)
    float acc = 0.f;
    for (int j = 0; j < tiles; ++j) {
      const int s = j % kSlots;
      if (nb) {
        nb_sync(5 + s);
      } else if (lane == 0) {
        if (sf && vf && !commit) vflag_wait(&f_mid[s], static_cast<uint32_t>(j / kSlots + 1));
        else if (sf && !commit) flag_wait(&f_mid[s], static_cast<uint32_t>(j / kSlots + 1));
        else wait_bar(mid(s), (j / kSlots) & 1u, test);
      }
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
      if (nb) {
        if (j + kSlots < tiles) nb_arrive(9 + s);
      } else if (lane == 0) {
        if (sf && vf) vflag_signal(&f_empty[s]);
        else if (sf) flag_signal(&f_empty[s]);
        else mbar_arrive(empty(s));
      }
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
    for (int flags : {0, 7, 16, 48, 49, 55, 64, 65, 69}) {
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
      printf("threads %3d fences %d commit %d ld %d test_wait %d smem_flags %d volatile %d named_bar %d: %7.1f cycles per slot\n",
             threads, flags & 1, (flags >> 1) & 1, (flags >> 2) & 1, (flags >> 3) & 1, (flags >> 4) & 1,
             (flags >> 5) & 1, (flags >> 6) & 1,
             static_cast<double>(h) / tiles);
    }
  }
  cudaFree(d);
  return 0;
}
