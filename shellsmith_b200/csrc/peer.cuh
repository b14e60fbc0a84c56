// Device helpers for exchanges over NVLink peer memory: system-scope release
// and acquire on 32-bit epoch flags, and a bounded wait on a set of flags.
#pragma once
#include "common.cuh"

namespace sc {

// Flag words hold epochs that grow by one per exchange; comparisons are
// modulo 2^32 so an epoch counter may wrap.
constexpr uint32_t kPeerSpinLimit = 1u << 24;  // ~seconds with the back-off below

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Where a merge kernel sends its rows: local is this rank's packed block
// (16-byte aligned, a multiple of 16 bytes), dst[p] rank p's receive slot for
// this rank, flag[p] rank p's flag for this rank; counter is a local word,
// zero between launches.
struct PeerPut {
  float* local = nullptr;
  float* const* dst = nullptr;
  unsigned int* const* flag = nullptr;
  unsigned int* counter = nullptr;
  const unsigned int* epoch_base = nullptr;
  unsigned int epoch_add = 0;
  int world = 0;
};

// What a merge kernel waits for: flags[r] (rank r's flag on this rank) to reach
// *epoch_base + epoch_add for every r < world.
struct PeerWait {
  const unsigned int* flags = nullptr;
  const unsigned int* epoch_base = nullptr;
  unsigned int epoch_add = 0;
  int world = 0;
  unsigned int* status = nullptr;
};

// Called by one thread: returns once flags[r] has reached `want` for every
// r < world. After `limit` polls of one flag (or when an earlier wait on this
// device already gave up) it flags DEV_WAIT_TIMEOUT and returns false.
__device__ __forceinline__ bool wait_epochs(const unsigned int* flags, int world,
                                            unsigned int want, unsigned int* status,
                                            uint32_t limit = kPeerSpinLimit) {
  if (status != nullptr && (*reinterpret_cast<volatile unsigned int*>(status) & DEV_WAIT_TIMEOUT))
    return false;
  for (int r = 0; r < world; ++r) {
    uint32_t i = 0;
    while ((int)(ld_acquire_sys(flags + r) - want) < 0) {
      if (++i >= limit) {
        flag_device(status, DEV_WAIT_TIMEOUT);
        return false;
      }
      if (i > 64) __nanosleep(64);
    }
  }
  return true;
}

}  // namespace sc
