// Flag protocol for kernels that exchange data with other GPUs through
// peer-mapped (symmetric) memory.  A flag is a monotonically increasing 32-bit
// sequence number: the producer publishes `seq` with a system-scope release
// store after its data stores; a consumer polls with system-scope acquire loads
// until the value has reached `seq` (wrap-safe comparison).  Every wait is
// bounded by the peer-flag limit (a run-time value next to the device error
// word, 20 s by default: ranks can be far apart at start-up): on timeout the
// kernel records kErrTimeoutPeer in the error word and gives up instead of
// hanging the GPU.
#pragma once

#include "sm100.cuh"

namespace nq {

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool seq_reached(unsigned v, unsigned seq) {
  return static_cast<int>(v - seq) >= 0;
}

// One thread waits until *f has reached seq.  False on timeout or when another
// thread already recorded an error.
__device__ __forceinline__ bool wait_flag(const unsigned* f, unsigned seq, int* err) {
  if (seq_reached(ld_acquire_sys(f), seq)) return true;
  const uint64_t t0 = globaltimer();
  const uint64_t limit = peer_limit_ns(err);
  uint32_t spins = 0;
  while (!seq_reached(ld_acquire_sys(f), seq)) {
    if ((++spins & 63u) == 0) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (globaltimer() - t0 > limit) {
        atomicCAS(err, 0, kErrTimeoutPeer);
        return false;
      }
    }
  }
  return true;
}

// Whole block: threads t < n wait for flags[t] to reach seq.  Returns false if
// any wait failed.
__device__ __forceinline__ bool block_wait_flags(const unsigned* flags, int n, unsigned seq, int* err) {
  __shared__ int s_fail;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  if (threadIdx.x < n && !wait_flag(flags + threadIdx.x, seq, err)) s_fail = 1;
  __syncthreads();
  return s_fail == 0;
}

// Whole block, at the end of a kernel: counts finished blocks in *counter (a
// monotonically increasing local counter whose value before this launch was
// target - gridDim.x); the last block to finish publishes `seq` into
// dst[r][idx] for every rank r < n (after a system-scope fence, so every
// block's peer stores are visible first).
__device__ __forceinline__ void grid_done_signal(unsigned* counter, unsigned target,
                                                 unsigned* const* dst, int idx, int n, unsigned seq) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned old = atomicAdd(counter, 1u);
    if (old == target - 1u) {
      __threadfence_system();
      for (int r = 0; r < n; ++r) st_release_sys(dst[r] + idx, seq);
    }
  }
}

}  // namespace nq
