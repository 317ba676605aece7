// device_shim.h -- lets the reference's MSDA kernel header
// (csrc_musa/msda/ms_deform_attn_kernels.cuh, compiled from where it lies)
// build as single-threaded host C++ for the oracle's reference check.  TEST
// INFRASTRUCTURE ONLY.
//
// A "launch" is one host call over a grid of one block.  The forward kernel
// runs with one thread (blockDim.x = 1), so the header's grid-stride loops
// (MSDA_1D_KERNEL_LOOP) visit every index in order.  The generic backward
// kernel (ms_deformable_col2im_shm_stride_v1_kernel) is block-cooperative: it
// runs as blockDim.x host threads, each with its own threadIdx, meeting at a
// barrier for __syncthreads and adding to grad_value with compare-and-swap
// atomics.  The warp-level kernels of the header only need to compile, so the
// warp intrinsics below are inert stand-ins.
#pragma once
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <mutex>

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __shared__
#define __restrict__

struct bevk_ref_dim3 {
  unsigned int x, y, z;
};
inline thread_local bevk_ref_dim3 threadIdx = {0, 0, 0};
inline bevk_ref_dim3 blockDim = {1, 1, 1};
static const bevk_ref_dim3 blockIdx = {0, 0, 0};
static const bevk_ref_dim3 gridDim = {1, 1, 1};

// The emulated block's barrier: all blockDim.x threads arrive, then all go on.
struct bevk_ref_barrier {
  std::mutex mu;
  std::condition_variable cv;
  unsigned count = 0, generation = 0, parties = 1;
  void wait() {
    std::unique_lock<std::mutex> lk(mu);
    const unsigned gen = generation;
    if (++count == parties) {
      count = 0;
      ++generation;
      cv.notify_all();
    } else {
      cv.wait(lk, [&] { return gen != generation; });
    }
  }
};
inline bevk_ref_barrier bevk_ref_block_barrier;

inline void __syncthreads() {
  if (blockDim.x > 1) bevk_ref_block_barrier.wait();
}
inline void __syncwarp(unsigned = 0xffffffffu) {}
template <typename T>
inline T __shfl_down_sync(unsigned, T v, int, int = 32) { return v; }
// Atomic add of a 4-byte float (or int) by compare-and-swap on its bits.
template <typename T>
inline T atomicAdd(T *p, T v) {
  static_assert(sizeof(T) == 4, "4-byte atomics only");
  uint32_t *q = reinterpret_cast<uint32_t *>(p);
  uint32_t old_bits = __atomic_load_n(q, __ATOMIC_RELAXED);
  for (;;) {
    T old;
    std::memcpy(&old, &old_bits, 4);
    const T nv = old + v;
    uint32_t new_bits;
    std::memcpy(&new_bits, &nv, 4);
    if (__atomic_compare_exchange_n(q, &old_bits, new_bits, false, __ATOMIC_RELAXED,
                                    __ATOMIC_RELAXED))
      return old;
  }
}

typedef _Float16 __half;
inline float __half2float(__half h) { return static_cast<float>(h); }
inline __half __float2half(float f) { return static_cast<__half>(f); }
