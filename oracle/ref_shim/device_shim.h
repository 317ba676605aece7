// device_shim.h -- lets the reference's MSDA kernel header
// (csrc_musa/msda/ms_deform_attn_kernels.cuh, compiled from where it lies)
// build as single-threaded host C++ for the oracle's reference check.  TEST
// INFRASTRUCTURE ONLY.
//
// A "launch" is one host call with a grid of one block of one thread, so the
// header's grid-stride loops (MSDA_1D_KERNEL_LOOP) visit every index in order.
// Only the generic forward kernel (ms_deformable_im2col_generic_kernel) is
// called; the warp-level kernels of the header only need to compile, so the
// warp and block intrinsics below are inert stand-ins.
#pragma once
#include <cmath>
#include <cstdint>

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __shared__
#define __restrict__

struct bevk_ref_dim3 {
  unsigned int x, y, z;
};
static const bevk_ref_dim3 threadIdx = {0, 0, 0};
static const bevk_ref_dim3 blockIdx = {0, 0, 0};
static const bevk_ref_dim3 blockDim = {1, 1, 1};
static const bevk_ref_dim3 gridDim = {1, 1, 1};

inline void __syncthreads() {}
inline void __syncwarp(unsigned = 0xffffffffu) {}
template <typename T>
inline T __shfl_down_sync(unsigned, T v, int, int = 32) { return v; }
template <typename T>
inline T atomicAdd(T *p, T v) {
  const T old = *p;
  *p = old + v;
  return old;
}

typedef _Float16 __half;
inline float __half2float(__half h) { return static_cast<float>(h); }
inline __half __float2half(float f) { return static_cast<__half>(f); }
