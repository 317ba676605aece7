// dcn_offset.cu -- the offset convolution of the DCNv2 Pack module
// (modulated_deform_conv/dcn_split_nhwc.py:171-172: conv2d(x, w_off, b_off)
// with the DCN's kernel size, stride, padding and dilation and 3T output
// channels) finished from its per-tap partial products.
//
// The offset convolution has only 3T = 27 output channels, which makes it a
// poor fit for a convolution library's implicit GEMM (cuDNN takes 21 us at
// the stage-4 shape on B200).  Its channel reduction is instead one plain
// GEMM over the input pixels, z[p, t*3T + c] = sum_ci x[p, ci] * w_off[c, ci, t]
// (fp32 output), and this kernel adds the T shifted taps:
//   y[m, c] = round_T(bias[c] + sum_t z[p_t(m), t*3T + c]),
// where p_t(m) is output pixel m's input pixel under tap t (taps outside the
// image contribute nothing, the convolution's zero padding).  y is what the
// unfused path's offset-conv output holds (fp32 sum, one rounding to the
// input dtype) and feeds the fused DCN kernel as offsets (channels [0, 2T))
// and pre-sigmoid mask (channels [2T, 3T)).
//
// One thread per (m, c); consecutive threads take consecutive channels, so a
// warp reads contiguous runs of z rows and writes contiguous y.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "bevk_internal.h"
#include "bevk_ptx.cuh"

namespace bevk {
namespace {

constexpr int kMaxTapsSum = 9;

template <typename T>
__device__ __forceinline__ T round_to(float v);
template <>
__device__ __forceinline__ __half round_to<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 round_to<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ float round_to<float>(float v) { return v; }

struct SumParams {
  int H, W, Ho, Wo, kW, T, c3;
  int sh, sw, ph, pw, dh, dw;
  int total;   // B*Ho*Wo*3T
  int ld;
};

template <typename T>
__global__ void __launch_bounds__(256) dcn_offset_sum_kernel(const SumParams p,
                                                             const float *__restrict__ z,
                                                             const float *__restrict__ bias,
                                                             T *__restrict__ y) {
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.total; i += gridDim.x * blockDim.x) {
    const int m = i / p.c3;
    const int c = i - m * p.c3;
    const int bo = m / p.Wo;
    const int ow = m - bo * p.Wo;
    const int b = bo / p.Ho;
    const int oh = bo - b * p.Ho;
    float v[kMaxTapsSum];
    int ui = 0, uj = 0;
    // every tap's load is issued before the sum (a tap outside the image
    // reads z[0] and is dropped by the select)
#pragma unroll
    for (int u = 0; u < kMaxTapsSum; ++u) {
      const int ih = oh * p.sh - p.ph + ui * p.dh;
      const int iw = ow * p.sw - p.pw + uj * p.dw;
      const bool in = u < p.T && ih >= 0 && ih < p.H && iw >= 0 && iw < p.W;
      const int64_t pix = (b * p.H + ih) * p.W + iw;
      const float zv = __ldg(z + (in ? pix * p.ld + (u * p.c3 + c) : 0));
      v[u] = in ? zv : 0.f;
      if (++uj == p.kW) {
        uj = 0;
        ++ui;
      }
    }
    float acc = bias != nullptr ? bias[c] : 0.f;
#pragma unroll
    for (int u = 0; u < kMaxTapsSum; ++u) acc += v[u];
    y[i] = round_to<T>(acc);
  }
}

}  // namespace

int launch_dcn_offset_sum(const bevk_dcn_problem *pr, const DcnDims &d, const float *z,
                          int64_t ld, const float *bias, void *y, cudaStream_t stream) {
  if (d.T > kMaxTapsSum)
    return fail(BEVK_ERR_UNSUPPORTED, "dcn offset sum: kernel of %d taps (at most %d)", d.T,
                kMaxTapsSum);
  SumParams p;
  p.H = d.H; p.W = d.W; p.Ho = d.Ho; p.Wo = d.Wo; p.kW = d.kW; p.T = d.T; p.c3 = 3 * d.T;
  p.sh = d.sh; p.sw = d.sw; p.ph = d.ph; p.pw = d.pw; p.dh = d.dh; p.dw = d.dw;
  if (d.M * 3 * d.T >= (int64_t(1) << 31) || ld >= (int64_t(1) << 31))
    return fail(BEVK_ERR_INDEX_OVERFLOW, "dcn offset sum: %lld outputs exceed 31-bit indexing",
                static_cast<long long>(d.M * 3 * d.T));
  p.total = static_cast<int>(d.M * p.c3);
  p.ld = static_cast<int>(ld);
  if (p.total == 0) return BEVK_OK;
  const int dev = current_device();
  if (dev < 0) return fail(BEVK_ERR_CUDA, "dcn offset sum: no device");
  const int64_t want = (p.total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(device_info(dev).sm_count) * 8;
  const int grid = static_cast<int>(want < cap ? want : cap);
  switch (pr->dtype) {
    case BEVK_DTYPE_F16:
      return launched(launch_dependent(dcn_offset_sum_kernel<__half>, dim3(grid), dim3(256), 0,
                                       stream, p, z, bias, static_cast<__half *>(y)),
                      "dcn_offset_sum_kernel");
    case BEVK_DTYPE_BF16:
      return launched(launch_dependent(dcn_offset_sum_kernel<__nv_bfloat16>, dim3(grid), dim3(256),
                                       0, stream, p, z, bias, static_cast<__nv_bfloat16 *>(y)),
                      "dcn_offset_sum_kernel");
    case BEVK_DTYPE_F32:
      return launched(launch_dependent(dcn_offset_sum_kernel<float>, dim3(grid), dim3(256), 0,
                                       stream, p, z, bias, static_cast<float *>(y)),
                      "dcn_offset_sum_kernel");
    default:
      return fail(BEVK_ERR_UNSUPPORTED, "dcn offset sum: dtype %d", pr->dtype);
  }
  return check_launch("dcn_offset_sum_kernel");
}

}  // namespace bevk
