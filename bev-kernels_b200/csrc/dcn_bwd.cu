// dcn_bwd.cu -- DCNv2 backward column scatter (col2im + coordinate gradients).
//
// Semantics are those of the reference's backward goldens
// (modulated_deform_conv/modulated_deform_conv.py:269-312: autograd through the
// differentiable im2col golden :184-266) and its CUDA ops
// modulated_deformable_col2im[_opt|_smem] / _col2im_coord[_opt]
// (csrc/binding.cpp:13-62) and the NHWC col2im family (:80-140,
// modulated_deform_conv/dcn_split_nhwc.py:48-120).  With the column gradient
// dcol[m, c, t] (m = output pixel, c = input channel, t = tap) and, for a sample
// inside the gate -1 < h < H, -1 < w < W, corner weights w1..w4 = hh*hw, hh*lw,
// lh*hw, lh*lw over the in-range corner values v1..v4 (0 outside):
//   grad_input[b, c, corner k]  += dcol * mask * wk
//   grad_offset_h[m, gi, t]     += mask * sum_c dcol * (-hw v1 - lw v2 + hw v3 + lw v4)
//   grad_offset_w[m, gi, t]     += mask * sum_c dcol * (-hh v1 + hh v2 - lh v3 + lh v4)
//   grad_mask[m, gi, t]         += sum_c dcol * (w1 v1 + w2 v2 + w3 v3 + w4 v4)
// (times sigmoid'(z) when the mask is given as pre-sigmoid logits z), sums over
// the channels c of deformable group gi.
//
// Design: one warp per (pixel, deformable group, tap); the warp's lanes cover
// the group's channels as 4-channel vectors when the input, the column
// gradient and grad_input are channel-contiguous (NHWC), else one channel per
// lane.  The geometry is computed once per warp; grad_input takes fp32 vector
// atomics (red.global.add.v4.f32) at the four corner lines and the three
// per-sample sums are folded with shuffles, so grad_offset / grad_mask need no
// atomics (each (pixel, group, tap) belongs to one warp).  Gradients accumulate
// in fp32 (fp64 for fp64 inputs) whatever the input dtype.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "bevk_internal.h"

namespace bevk {
namespace {

struct Col2imParams {
  int C, H, W, Ho, Wo, kW, T, dg, cpg;
  int sh, sw, ph, pw, dh, dw;
  int mask_is_logit;
  int64_t units;  // M * dg * T
  int64_t xs[4], os[4], ms[4];       // input, offset, mask strides (b, c, h, w)
  int64_t cs[3];                      // column-gradient strides (m, c, t)
  int64_t gxs[4], gos[4], gms[4];    // gradient strides (b, c, h, w)
};

template <typename T>
__device__ __forceinline__ float ldf(const T *p) { return static_cast<float>(*p); }
template <>
__device__ __forceinline__ float ldf<__half>(const __half *p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16 *p) {
  return __bfloat162float(*p);
}

// 4 consecutive elements as floats (the address is aligned to 4 elements).
template <typename T>
__device__ __forceinline__ float4 ld4(const T *p);
template <>
__device__ __forceinline__ float4 ld4<float>(const float *p) {
  return __ldg(reinterpret_cast<const float4 *>(p));
}
template <>
__device__ __forceinline__ float4 ld4<__half>(const __half *p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2 *>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <>
__device__ __forceinline__ float4 ld4<__nv_bfloat16>(const __nv_bfloat16 *p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2 *>(p));
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
}

__device__ __forceinline__ void red_add4(float *p, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a),
               "f"(b), "f"(c), "f"(d)
               : "memory");
}

constexpr int kCol2imWarps = 8;

// TX: input / offset / mask type; TD: column-gradient type; AccT: gradient
// type (float, or double for fp64 problems); VEC: channels per lane step.
template <typename TX, typename TD, typename AccT, int VEC>
__global__ void __launch_bounds__(kCol2imWarps * 32)
dcn_col2im_kernel(const Col2imParams p, const TX *__restrict__ x, const TX *__restrict__ off,
                  const TX *__restrict__ msk, const TD *__restrict__ dcol,
                  AccT *__restrict__ gx, AccT *__restrict__ goff, AccT *__restrict__ gmask) {
  const int lane = threadIdx.x & 31;
  const int64_t unit = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (unit >= p.units) return;
  const int t = static_cast<int>(unit % p.T);
  const int64_t mg = unit / p.T;
  const int gi = static_cast<int>(mg % p.dg);
  const int64_t m = mg / p.dg;
  const int64_t HoWo = static_cast<int64_t>(p.Ho) * p.Wo;
  const int64_t b = m / HoWo;
  const int rem = static_cast<int>(m - b * HoWo);
  const int oh = rem / p.Wo, ow = rem - (rem / p.Wo) * p.Wo;
  const int ki = t / p.kW, kj = t - (t / p.kW) * p.kW;

  const TX *ob = off + b * p.os[0] + oh * p.os[2] + ow * p.os[3];
  const float off_h = ldf(ob + static_cast<int64_t>(gi * 2 * p.T + 2 * t) * p.os[1]);
  const float off_w = ldf(ob + static_cast<int64_t>(gi * 2 * p.T + 2 * t + 1) * p.os[1]);
  const int64_t mask_off = b * p.ms[0] + static_cast<int64_t>(gi * p.T + t) * p.ms[1] +
                           oh * p.ms[2] + ow * p.ms[3];
  float mk = ldf(msk + mask_off);
  if (p.mask_is_logit) mk = 1.f / (1.f + __expf(-mk));
  const float h_im = static_cast<float>(oh * p.sh - p.ph + ki * p.dh) + off_h;
  const float w_im = static_cast<float>(ow * p.sw - p.pw + kj * p.dw) + off_w;
  if (!(h_im > -1.f && w_im > -1.f && h_im < static_cast<float>(p.H) &&
        w_im < static_cast<float>(p.W)))
    return;  // whole warp: the sample contributes nothing
  const int h_low = static_cast<int>(floorf(h_im)), w_low = static_cast<int>(floorf(w_im));
  const float lh = h_im - static_cast<float>(h_low), lw = w_im - static_cast<float>(w_low);
  const float hh = 1.f - lh, hw = 1.f - lw;
  const int hs[4] = {h_low, h_low, h_low + 1, h_low + 1};
  const int ws[4] = {w_low, w_low + 1, w_low, w_low + 1};
  const float wk[4] = {hh * hw, hh * lw, lh * hw, lh * lw};
  const float cy[4] = {-hw, -lw, hw, lw};
  const float cx[4] = {-hh, hh, -lh, lh};
  bool valid[4];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    valid[k] = hs[k] >= 0 && hs[k] <= p.H - 1 && ws[k] >= 0 && ws[k] <= p.W - 1;

  float acc_m = 0.f, acc_h = 0.f, acc_w = 0.f;
  const int c0 = gi * p.cpg;
  const TD *dcol_mt = dcol + m * p.cs[0] + static_cast<int64_t>(t) * p.cs[2];
  for (int cl = lane * VEC; cl < p.cpg; cl += 32 * VEC) {
    const int c = c0 + cl;
    float dc[VEC];
    if constexpr (VEC == 4) {
      const float4 v = ld4(dcol_mt + c);  // channel-contiguous
      dc[0] = v.x; dc[1] = v.y; dc[2] = v.z; dc[3] = v.w;
    } else {
      dc[0] = ldf(dcol_mt + static_cast<int64_t>(c) * p.cs[1]);
    }
    float val[VEC], dvh[VEC], dvw[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) val[v] = dvh[v] = dvw[v] = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (!valid[k]) continue;
      if (x != nullptr) {  // input values: only the coordinate gradients need them
        const int64_t xo = b * p.xs[0] + static_cast<int64_t>(c) * p.xs[1] +
                           hs[k] * p.xs[2] + ws[k] * p.xs[3];
        float xv[VEC];
        if constexpr (VEC == 4) {
          const float4 v = ld4(x + xo);
          xv[0] = v.x; xv[1] = v.y; xv[2] = v.z; xv[3] = v.w;
        } else {
          xv[0] = ldf(x + xo);
        }
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          val[v] = fmaf(wk[k], xv[v], val[v]);
          dvh[v] = fmaf(cy[k], xv[v], dvh[v]);
          dvw[v] = fmaf(cx[k], xv[v], dvw[v]);
        }
      }
      if (gx != nullptr) {
        const float s = mk * wk[k];
        AccT *g = gx + b * p.gxs[0] + static_cast<int64_t>(c) * p.gxs[1] + hs[k] * p.gxs[2] +
                  ws[k] * p.gxs[3];
        if constexpr (VEC == 4) {
          red_add4(reinterpret_cast<float *>(g), s * dc[0], s * dc[1], s * dc[2], s * dc[3]);
        } else {
          atomicAdd(g, static_cast<AccT>(s * dc[0]));
        }
      }
    }
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      acc_m = fmaf(dc[v], val[v], acc_m);
      acc_h = fmaf(dc[v], dvh[v], acc_h);
      acc_w = fmaf(dc[v], dvw[v], acc_w);
    }
  }
  if (goff == nullptr && gmask == nullptr) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc_m += __shfl_xor_sync(0xffffffffu, acc_m, o);
    acc_h += __shfl_xor_sync(0xffffffffu, acc_h, o);
    acc_w += __shfl_xor_sync(0xffffffffu, acc_w, o);
  }
  if (lane == 0) {
    if (goff != nullptr) {
      AccT *gb = goff + b * p.gos[0] + oh * p.gos[2] + ow * p.gos[3];
      gb[static_cast<int64_t>(gi * 2 * p.T + 2 * t) * p.gos[1]] += static_cast<AccT>(mk * acc_h);
      gb[static_cast<int64_t>(gi * 2 * p.T + 2 * t + 1) * p.gos[1]] +=
          static_cast<AccT>(mk * acc_w);
    }
    if (gmask != nullptr) {
      const float gm = p.mask_is_logit ? acc_m * mk * (1.f - mk) : acc_m;
      gmask[b * p.gms[0] + static_cast<int64_t>(gi * p.T + t) * p.gms[1] + oh * p.gms[2] +
            ow * p.gms[3]] += static_cast<AccT>(gm);
    }
  }
}

template <typename TX, typename TD, typename AccT>
int launch_col2im(const Col2imParams &p, const void *x, const void *off, const void *msk,
                  const void *dcol, void *gx, void *goff, void *gmask, bool vec4,
                  cudaStream_t stream) {
  const int64_t blocks = (p.units + kCol2imWarps - 1) / kCol2imWarps;
  if (blocks > 0x7FFFFFFF) return fail(BEVK_ERR_INDEX_OVERFLOW, "dcn col2im: grid too large");
  auto args = [&](auto kern) {
    kern<<<static_cast<unsigned>(blocks), kCol2imWarps * 32, 0, stream>>>(
        p, static_cast<const TX *>(x), static_cast<const TX *>(off),
        static_cast<const TX *>(msk), static_cast<const TD *>(dcol), static_cast<AccT *>(gx),
        static_cast<AccT *>(goff), static_cast<AccT *>(gmask));
  };
  if constexpr (sizeof(AccT) == 4) {
    if (vec4) {
      args(dcn_col2im_kernel<TX, TD, AccT, 4>);
      return check_launch("dcn_col2im_kernel");
    }
  }
  args(dcn_col2im_kernel<TX, TD, AccT, 1>);
  return check_launch("dcn_col2im_kernel");
}

}  // namespace

int launch_dcn_col2im(const bevk_dcn_col2im_args *a, const DcnDims &d, const void *input,
                      const void *offset, const void *mask, const void *dcol, void *grad_input,
                      void *grad_offset, void *grad_mask, cudaStream_t stream) {
  const bevk_dcn_problem &pr = a->problem;
  Col2imParams p;
  p.C = d.Cin; p.H = d.H; p.W = d.W; p.Ho = d.Ho; p.Wo = d.Wo; p.kW = d.kW; p.T = d.T;
  p.dg = d.dg; p.cpg = d.cpdg;
  p.sh = d.sh; p.sw = d.sw; p.ph = d.ph; p.pw = d.pw; p.dh = d.dh; p.dw = d.dw;
  p.mask_is_logit = pr.mask_is_logit;
  p.units = d.M * d.dg * d.T;
  for (int i = 0; i < 4; ++i) {
    p.xs[i] = pr.input_strides[i];
    p.os[i] = pr.offset_strides[i];
    p.ms[i] = pr.mask_strides[i];
    p.gxs[i] = a->grad_input_strides[i];
    p.gos[i] = a->grad_offset_strides[i];
    p.gms[i] = a->grad_mask_strides[i];
  }
  for (int i = 0; i < 3; ++i) p.cs[i] = a->col_strides[i];
  if (p.units == 0) return BEVK_OK;

  const size_t es = dtype_size(pr.dtype), cs = dtype_size(a->col_dtype);
  // 4-channel vectors: channel-contiguous input, column gradient and grad_input,
  // every other stride and the base pointers aligned to 4 elements
  auto al4 = [](const int64_t *s, int n) {
    for (int i = 0; i < n; ++i)
      if (s[i] % 4 != 0) return false;
    return true;
  };
  const int64_t xo[3] = {p.xs[0], p.xs[2], p.xs[3]};
  const int64_t co[2] = {p.cs[0], p.cs[2]};
  const int64_t go[3] = {p.gxs[0], p.gxs[2], p.gxs[3]};
  const bool vec4 = d.cpdg % 4 == 0 && (input == nullptr || (p.xs[1] == 1 && al4(xo, 3) &&
                                                            aligned(input, 4 * es))) &&
                    p.cs[1] == 1 && al4(co, 2) && aligned(dcol, 4 * cs) &&
                    (grad_input == nullptr ||
                     (p.gxs[1] == 1 && al4(go, 3) && aligned(grad_input, 16)));
  cudaStream_t s = stream;
  switch (pr.dtype) {
    case BEVK_DTYPE_F32:
      if (a->col_dtype != BEVK_DTYPE_F32) break;
      return launch_col2im<float, float, float>(p, input, offset, mask, dcol, grad_input,
                                                grad_offset, grad_mask, vec4, s);
    case BEVK_DTYPE_F64:
      if (a->col_dtype != BEVK_DTYPE_F64) break;
      return launch_col2im<double, double, double>(p, input, offset, mask, dcol, grad_input,
                                                   grad_offset, grad_mask, false, s);
    case BEVK_DTYPE_F16:
      if (a->col_dtype == BEVK_DTYPE_F16)
        return launch_col2im<__half, __half, float>(p, input, offset, mask, dcol, grad_input,
                                                    grad_offset, grad_mask, vec4, s);
      if (a->col_dtype == BEVK_DTYPE_F32)
        return launch_col2im<__half, float, float>(p, input, offset, mask, dcol, grad_input,
                                                   grad_offset, grad_mask, vec4, s);
      break;
    case BEVK_DTYPE_BF16:
      if (a->col_dtype == BEVK_DTYPE_BF16)
        return launch_col2im<__nv_bfloat16, __nv_bfloat16, float>(
            p, input, offset, mask, dcol, grad_input, grad_offset, grad_mask, vec4, s);
      if (a->col_dtype == BEVK_DTYPE_F32)
        return launch_col2im<__nv_bfloat16, float, float>(
            p, input, offset, mask, dcol, grad_input, grad_offset, grad_mask, vec4, s);
      break;
    default:
      break;
  }
  return fail(BEVK_ERR_UNSUPPORTED, "dcn col2im: input dtype %d with column dtype %d",
              pr.dtype, a->col_dtype);
}

}  // namespace bevk
