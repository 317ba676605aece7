// dcn_bwd_data.cu -- data-side DCNv2 backward without floating-point atomics.
//
// For channel-contiguous (NHWC) input and column matrices this computes, from
// the column gradient dcol[m, t*C + c] (m = output pixel, t = tap):
//   grad_input[b, c, y, x] = sum over the samples (m, t) whose in-range bilinear
//                            corners include (y, x) of mask * w_corner * dcol
//   grad_offset, grad_mask   as the col2im_coord ops (dcn_bwd.cu's formulas)
//   col[m, t*C + c]        = mask * bilinear(input), the column matrix of the
//                            grad_weight GEMM (the deformable im2col)
// i.e. the reference's NHWC col2im + col2im_coord + im2col sequence of the
// backward (csrc/binding.cpp:63-140; dcn_split_nhwc.py:48-120, :231-291;
// modulated_deform_conv.py:405-499 for the NCHW Function), with the semantics
// of its backward goldens (modulated_deform_conv.py:269-312).
//
// grad_input.  The reference scatters every (sample, corner, channel) product
// into grad_input with floating-point atomics; on this part that runs at the
// L2's atomic rate.  Here the samples' corners are bucketed by destination
// pixel with a counting sort and every grad_input element is summed in
// registers and written once:
//   1. dcn_bwd_count_kernel  -- one thread per sample counts its in-range
//      corners per destination bucket (b, deformable group, y, x) with integer
//      reductions;
//   2. dcn_bwd_scan_kernel   -- one CTA turns the counts into bucket ends
//      (inclusive prefix sums, in place);
//   3. dcn_bwd_fill_kernel   -- one thread per sample takes a slot in each
//      in-range corner's bucket (decrementing the end, so the array holds the
//      bucket starts afterwards) and stores (dcol row offset, weight);
//   4. dcn_bwd_gradx_kernel  -- one group of lanes per (bucket, channel chunk)
//      sums its entries' dcol vectors times the weights in fp32 and writes the
//      grad_input vector: no zeroing pass, no fp32 workspace, no cast pass;
//   5. dcn_bwd_sample_kernel -- one warp per (pixel, 3 taps): the column rows
//      and the coordinate gradients.
// Count and fill derive a sample's corners from the same arithmetic on the
// same offsets, so each bucket receives exactly the entries it counted.  The
// order of the entries inside a bucket follows the order of the fill atomics,
// so the last bits of grad_input may vary between runs (as with the
// reference's atomics); grad_offset, grad_mask and col are deterministic.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <type_traits>

#include "bevk_internal.h"
#include "bevk_ptx.cuh"

namespace bevk {
namespace {

struct BwdDataParams {
  int C, H, W, Ho, Wo, kW, T, dg, cpg;
  int sh, sw, ph, pw, dh, dw;
  int mask_is_logit;
  int nb;              // destination buckets B*dg*H*W
  int64_t M, units;    // output pixels; samples M*dg*T
  int64_t xs[4], os[4], ms[4];
  int xs2, xs3;        // input h / w strides (the input's extent fits 32-bit offsets)
  int64_t dcol_ld, col_ld;
  uint32_t max_row_off;  // largest dcol row offset m*dcol_ld + t*C an entry can hold
  int64_t gxs[4], gos[4], gms[4];
};

template <typename T>
__device__ __forceinline__ float ld1(const T *p) {
  return static_cast<float>(*p);
}
template <>
__device__ __forceinline__ float ld1<__half>(const __half *p) {
  return __half2float(*p);
}
template <>
__device__ __forceinline__ float ld1<__nv_bfloat16>(const __nv_bfloat16 *p) {
  return __bfloat162float(*p);
}

// Elements 2i, 2i+1 of 16 raw bytes of T (i a compile-time index).
__device__ __forceinline__ uint32_t word(const uint4 &u, int i) {
  return i == 0 ? u.x : i == 1 ? u.y : i == 2 ? u.z : u.w;
}
template <typename T>
__device__ __forceinline__ float2 pair_at(const uint4 &u, int i) {
  if constexpr (std::is_same_v<T, float>) {
    return make_float2(__uint_as_float(word(u, 2 * i)), __uint_as_float(word(u, 2 * i + 1)));
  } else if constexpr (std::is_same_v<T, __half>) {
    __half2 h;
    *reinterpret_cast<uint32_t *>(&h) = word(u, i);
    return __half22float2(h);
  } else {
    const uint32_t w = word(u, i);
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  }
}

__device__ __forceinline__ __half2 u32_as_half2(uint32_t w) {
  __half2 h;
  *reinterpret_cast<uint32_t *>(&h) = w;
  return h;
}
__device__ __forceinline__ uint32_t half2_as_u32(__half2 h) {
  return *reinterpret_cast<uint32_t *>(&h);
}

// Packed pairs of fp16 or bf16 in 32-bit words: a weight broadcast to both
// halves, a * b, and a * b + c, each rounded to the type.
template <typename T>
__device__ __forceinline__ uint32_t pack2_weight(float w) {
  if constexpr (std::is_same_v<T, __half>) {
    return half2_as_u32(__float2half2_rn(w));
  } else {
    const __nv_bfloat162 h = __float2bfloat162_rn(w);
    return *reinterpret_cast<const uint32_t *>(&h);
  }
}
template <typename T>
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
  if constexpr (std::is_same_v<T, __half>) {
    return half2_as_u32(__hmul2(u32_as_half2(a), u32_as_half2(b)));
  } else {
    __nv_bfloat162 x, y;
    *reinterpret_cast<uint32_t *>(&x) = a;
    *reinterpret_cast<uint32_t *>(&y) = b;
    const __nv_bfloat162 r = __hmul2(x, y);
    return *reinterpret_cast<const uint32_t *>(&r);
  }
}
template <typename T>
__device__ __forceinline__ uint32_t fma2(uint32_t a, uint32_t b, uint32_t c) {
  if constexpr (std::is_same_v<T, __half>) {
    return half2_as_u32(__hfma2(u32_as_half2(a), u32_as_half2(b), u32_as_half2(c)));
  } else {
    __nv_bfloat162 x, y, z;
    *reinterpret_cast<uint32_t *>(&x) = a;
    *reinterpret_cast<uint32_t *>(&y) = b;
    *reinterpret_cast<uint32_t *>(&z) = c;
    const __nv_bfloat162 r = __hfma2(x, y, z);
    return *reinterpret_cast<const uint32_t *>(&r);
  }
}

// d0 += a.lo * b.lo, d1 += a.hi * b.hi for channel pair i of two 16-byte
// vectors.  fp16 / bf16 operands go straight from their packed words into
// mixed-precision FMAs (the product of two 16-bit floats is exact in fp32, so
// each step rounds once, exactly as an fp32 FMA of the converted operands);
// fp32 operands use fmaf.
template <typename T>
__device__ __forceinline__ void fma_pair(float &d0, float &d1, const uint4 &a, const uint4 &b,
                                         int i) {
  if constexpr (std::is_same_v<T, float>) {
    d0 = fmaf(__uint_as_float(word(a, 2 * i)), __uint_as_float(word(b, 2 * i)), d0);
    d1 = fmaf(__uint_as_float(word(a, 2 * i + 1)), __uint_as_float(word(b, 2 * i + 1)), d1);
  } else if constexpr (std::is_same_v<T, __half>) {
    asm("{\n\t.reg .b16 a0, a1, b0, b1;\n\tmov.b32 {a0, a1}, %2;\n\tmov.b32 {b0, b1}, %3;\n\t"
        "fma.rn.f32.f16 %0, a0, b0, %0;\n\tfma.rn.f32.f16 %1, a1, b1, %1;\n\t}"
        : "+f"(d0), "+f"(d1)
        : "r"(word(a, i)), "r"(word(b, i)));
  } else {
    asm("{\n\t.reg .b16 a0, a1, b0, b1;\n\tmov.b32 {a0, a1}, %2;\n\tmov.b32 {b0, b1}, %3;\n\t"
        "fma.rn.f32.bf16 %0, a0, b0, %0;\n\tfma.rn.f32.bf16 %1, a1, b1, %1;\n\t}"
        : "+f"(d0), "+f"(d1)
        : "r"(word(a, i)), "r"(word(b, i)));
  }
}

// V floats rounded to TO and stored (p aligned to 16 bytes; V*sizeof(TO) a
// multiple of 16).
template <typename TO, int V>
__device__ __forceinline__ void st_vec(TO *p, const float (&f)[V]) {
  if constexpr (sizeof(TO) == 4) {
#pragma unroll
    for (int i = 0; i < V; i += 4)
      *reinterpret_cast<float4 *>(p + i) = make_float4(f[i], f[i + 1], f[i + 2], f[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < V; i += 8) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t lo, hi;
        if constexpr (std::is_same_v<TO, __half>) {
          lo = __half_as_ushort(__float2half_rn(f[i + 2 * j]));
          hi = __half_as_ushort(__float2half_rn(f[i + 2 * j + 1]));
        } else {
          lo = __bfloat16_as_ushort(__float2bfloat16_rn(f[i + 2 * j]));
          hi = __bfloat16_as_ushort(__float2bfloat16_rn(f[i + 2 * j + 1]));
        }
        w[j] = lo | (hi << 16);
      }
      *reinterpret_cast<uint4 *>(p + i) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <typename TO>
__device__ __forceinline__ TO cast_out(float v) {
  if constexpr (std::is_same_v<TO, __half>) return __float2half_rn(v);
  else if constexpr (std::is_same_v<TO, __nv_bfloat16>) return __float2bfloat16_rn(v);
  else return v;
}

// Position of sample `unit` = (m*dg + gi)*T + t in the input image (32-bit
// indices: the entry point keeps 4 * samples below 2^31).
struct Sample {
  int m, b, gi, t, oh, ow;
  float h_im, w_im;
};

template <typename T>
__device__ __forceinline__ Sample sample_at(const BwdDataParams &p, const T *off, int unit) {
  Sample s;
  const int mg = unit / p.T;
  s.t = unit - mg * p.T;
  s.m = mg / p.dg;
  s.gi = mg - s.m * p.dg;
  const int HoWo = p.Ho * p.Wo;
  s.b = s.m / HoWo;
  const int rem = s.m - s.b * HoWo;
  s.oh = rem / p.Wo;
  s.ow = rem - s.oh * p.Wo;
  const int ki = s.t / p.kW, kj = s.t - ki * p.kW;
  const T *ob = off + s.b * p.os[0] + s.oh * p.os[2] + s.ow * p.os[3];
  const float off_h = ld1(ob + static_cast<int64_t>(s.gi * 2 * p.T + 2 * s.t) * p.os[1]);
  const float off_w = ld1(ob + static_cast<int64_t>(s.gi * 2 * p.T + 2 * s.t + 1) * p.os[1]);
  s.h_im = static_cast<float>(s.oh * p.sh - p.ph + ki * p.dh) + off_h;
  s.w_im = static_cast<float>(s.ow * p.sw - p.pw + kj * p.dw) + off_w;
  return s;
}

__device__ __forceinline__ bool in_gate(const BwdDataParams &p, const Sample &s) {
  return s.h_im > -1.f && s.w_im > -1.f && s.h_im < static_cast<float>(p.H) &&
         s.w_im < static_cast<float>(p.W);
}

// Bucket of corner k (0: (h_low, w_low), 1: (h_low, w_low+1), 2: (h_low+1,
// w_low), 3: (h_low+1, w_low+1)), or -1 when it lies outside the image.
__device__ __forceinline__ int corner_bucket(const BwdDataParams &p, const Sample &s, int h_low,
                                             int w_low, int k) {
  const int y = h_low + (k >> 1), x = w_low + (k & 1);
  if (y < 0 || y > p.H - 1 || x < 0 || x > p.W - 1) return -1;
  return ((s.b * p.dg + s.gi) * p.H + y) * p.W + x;
}

template <typename T>
__global__ void __launch_bounds__(256)
dcn_bwd_count_kernel(const BwdDataParams p, const T *__restrict__ off, int *__restrict__ cnt) {
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  const int units = static_cast<int>(p.units);
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < units; u += gridDim.x * blockDim.x) {
    const Sample s = sample_at(p, off, u);
    if (!in_gate(p, s)) continue;
    const int h_low = static_cast<int>(floorf(s.h_im)), w_low = static_cast<int>(floorf(s.w_im));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int bk = corner_bucket(p, s, h_low, w_low, k);
      if (bk >= 0) atomicAdd(cnt + bk, 1);
    }
  }
}

constexpr int kScanThreads = 1024, kScanItems = 8;

// In-place inclusive prefix sums of cnt[0, nb); cnt[nb] = the total.  Each
// thread takes 8 consecutive counts (two 16-byte vectors; cnt is 16-byte
// aligned and tiles start at multiples of 8192).
__global__ void __launch_bounds__(kScanThreads)
dcn_bwd_scan_kernel(int *__restrict__ cnt, int nb) {
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  __shared__ int warp_sum[kScanThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int carry = 0;
  for (int base = 0; base < nb; base += kScanThreads * kScanItems) {
    const int i0 = base + threadIdx.x * kScanItems;
    int v[kScanItems];
    if (i0 + kScanItems <= nb) {
      const int4 a = *reinterpret_cast<const int4 *>(cnt + i0);
      const int4 b = *reinterpret_cast<const int4 *>(cnt + i0 + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int j = 0; j < kScanItems; ++j) v[j] = i0 + j < nb ? cnt[i0 + j] : 0;
    }
#pragma unroll
    for (int j = 1; j < kScanItems; ++j) v[j] += v[j - 1];
    const int run = v[kScanItems - 1];
    int incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sum[lane] = w;
    }
    __syncthreads();
    const int before = carry + (warp > 0 ? warp_sum[warp - 1] : 0) + (incl - run);
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) v[j] += before;
    if (i0 + kScanItems <= nb) {
      *reinterpret_cast<int4 *>(cnt + i0) = make_int4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<int4 *>(cnt + i0 + 4) = make_int4(v[4], v[5], v[6], v[7]);
    } else {
#pragma unroll
      for (int j = 0; j < kScanItems; ++j)
        if (i0 + j < nb) cnt[i0 + j] = v[j];
    }
    carry += warp_sum[kScanThreads / 32 - 1];
    __syncthreads();  // warp_sum is rewritten by the next tile
  }
  if (threadIdx.x == 0) cnt[nb] = carry;
}

// Bucket fill: one thread per sample takes a slot in each in-range corner's
// bucket (decrementing the bucket's end, so the array holds the bucket starts
// afterwards) and stores (dcol row offset, mask * corner weight).  A kernel of
// its own: atomics that return a value stall the warps that issue them, so
// they are kept away from the channel loops.
template <typename T>
__global__ void __launch_bounds__(256)
dcn_bwd_fill_kernel(const BwdDataParams p, const T *__restrict__ off, const T *__restrict__ msk,
                    int *__restrict__ ends, uint2 *__restrict__ entries) {
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  const int units = static_cast<int>(p.units);
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < units; u += gridDim.x * blockDim.x) {
    const Sample s = sample_at(p, off, u);
    if (!in_gate(p, s)) continue;
    float mk = ld1(msk + s.b * p.ms[0] + static_cast<int64_t>(s.gi * p.T + s.t) * p.ms[1] +
                   s.oh * p.ms[2] + s.ow * p.ms[3]);
    if (p.mask_is_logit) mk = 1.f / (1.f + __expf(-mk));
    const int h_low = static_cast<int>(floorf(s.h_im)), w_low = static_cast<int>(floorf(s.w_im));
    const float lh = s.h_im - static_cast<float>(h_low), lw = s.w_im - static_cast<float>(w_low);
    const uint32_t row =
        static_cast<uint32_t>(static_cast<int64_t>(s.m) * p.dcol_ld + static_cast<int64_t>(s.t) * p.C);
    int slot[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int bk = corner_bucket(p, s, h_low, w_low, k);
      slot[k] = bk >= 0 ? atomicAdd(ends + bk, -1) - 1 : -1;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (slot[k] < 0) continue;
      const float wk = (k >> 1 ? lh : 1.f - lh) * (k & 1 ? lw : 1.f - lw);
      entries[slot[k]] = make_uint2(row, __float_as_uint(mk * wk));
    }
  }
}

constexpr int kSampleWarps = 1;  // one-warp CTAs: measured fastest (more CTAs in flight)
constexpr int kOutside = -(1 << 20);  // h_low of a sample outside the gate: no corner in range

// One warp per (output pixel, deformable group, group of `tpw` taps).  Lane j
// first takes tap t0 + j (position, mask, corner weights); the warp then walks
// the taps, each lane covering 16-byte channel vectors of the four corner
// lines and the column-gradient row: the column row, and the tap's per-corner
// channel sums.  Invalid corners load zeros and take part in the arithmetic
// (adding zero products leaves every sum as it is), so the channel loop has
// no branches.
//
// The coordinate gradients come from the four per-corner dot products
// D_k = sum_c dcol_c * x_k,c (zero for corners outside the image):
//   grad_mask   = sum_k w_k D_k                 (bilinear weights w_k)
//   grad_off_h  = mask * (hw (D2 - D0) + lw (D3 - D1))
//   grad_off_w  = mask * (hh (D1 - D0) + lh (D3 - D2))
// -- the derivatives of the bilinear weights, summed over the channels once
// per corner instead of once per derivative.
template <typename T, typename TG>
__global__ void __launch_bounds__(kSampleWarps * 32)
dcn_bwd_sample_kernel(const BwdDataParams p, const T *__restrict__ x, const T *__restrict__ off,
                      const T *__restrict__ msk, const T *__restrict__ dcol,
                      TG *__restrict__ goff, TG *__restrict__ gmask, T *__restrict__ col, int tpw,
                      int ngroups) {
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  constexpr int V = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int unit = blockIdx.x * kSampleWarps + (threadIdx.x >> 5);
  if (unit >= static_cast<int>(p.M) * p.dg * ngroups) return;
  const int mg = unit / ngroups;
  const int t0 = (unit - mg * ngroups) * tpw;
  const int nt = min(tpw, p.T - t0);
  const int m = mg / p.dg;
  const int gi = mg - m * p.dg;
  const int HoWo = p.Ho * p.Wo;
  const int b = m / HoWo;
  const int rem = m - b * HoWo;
  const int oh = rem / p.Wo;
  const int ow = rem - oh * p.Wo;

  // ---- lane j: tap t0 + j
  int hl = kOutside, wl = 0;
  float lh = 0.f, lw = 0.f, mk = 0.f;
  if (lane < nt) {
    const int t = t0 + lane;
    const int ki = t / p.kW, kj = t - ki * p.kW;
    const T *ob = off + b * p.os[0] + oh * p.os[2] + ow * p.os[3];
    const float off_h = ld1(ob + static_cast<int64_t>(gi * 2 * p.T + 2 * t) * p.os[1]);
    const float off_w = ld1(ob + static_cast<int64_t>(gi * 2 * p.T + 2 * t + 1) * p.os[1]);
    mk = ld1(msk + b * p.ms[0] + static_cast<int64_t>(gi * p.T + t) * p.ms[1] + oh * p.ms[2] +
             ow * p.ms[3]);
    if (p.mask_is_logit) mk = 1.f / (1.f + __expf(-mk));
    const float h_im = static_cast<float>(oh * p.sh - p.ph + ki * p.dh) + off_h;
    const float w_im = static_cast<float>(ow * p.sw - p.pw + kj * p.dw) + off_w;
    if (h_im > -1.f && w_im > -1.f && h_im < static_cast<float>(p.H) &&
        w_im < static_cast<float>(p.W)) {
      hl = static_cast<int>(floorf(h_im));
      wl = static_cast<int>(floorf(w_im));
      lh = h_im - static_cast<float>(hl);
      lw = w_im - static_cast<float>(wl);
    }
  }

  const bool coord = goff != nullptr || gmask != nullptr;
  const T *xb = x + b * p.xs[0] + gi * p.cpg;
  const int64_t row_d = static_cast<int64_t>(m) * p.dcol_ld + gi * p.cpg;
  const int64_t row_c = static_cast<int64_t>(m) * p.col_ld + gi * p.cpg;
  float myd[4] = {0.f, 0.f, 0.f, 0.f};  // lane j: the four corner sums of tap t0 + j
  for (int j = 0; j < nt; ++j) {
    const int h0 = __shfl_sync(0xffffffffu, hl, j);
    const int w0 = __shfl_sync(0xffffffffu, wl, j);
    const float fh = __shfl_sync(0xffffffffu, lh, j);
    const float fw = __shfl_sync(0xffffffffu, lw, j);
    const float m0 = __shfl_sync(0xffffffffu, mk, j);
    const float gh = 1.f - fh, gw = 1.f - fw;
    const float wk[4] = {gh * gw, gh * fw, fh * gw, fh * fw};
    int xo[4];
    bool valid[4];
    float wm[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int y = h0 + (k >> 1), xx = w0 + (k & 1);
      valid[k] = y >= 0 && y <= p.H - 1 && xx >= 0 && xx <= p.W - 1;
      xo[k] = valid[k] ? y * p.xs2 + xx * p.xs3 : 0;
      wm[k] = wk[k] * m0;  // the forward's corner weight, mask folded in
    }
    uint32_t w2[4];  // 16-bit paths: the weights as packed pairs of the input type
#pragma unroll
    for (int k = 0; k < 4; ++k) w2[k] = pack2_weight<T>(wm[k]);
    const bool load_d = coord && h0 != kOutside;
    const T *dc_row = dcol + row_d + static_cast<int64_t>(t0 + j) * p.C;
    T *col_row = col != nullptr ? col + row_c + static_cast<int64_t>(t0 + j) * p.C : nullptr;
    float2 D[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) D[k] = make_float2(0.f, 0.f);
#pragma unroll 2
    for (int c = lane * V; c < p.cpg; c += 32 * V) {
      uint4 xr[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        xr[k] = valid[k] ? __ldg(reinterpret_cast<const uint4 *>(xb + (xo[k] + c)))
                         : make_uint4(0, 0, 0, 0);
      const uint4 dr = load_d ? __ldg(reinterpret_cast<const uint4 *>(dc_row + c))
                              : make_uint4(0, 0, 0, 0);
      if constexpr (sizeof(T) == 2) {
        // fp16 / bf16: the column values as the fused forward kernel builds
        // its A tiles -- corner weights in the input type (mask folded in), a
        // packed multiply and three packed FMAs per channel pair, each step
        // rounded to the input type -- so no operand is converted to fp32 in
        // this loop (the corner sums take the packed words directly)
        uint32_t cw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t r = mul2<T>(w2[0], word(xr[0], i));
#pragma unroll
          for (int k = 1; k < 4; ++k) r = fma2<T>(w2[k], word(xr[k], i), r);
          cw[i] = r;
#pragma unroll
          for (int k = 0; k < 4; ++k) fma_pair<T>(D[k].x, D[k].y, dr, xr[k], i);
        }
        if (col_row != nullptr)
          *reinterpret_cast<uint4 *>(col_row + c) = make_uint4(cw[0], cw[1], cw[2], cw[3]);
      } else {
        float cv[V];
#pragma unroll
        for (int i = 0; i < V / 2; ++i) {
          // column value: corners in order, products with the mask-folded
          // weights in fp32, rounded once (the im2col kernel's arithmetic)
          float a0 = 0.f, a1 = 0.f;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 x2 = pair_at<T>(xr[k], i);
            a0 = fmaf(wm[k], x2.x, a0);
            a1 = fmaf(wm[k], x2.y, a1);
            fma_pair<T>(D[k].x, D[k].y, dr, xr[k], i);
          }
          cv[2 * i] = a0;
          cv[2 * i + 1] = a1;
        }
        if (col_row != nullptr) st_vec<T, V>(col_row + c, cv);
      }
    }
    if (coord) {
      float d[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) d[k] = D[k].x + D[k].y;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int k = 0; k < 4; ++k) d[k] += __shfl_xor_sync(0xffffffffu, d[k], o);
      if (lane == j) {
#pragma unroll
        for (int k = 0; k < 4; ++k) myd[k] = d[k];
      }
    }
  }
  if (coord && lane < nt) {
    const int t = t0 + lane;
    const float hh = 1.f - lh, hw = 1.f - lw;
    if (goff != nullptr) {
      const float gh = mk * (hw * (myd[2] - myd[0]) + lw * (myd[3] - myd[1]));
      const float gw = mk * (hh * (myd[1] - myd[0]) + lh * (myd[3] - myd[2]));
      TG *gb = goff + b * p.gos[0] + oh * p.gos[2] + ow * p.gos[3];
      gb[static_cast<int64_t>(gi * 2 * p.T + 2 * t) * p.gos[1]] = cast_out<TG>(gh);
      gb[static_cast<int64_t>(gi * 2 * p.T + 2 * t + 1) * p.gos[1]] = cast_out<TG>(gw);
    }
    if (gmask != nullptr) {
      const float am = hh * hw * myd[0] + hh * lw * myd[1] + lh * hw * myd[2] + lh * lw * myd[3];
      const float gm = p.mask_is_logit ? am * mk * (1.f - mk) : am;
      gmask[b * p.gms[0] + static_cast<int64_t>(gi * p.T + t) * p.gms[1] + oh * p.gms[2] +
            ow * p.gms[3]] = cast_out<TG>(gm);
    }
  }
}

constexpr int kGatherThreads = 128;

// One group of 2^lpg_log2 lanes per (bucket, chunk of VPL * 2^lpg_log2 * V
// channels): each lane sums VPL channel vectors of its bucket's entries.
template <typename T, typename TG, int VPL>
__global__ void __launch_bounds__(kGatherThreads, 8)
dcn_bwd_gradx_kernel(const BwdDataParams p, const T *__restrict__ dcol,
                     const int *__restrict__ starts, const uint2 *__restrict__ entries,
                     TG *__restrict__ gx, int lpg_log2, int nchunks) {
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  constexpr int V = 16 / sizeof(T);
  // entries per batch: loads in flight per lane = kUnroll * VPL, with the
  // register budget of eight CTAs per SM
  constexpr int kGatherUnroll = VPL == 2 ? 2 : 4;
  const int lane = threadIdx.x & 31;
  const int lpg = 1 << lpg_log2;
  const int li = lane & (lpg - 1);
  const unsigned gmask = lpg == 32 ? 0xffffffffu
                                   : ((1u << lpg) - 1u) << (lane & ~(lpg - 1));
  const int64_t group = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> lpg_log2;
  if (group >= static_cast<int64_t>(p.nb) * nchunks) return;  // whole groups leave together
  const int bucket = static_cast<int>(group / nchunks);
  const int chunk = static_cast<int>(group - static_cast<int64_t>(bucket) * nchunks);
  const int xw = bucket % p.W;
  int r = bucket / p.W;
  const int yh = r % p.H;
  r /= p.H;
  const int gi = r % p.dg;
  const int b = r / p.dg;
  const int cl = chunk * VPL * lpg * V + li * V;  // first channel (within the group) of the lane
  bool on[VPL];
#pragma unroll
  for (int h = 0; h < VPL; ++h) on[h] = cl + h * lpg * V < p.cpg;
  const T *src = dcol + (gi * p.cpg + cl);
  const int beg = starts[bucket], end = starts[bucket + 1];

  float acc[VPL][V];
#pragma unroll
  for (int h = 0; h < VPL; ++h)
#pragma unroll
    for (int v = 0; v < V; ++v) acc[h][v] = 0.f;
  for (int j0 = beg; j0 < end; j0 += lpg) {
    const uint2 e = j0 + li < end ? entries[j0 + li] : make_uint2(0u, 0u);
    const int n = min(lpg, end - j0);
    for (int jj = 0; jj < n; jj += kGatherUnroll) {
      uint32_t o[kGatherUnroll];
      float w[kGatherUnroll];
      uint4 raw[kGatherUnroll][VPL];
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        // (lanes past n read a neighbour's entry; it is not used)
        o[u] = min(__shfl_sync(gmask, e.x, (jj + u) & (lpg - 1), lpg), p.max_row_off);
        w[u] = __uint_as_float(__shfl_sync(gmask, e.y, (jj + u) & (lpg - 1), lpg));
      }
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u)
#pragma unroll
        for (int h = 0; h < VPL; ++h)
          raw[u][h] = on[h] && jj + u < n
                          ? __ldg(reinterpret_cast<const uint4 *>(src + o[u] + h * lpg * V))
                          : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        if (jj + u >= n) continue;
#pragma unroll
        for (int h = 0; h < VPL; ++h)
#pragma unroll
          for (int i = 0; i < V / 2; ++i) {
            const float2 f = pair_at<T>(raw[u][h], i);
            acc[h][2 * i] = fmaf(w[u], f.x, acc[h][2 * i]);
            acc[h][2 * i + 1] = fmaf(w[u], f.y, acc[h][2 * i + 1]);
          }
      }
    }
  }
  TG *dst = gx + b * p.gxs[0] + static_cast<int64_t>(gi * p.cpg + cl) + yh * p.gxs[2] +
            xw * p.gxs[3];
#pragma unroll
  for (int h = 0; h < VPL; ++h)
    if (on[h]) st_vec<TG, V>(dst + h * lpg * V, acc[h]);
}

size_t round16(size_t n) { return (n + 15) & ~static_cast<size_t>(15); }

template <typename T, typename TG>
int launch_typed(const BwdDataParams &p, const void *input, const void *offset,
                 const void *mask, const void *dcol, void *grad_input, void *grad_offset,
                 void *grad_mask, void *col, void *workspace, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(T);
  const T *off = static_cast<const T *>(offset);
  const int64_t max_blocks = static_cast<int64_t>(device_info(current_device()).sm_count) * 8;
  int *cnt = nullptr;
  uint2 *entries = nullptr;
  if (grad_input != nullptr) {
    cnt = static_cast<int *>(workspace);
    entries = reinterpret_cast<uint2 *>(static_cast<char *>(workspace) +
                                        round16((static_cast<size_t>(p.nb) + 1) * sizeof(int)));
    if (cudaMemsetAsync(cnt, 0, (static_cast<size_t>(p.nb) + 1) * sizeof(int), stream) !=
        cudaSuccess)
      return check_launch("dcn backward data: bucket count reset");
    const int64_t blocks = std::min<int64_t>((p.units + 255) / 256, max_blocks);
    int st = launched(launch_dependent(dcn_bwd_count_kernel<T>, dim3(static_cast<unsigned>(blocks)),
                                       dim3(256), 0, stream, p, off, cnt),
                      "dcn_bwd_count_kernel");
    if (st != BEVK_OK) return st;
    st = launched(launch_dependent(dcn_bwd_scan_kernel, dim3(1), dim3(kScanThreads), 0, stream,
                                   cnt, p.nb),
                  "dcn_bwd_scan_kernel");
    if (st != BEVK_OK) return st;
  }
  if (grad_input != nullptr) {
    const int64_t fblocks = std::min<int64_t>((p.units + 255) / 256, max_blocks);
    int st = launched(launch_dependent(dcn_bwd_fill_kernel<T>, dim3(static_cast<unsigned>(fblocks)),
                                       dim3(256), 0, stream, p, off,
                                       static_cast<const T *>(mask), cnt, entries),
                      "dcn_bwd_fill_kernel");
    if (st != BEVK_OK) return st;
    // The gather runs before the sample kernel, while the column gradient
    // (written just before this call) is still in L2.  Lanes per bucket:
    // enough for the group's channel vectors (a power of two, at most 32);
    // two vectors per lane once a warp's 32 lanes would otherwise take a
    // bucket in two or more chunks.
    const int nvec = (p.cpg + V - 1) / V;
    int lpg_log2 = 0;
    while ((1 << lpg_log2) < nvec && lpg_log2 < 5) ++lpg_log2;
    const int lpg = 1 << lpg_log2;
    const int vpl = nvec >= 2 * lpg ? 2 : 1;
    const int nchunks = (nvec + vpl * lpg - 1) / (vpl * lpg);
    const int64_t threads = static_cast<int64_t>(p.nb) * nchunks * lpg;
    const int64_t gblocks = (threads + kGatherThreads - 1) / kGatherThreads;
    if (gblocks > 0x7FFFFFFF)
      return fail(BEVK_ERR_INDEX_OVERFLOW, "dcn backward data: grid too large");
    auto kern = vpl == 2 ? dcn_bwd_gradx_kernel<T, TG, 2> : dcn_bwd_gradx_kernel<T, TG, 1>;
    st = launched(launch_dependent(kern, dim3(static_cast<unsigned>(gblocks)),
                                   dim3(kGatherThreads), 0, stream, p,
                                   static_cast<const T *>(dcol), static_cast<const int *>(cnt),
                                   static_cast<const uint2 *>(entries),
                                   static_cast<TG *>(grad_input), lpg_log2, nchunks),
                  "dcn_bwd_gradx_kernel");
    if (st != BEVK_OK) return st;
  }
  if (grad_offset == nullptr && grad_mask == nullptr && col == nullptr) return BEVK_OK;
  // taps per warp: threes for the usual 3-wide kernels, else all taps (at
  // most 32)
  const int tpw = p.T % 3 == 0 ? 3 : std::min(p.T, 32);
  const int ngroups = (p.T + tpw - 1) / tpw;
  const int64_t warps = p.M * p.dg * ngroups;
  if (warps > 0x7FFFFFFF) return fail(BEVK_ERR_INDEX_OVERFLOW, "dcn backward data: grid too large");
  const int64_t blocks = (warps + kSampleWarps - 1) / kSampleWarps;
  return launched(launch_dependent(dcn_bwd_sample_kernel<T, TG>, dim3(static_cast<unsigned>(blocks)),
                                   dim3(kSampleWarps * 32), 0, stream, p,
                                   static_cast<const T *>(input), off,
                                   static_cast<const T *>(mask), static_cast<const T *>(dcol),
                                   static_cast<TG *>(grad_offset), static_cast<TG *>(grad_mask),
                                   static_cast<T *>(col), tpw, ngroups),
                  "dcn_bwd_sample_kernel");
}

}  // namespace

size_t dcn_backward_data_workspace_bytes(const DcnDims &d) {
  const size_t nb = static_cast<size_t>(d.B) * d.dg * d.H * d.W;
  const size_t units = static_cast<size_t>(d.M) * d.dg * d.T;
  return round16((nb + 1) * sizeof(int)) + 4 * units * sizeof(uint2);
}

int launch_dcn_backward_data(const bevk_dcn_backward_data_args *a, const DcnDims &d,
                             const void *input, const void *offset, const void *mask,
                             const void *dcol, void *grad_input, void *grad_offset,
                             void *grad_mask, void *col, void *workspace,
                             size_t workspace_bytes, cudaStream_t stream) {
  const bevk_dcn_problem &pr = a->problem;
  const int dt = pr.dtype;
  if (dt != BEVK_DTYPE_F32 && dt != BEVK_DTYPE_F16 && dt != BEVK_DTYPE_BF16)
    return fail(BEVK_ERR_UNSUPPORTED, "dcn backward data: dtype %d not supported", dt);
  if (a->grad_dtype != dt && a->grad_dtype != BEVK_DTYPE_F32)
    return fail(BEVK_ERR_UNSUPPORTED,
                "dcn backward data: gradient dtype must be the problem dtype or f32");
  const int64_t V = 16 / static_cast<int64_t>(dtype_size(dt));
  auto mult = [V](int64_t v) { return v % V == 0; };
  const bool need_x = grad_offset != nullptr || grad_mask != nullptr || col != nullptr;
  const bool need_dcol = grad_offset != nullptr || grad_mask != nullptr || grad_input != nullptr;
  // channel-contiguous, 16-byte-vector layouts only
  bool ok = mult(d.cpdg) && mult(d.Cin);
  if (need_x)
    ok = ok && pr.input_strides[1] == 1 && mult(pr.input_strides[0]) &&
         mult(pr.input_strides[2]) && mult(pr.input_strides[3]) && aligned(input, 16);
  if (need_dcol) ok = ok && mult(a->dcol_ld) && aligned(dcol, 16);
  if (col != nullptr) ok = ok && mult(a->col_ld) && aligned(col, 16);
  if (grad_input != nullptr) {
    const int64_t *g = a->grad_input_strides;
    ok = ok && g[1] == 1 && mult(g[0]) && mult(g[2]) && mult(g[3]) && aligned(grad_input, 16);
  }
  if (!ok)
    return fail(BEVK_ERR_UNSUPPORTED,
                "dcn backward data: needs channel-contiguous input / gradient, channels and "
                "row strides in whole 16-byte vectors, 16-byte-aligned pointers");
  // 32-bit indices: bucket entries hold 32-bit dcol row offsets, a pixel's
  // channel vector inside one image is a 32-bit offset, and the sort counts
  // (4 corners per sample) fit an int
  const int64_t nb = static_cast<int64_t>(d.B) * d.dg * d.H * d.W;
  const int64_t units = d.M * d.dg * d.T;
  if (need_dcol && static_cast<uint64_t>(d.M) * static_cast<uint64_t>(a->dcol_ld) > 0xFFFFFFFFull)
    return fail(BEVK_ERR_INDEX_OVERFLOW,
                "dcn backward data: column gradient of %lld rows x %lld elements exceeds "
                "32-bit offsets", static_cast<long long>(d.M), static_cast<long long>(a->dcol_ld));
  if (need_x && (static_cast<int64_t>(d.H) - 1) * pr.input_strides[2] +
                        (static_cast<int64_t>(d.W) - 1) * pr.input_strides[3] + d.Cin >
                    0x7FFFFFFF)
    return fail(BEVK_ERR_INDEX_OVERFLOW, "dcn backward data: one input image exceeds 32-bit offsets");
  if (nb + 1 > 0x7FFFFFFF || 4 * units > 0x7FFFFFFF)
    return fail(BEVK_ERR_INDEX_OVERFLOW,
                "dcn backward data: %lld samples (4 corners each) exceed 32-bit counts",
                static_cast<long long>(units));
  if (grad_input != nullptr &&
      (workspace == nullptr || workspace_bytes < dcn_backward_data_workspace_bytes(d)))
    return fail(BEVK_ERR_WORKSPACE, "dcn backward data: workspace of %zu bytes, %zu needed",
                workspace_bytes, dcn_backward_data_workspace_bytes(d));
  if (grad_input != nullptr && !aligned(workspace, 16))
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn backward data: workspace not 16-byte aligned");

  BwdDataParams p;
  p.C = d.Cin; p.H = d.H; p.W = d.W; p.Ho = d.Ho; p.Wo = d.Wo; p.kW = d.kW; p.T = d.T;
  p.dg = d.dg; p.cpg = d.cpdg;
  p.sh = d.sh; p.sw = d.sw; p.ph = d.ph; p.pw = d.pw; p.dh = d.dh; p.dw = d.dw;
  p.mask_is_logit = pr.mask_is_logit;
  p.nb = static_cast<int>(nb);
  p.M = d.M;
  p.units = units;
  p.xs2 = need_x ? static_cast<int>(pr.input_strides[2]) : 0;
  p.xs3 = need_x ? static_cast<int>(pr.input_strides[3]) : 0;
  for (int i = 0; i < 4; ++i) {
    p.xs[i] = pr.input_strides[i];
    p.os[i] = pr.offset_strides[i];
    p.ms[i] = pr.mask_strides[i];
    p.gxs[i] = a->grad_input_strides[i];
    p.gos[i] = a->grad_offset_strides[i];
    p.gms[i] = a->grad_mask_strides[i];
  }
  p.dcol_ld = a->dcol_ld;
  p.col_ld = a->col_ld;
  p.max_row_off = static_cast<uint32_t>((d.M - 1) * a->dcol_ld + (d.T - 1) * d.Cin);
  if (units == 0) return BEVK_OK;
  const bool f32g = a->grad_dtype == BEVK_DTYPE_F32;
  switch (dt) {
    case BEVK_DTYPE_F32:
      return launch_typed<float, float>(p, input, offset, mask, dcol, grad_input, grad_offset,
                                        grad_mask, col, workspace, stream);
    case BEVK_DTYPE_F16:
      return f32g ? launch_typed<__half, float>(p, input, offset, mask, dcol, grad_input,
                                                grad_offset, grad_mask, col, workspace, stream)
                  : launch_typed<__half, __half>(p, input, offset, mask, dcol, grad_input,
                                                 grad_offset, grad_mask, col, workspace, stream);
    default:
      return f32g ? launch_typed<__nv_bfloat16, float>(p, input, offset, mask, dcol, grad_input,
                                                       grad_offset, grad_mask, col, workspace,
                                                       stream)
                  : launch_typed<__nv_bfloat16, __nv_bfloat16>(p, input, offset, mask, dcol,
                                                               grad_input, grad_offset, grad_mask,
                                                               col, workspace, stream);
  }
}

}  // namespace bevk
