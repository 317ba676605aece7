// msda_bwd.cu -- multi-scale deformable attention backward for sm_100a.
//
// Semantics follow csrc_musa/msda/ms_deform_attn_kernels.cuh:425-494
// (msda_col2im_bilinear_grad) and :638-788 (the C = 32 warp-reduce kernel),
// host side binding_musa.mu:414-543.  For every sample (b, q, m, l, p) inside
// the gate -1 < h < H_l, -1 < w < W_l (h = loc_y*H_l - 0.5, w = loc_x*W_l -
// 0.5), with corner weights w1..w4 = hh*hw, hh*lw, lh*hw, lh*lw and v1..v4 the
// in-range corner values (0 outside), and g = grad_out[b, q, m*C : m*C + C]:
//   grad_value[corner k, m, :] += wk * attn * g
//   grad_attn  = sum_c g * (w1 v1 + w2 v2 + w3 v3 + w4 v4)
//   grad_loc_x = W_l * attn * sum_c g * (-hh v1 + hh v2 - lh v3 + lh v4)
//   grad_loc_y = H_l * attn * sum_c g * (-hw v1 - lw v2 + hw v3 + lw v4)
// Samples outside the gate get zero grad_loc / grad_attn (written).
//
// Design (C == 32): backward has no per-unit reduction, so the sample index
// space (units x L*P, memory order of sampling_loc) is cut into passes of 32
// consecutive samples whatever L*P is.  Lane s of a warp computes sample s's
// geometry into shared memory; then for each sample lanes 8g..8g+7 own corner
// g as 4-channel vectors: one predicated vector load of the corner line, a
// 4-wide dot with grad_out, and one vector red.global.add.v4.f32 of
// wk*attn*g into grad_value (a quarter of the reference's per-channel
// atomics).  The per-corner dots of a batch of samples are folded by a
// reduce-scatter inside each corner group, the corners' shares summed with
// two shuffle rounds, and the grad_loc / grad_attn of a batch written by 8
// (or 4) lanes.  Loads of a batch of samples are issued before any of them is
// consumed.  grad_value of fp16 / bf16 problems accumulates in an fp32
// workspace and is narrowed at the end, as the reference does
// (binding_musa.mu:450-507).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

#include "bevk_internal.h"
#include "bevk_ptx.cuh"

namespace bevk {
namespace {

constexpr int kMaxLevels = 16;
constexpr int kBwdWarps = 8;

template <typename T>
__device__ __forceinline__ float to_f(T v) { return static_cast<float>(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v) { return static_cast<T>(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// 4 consecutive channels of T as float4: predicated load (zeros when off).
template <typename T>
struct Ch4;
template <>
struct Ch4<float> {
  __device__ static float4 load(const float *p, uint32_t pred) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %4, 0;\n\t"
                 "@q ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%5];\n\t}"
                 : "+f"(v.x), "+f"(v.y), "+f"(v.z), "+f"(v.w)
                 : "r"(pred), "l"(p));
    return v;
  }
};
template <typename H>
struct Ch4Half {
  __device__ static float4 load(const H *p, uint32_t pred) {
    uint32_t a = 0u, b = 0u;
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t"
                 "@q ld.global.nc.v2.b32 {%0, %1}, [%3];\n\t}"
                 : "+r"(a), "+r"(b)
                 : "r"(pred), "l"(p));
    const H *h = reinterpret_cast<const H *>(&a);
    const H *k = reinterpret_cast<const H *>(&b);
    return make_float4(to_f(h[0]), to_f(h[1]), to_f(k[0]), to_f(k[1]));
  }
};
template <>
struct Ch4<__half> : Ch4Half<__half> {};
template <>
struct Ch4<__nv_bfloat16> : Ch4Half<__nv_bfloat16> {};

__device__ __forceinline__ void red_add_v4(float *p, float4 v) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// Per-warp geometry table of one pass of 32 samples, corner-major: corner k's
// entries are 16 pairs of samples x {line, scale, line, scale} (line -1 for a
// corner outside the level, scale = corner weight x attention weight), with a
// 4-word pad between corners, so the 8 lanes of corner slot g read two
// samples' entries in one 16-byte load and the four slots hit distinct banks.
constexpr int kGeoCornerWords = 16 * 4 + 4;
constexpr int kGeoWords = 4 * kGeoCornerWords;

// BATCH samples are gathered together: their corner loads are issued, then
// the grad_value reds, then the per-lane partial dots.  The per-corner dots of
// a batch are folded by a reduce-scatter inside each 8-lane corner group (7
// shuffles for 8 samples, 4 for 4, where one shuffle per partial sum folded
// on its own cost 3), leaving lane j of every group with its corner's dot for
// one sample of the batch; the lane turns it into that corner's shares of
// grad_attn / grad_loc, and two more rounds of 3 shuffles sum the corners.
// UNITB: L*P is a multiple of BATCH, so a batch never straddles two (b, q, m)
// units and one grad_out vector serves the whole batch; otherwise each sample
// loads its own (an L1 hit for the unit's later samples).
template <typename T, int BATCH, bool UNITB>
__global__ void __launch_bounds__(kBwdWarps * 32)
msda_bwd_c32_kernel(const T *__restrict__ value, const int64_t *__restrict__ shapes,
                    const int64_t *__restrict__ lsi, const T *__restrict__ loc,
                    const T *__restrict__ attn, const T *__restrict__ grad_out,
                    float *__restrict__ grad_value, T *__restrict__ grad_loc,
                    T *__restrict__ grad_attn, int S, int heads, int L, int Q, int P,
                    int64_t n_samples) {
  static_assert(BATCH == 4 || BATCH == 8, "batches of 4 or 8 samples");
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  constexpr int C = 32;
  __shared__ int s_lvl[kMaxLevels][3];
  __shared__ __align__(16) uint32_t s_geo[kBwdWarps][kGeoWords];
  __shared__ float4 s_smp[kBwdWarps][32];  // per sample: lh, lw, W_l * a, H_l * a
  if (threadIdx.x < L) {
    s_lvl[threadIdx.x][0] = static_cast<int>(shapes[2 * threadIdx.x]);
    s_lvl[threadIdx.x][1] = static_cast<int>(shapes[2 * threadIdx.x + 1]);
    s_lvl[threadIdx.x][2] = static_cast<int>(lsi[threadIdx.x]);
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 3;  // corner of this lane
  const int j = lane & 7;   // 4-channel chunk
  const int LP = L * P;
  const uint32_t geo_s = ptx::smem_u32(&s_geo[warp][0]);
  const uint32_t my_geo = geo_s + 4u * (g * kGeoCornerWords);
  const int64_t passes = (n_samples + 31) / 32;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kBwdWarps;
  for (int64_t ps = static_cast<int64_t>(blockIdx.x) * kBwdWarps + warp; ps < passes;
       ps += stride) {
    const int64_t s0 = ps * 32;
    // ---- geometry of sample s0 + lane
    {
      int line[4] = {-1, -1, -1, -1};
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
      float4 fr = make_float4(0.f, 0.f, 0.f, 0.f);
      const int64_t smp = s0 + lane;
      if (smp < n_samples) {
        const int64_t u = smp / LP;
        const int lp = static_cast<int>(smp - u * LP);
        const int l = lp / P;
        const int m = static_cast<int>(u % heads);
        const int b = static_cast<int>(u / (static_cast<int64_t>(Q) * heads));
        const int Hl = s_lvl[l][0], Wl = s_lvl[l][1], start = s_lvl[l][2];
        const float lx = to_f(loc[2 * smp]), ly = to_f(loc[2 * smp + 1]);
        const float a = to_f(attn[smp]);
        const float h_im = __fmaf_rn(ly, static_cast<float>(Hl), -0.5f);
        const float w_im = __fmaf_rn(lx, static_cast<float>(Wl), -0.5f);
        fr.z = static_cast<float>(Wl) * a;
        fr.w = static_cast<float>(Hl) * a;
        if (h_im > -1.f && w_im > -1.f && h_im < static_cast<float>(Hl) &&
            w_im < static_cast<float>(Wl)) {
          const int h_low = static_cast<int>(floorf(h_im));
          const int w_low = static_cast<int>(floorf(w_im));
          const float lh = h_im - static_cast<float>(h_low);
          const float lw = w_im - static_cast<float>(w_low);
          const float hh = 1.f - lh, hw = 1.f - lw;
          fr.x = lh;
          fr.y = lw;
          const bool y0 = h_low >= 0, y1 = h_low + 1 <= Hl - 1;
          const bool x0 = w_low >= 0, x1 = w_low + 1 <= Wl - 1;
          // line of corner (y0, x0): the launcher checks B*S*heads fits 31 bits
          const int base = (b * S + start + h_low * Wl + w_low) * heads + m;
          if (y0 && x0) { line[0] = base;                   sc[0] = hh * hw * a; }
          if (y0 && x1) { line[1] = base + heads;           sc[1] = hh * lw * a; }
          if (y1 && x0) { line[2] = base + Wl * heads;      sc[2] = lh * hw * a; }
          if (y1 && x1) { line[3] = base + (Wl + 1) * heads; sc[3] = lh * lw * a; }
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t a_s =
            geo_s + 4u * (k * kGeoCornerWords + (lane >> 1) * 4 + (lane & 1) * 2);
        asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(a_s), "r"(line[k]),
                     "r"(__float_as_uint(sc[k]))
                     : "memory");
      }
      s_smp[warp][lane] = fr;
    }
    __syncwarp();

    const int n_here = n_samples - s0 < 32 ? static_cast<int>(n_samples - s0) : 32;
    // unit of the pass's first sample and the samples left in it (warp-uniform)
    int64_t u_cur = s0 / LP;
    int left = LP - static_cast<int>(s0 - u_cur * LP);
    float4 t_unit = make_float4(0.f, 0.f, 0.f, 0.f);
    if (UNITB) t_unit = Ch4<T>::load(grad_out + u_cur * C + 4 * j, 1u);
    for (int i0 = 0; i0 < n_here; i0 += BATCH) {
      float4 v[BATCH], t[BATCH];
      int ln[BATCH];
      float sc[BATCH];
      if (UNITB) {
        if (left == 0) {
          ++u_cur;
          left = LP;
          t_unit = Ch4<T>::load(grad_out + u_cur * C + 4 * j, 1u);
        }
        left -= BATCH;
      }
#pragma unroll
      for (int k = 0; k < BATCH; k += 2) {
        const uint4 e = ptx::ld_shared_v4(my_geo + 16u * ((i0 + k) >> 1));
        ln[k] = static_cast<int>(e.x);
        sc[k] = __uint_as_float(e.y);
        ln[k + 1] = static_cast<int>(e.z);
        sc[k + 1] = __uint_as_float(e.w);
      }
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        v[k] = Ch4<T>::load(value + static_cast<int64_t>(ln[k]) * C + 4 * j, ln[k] >= 0);
        if (!UNITB) {
          const bool here = i0 + k < n_here;
          if (here && left == 0) {
            ++u_cur;
            left = LP;
          }
          left -= here ? 1 : 0;
          t[k] = Ch4<T>::load(grad_out + u_cur * C + 4 * j, here);
        } else {
          t[k] = t_unit;
        }
      }
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        if (sc[k] != 0.f)  // a dropped corner and a zero weight add nothing
          red_add_v4(grad_value + static_cast<int64_t>(ln[k]) * C + 4 * j,
                     make_float4(sc[k] * t[k].x, sc[k] * t[k].y, sc[k] * t[k].z,
                                 sc[k] * t[k].w));
      }
      float p[BATCH];
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        float d = v[k].x * t[k].x;
        d = fmaf(v[k].y, t[k].y, d);
        d = fmaf(v[k].z, t[k].z, d);
        p[k] = fmaf(v[k].w, t[k].w, d);
      }
      // reduce-scatter over the 8 lanes of the corner group
      constexpr int H1 = BATCH / 2, H2 = BATCH / 4;
      const bool b2 = (j & 4) != 0, b1 = (j & 2) != 0, b0 = (j & 1) != 0;
      float q1[H1], q2[H2];
#pragma unroll
      for (int i = 0; i < H1; ++i) {
        const float send = b2 ? p[i] : p[i + H1];
        q1[i] = (b2 ? p[i + H1] : p[i]) + __shfl_xor_sync(0xffffffffu, send, 4);
      }
#pragma unroll
      for (int i = 0; i < H2; ++i) {
        const float send = b1 ? q1[i] : q1[i + H2];
        q2[i] = (b1 ? q1[i + H2] : q1[i]) + __shfl_xor_sync(0xffffffffu, send, 2);
      }
      float D;
      int si;  // sample of the batch whose corner-g dot this lane now holds
      if constexpr (BATCH == 8) {
        const float send = b0 ? q2[0] : q2[1];
        D = (b0 ? q2[1] : q2[0]) + __shfl_xor_sync(0xffffffffu, send, 1);
        si = i0 + j;
      } else {
        D = q2[0] + __shfl_xor_sync(0xffffffffu, q2[0], 1);
        si = i0 + (j >> 1);
      }
      const float4 fr = s_smp[warp][si];
      const float wy = (g & 2) ? fr.x : 1.f - fr.x;  // lh or hh
      const float wx = (g & 1) ? fr.y : 1.f - fr.y;  // lw or hw
      float qa = wy * wx * D;
      float qx = ((g & 1) ? wy : -wy) * D;
      float qy = ((g & 2) ? wx : -wx) * D;
#pragma unroll
      for (int o = 8; o <= 16; o <<= 1) {  // across the four corners
        qa += __shfl_xor_sync(0xffffffffu, qa, o);
        qx += __shfl_xor_sync(0xffffffffu, qx, o);
        qy += __shfl_xor_sync(0xffffffffu, qy, o);
      }
      if (g == 0 && (BATCH == 8 || !b0) && si < n_here) {
        const int64_t smp = s0 + si;
        grad_attn[smp] = from_f<T>(qa);
        grad_loc[2 * smp] = from_f<T>(fr.z * qx);
        grad_loc[2 * smp + 1] = from_f<T>(fr.w * qy);
      }
    }
    __syncwarp();
  }
}

// Any head dim: one warp per sample, lanes over channels.
template <typename T>
__global__ void __launch_bounds__(256)
msda_bwd_generic_kernel(const T *__restrict__ value, const int64_t *__restrict__ shapes,
                        const int64_t *__restrict__ lsi, const T *__restrict__ loc,
                        const T *__restrict__ attn, const T *__restrict__ grad_out,
                        float *__restrict__ grad_value, T *__restrict__ grad_loc,
                        T *__restrict__ grad_attn, int S, int heads, int C, int L, int Q,
                        int P, int64_t n_samples) {
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  const int lane = threadIdx.x & 31;
  const int64_t smp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (smp >= n_samples) return;
  const int LP = L * P;
  const int64_t u = smp / LP;
  const int l = static_cast<int>(smp - u * LP) / P;
  const int m = static_cast<int>(u % heads);
  const int64_t b = u / (static_cast<int64_t>(Q) * heads);
  const int Hl = static_cast<int>(shapes[2 * l]), Wl = static_cast<int>(shapes[2 * l + 1]);
  const int64_t start = lsi[l];
  const float lx = to_f(loc[2 * smp]), ly = to_f(loc[2 * smp + 1]), a = to_f(attn[smp]);
  const float h_im = __fmaf_rn(ly, static_cast<float>(Hl), -0.5f);
  const float w_im = __fmaf_rn(lx, static_cast<float>(Wl), -0.5f);
  float sa = 0.f, sx = 0.f, sy = 0.f;
  if (h_im > -1.f && w_im > -1.f && h_im < static_cast<float>(Hl) &&
      w_im < static_cast<float>(Wl)) {
    const int h_low = static_cast<int>(floorf(h_im)), w_low = static_cast<int>(floorf(w_im));
    const float lh = h_im - h_low, lw = w_im - w_low, hh = 1.f - lh, hw = 1.f - lw;
    const float wk[4] = {hh * hw, hh * lw, lh * hw, lh * lw};
    const float cx[4] = {-hh, hh, -lh, lh};
    const float cy[4] = {-hw, -lw, hw, lw};
    const int hs[4] = {h_low, h_low, h_low + 1, h_low + 1};
    const int ws[4] = {w_low, w_low + 1, w_low, w_low + 1};
    const T *g = grad_out + u * C;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (hs[k] < 0 || hs[k] > Hl - 1 || ws[k] < 0 || ws[k] > Wl - 1) continue;
      const int64_t line = (b * S + start + static_cast<int64_t>(hs[k]) * Wl + ws[k]) * heads + m;
      float d = 0.f;
      for (int c = lane; c < C; c += 32) {
        const float gc = to_f(g[c]);
        d = fmaf(to_f(value[line * C + c]), gc, d);
        atomicAdd(grad_value + line * C + c, wk[k] * a * gc);
      }
      sa = fmaf(wk[k], d, sa);
      sx = fmaf(cx[k], d, sx);
      sy = fmaf(cy[k], d, sy);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, o);
    sx += __shfl_xor_sync(0xffffffffu, sx, o);
    sy += __shfl_xor_sync(0xffffffffu, sy, o);
  }
  if (lane == 0) {
    grad_attn[smp] = from_f<T>(sa);
    grad_loc[2 * smp] = from_f<T>(static_cast<float>(Wl) * a * sx);
    grad_loc[2 * smp + 1] = from_f<T>(static_cast<float>(Hl) * a * sy);
  }
}

template <typename T>
__global__ void narrow_kernel(const float *__restrict__ src, T *__restrict__ dst, int64_t n) {
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = from_f<T>(src[i]);
}

template <typename T>
int launch_bwd_typed(const void *value, const int64_t *shapes, const int64_t *lsi,
                     const void *loc, const void *attn, const void *grad_out, void *grad_value,
                     void *grad_loc, void *grad_attn, int B, int S, int heads, int C, int L,
                     int Q, int P, void *workspace, size_t workspace_bytes,
                     cudaStream_t stream) {
  const int64_t n_samples = static_cast<int64_t>(B) * Q * heads * L * P;
  const int64_t n_value = static_cast<int64_t>(B) * S * heads * C;
  const bool f32 = sizeof(T) == 4;
  float *gv = f32 ? static_cast<float *>(grad_value) : static_cast<float *>(workspace);
  if (!f32) {
    if (workspace_bytes < static_cast<size_t>(n_value) * 4 || workspace == nullptr)
      return fail(BEVK_ERR_WORKSPACE, "msda backward: fp32 grad_value workspace of %lld bytes required",
                  static_cast<long long>(n_value) * 4);
    if (!aligned(workspace, 16))
      return fail(BEVK_ERR_MISALIGNED, "msda backward: workspace must be 16-byte aligned");
    if (n_value > 0 && cudaMemsetAsync(gv, 0, static_cast<size_t>(n_value) * 4, stream) != cudaSuccess)
      return fail(BEVK_ERR_CUDA, "msda backward: workspace memset failed");
  }
  if (n_samples > 0) {
    const int sms = device_info(current_device()).sm_count;
    const bool fast = C == 32 && L <= kMaxLevels && aligned(value, sizeof(T) * 4) &&
                      aligned(grad_out, sizeof(T) * 4) && aligned(gv, 16) &&
                      static_cast<int64_t>(B) * Q * heads < (int64_t(1) << 31) &&
                      static_cast<int64_t>(B) * S * heads < (int64_t(1) << 31);
    if (fast) {
      const int64_t passes = (n_samples + 31) / 32;
      const int64_t want = (passes + kBwdWarps - 1) / kBwdWarps;
      const int64_t ctas = std::min<int64_t>(want, static_cast<int64_t>(sms > 0 ? sms : 148) * 8);
      const int LP = L * P;
      const auto kern = LP % 8 == 0   ? msda_bwd_c32_kernel<T, 8, true>
                        : LP % 4 == 0 ? msda_bwd_c32_kernel<T, 4, true>
                                      : msda_bwd_c32_kernel<T, 4, false>;
      const int st = launched(
          launch_dependent(kern, dim3(static_cast<unsigned>(ctas)),
                           dim3(kBwdWarps * 32), 0, stream, static_cast<const T *>(value), shapes,
                           lsi, static_cast<const T *>(loc), static_cast<const T *>(attn),
                           static_cast<const T *>(grad_out), gv, static_cast<T *>(grad_loc),
                           static_cast<T *>(grad_attn), S, heads, L, Q, P, n_samples),
          "msda_bwd_c32_kernel");
      if (st != BEVK_OK) return st;
    } else {
      const int64_t blocks = (n_samples * 32 + 255) / 256;
      if (blocks > 0x7FFFFFFF) return fail(BEVK_ERR_INDEX_OVERFLOW, "msda backward: grid too large");
      const int st = launched(
          launch_dependent(msda_bwd_generic_kernel<T>, dim3(static_cast<unsigned>(blocks)),
                           dim3(256), 0, stream, static_cast<const T *>(value), shapes, lsi,
                           static_cast<const T *>(loc), static_cast<const T *>(attn),
                           static_cast<const T *>(grad_out), gv, static_cast<T *>(grad_loc),
                           static_cast<T *>(grad_attn), S, heads, C, L, Q, P, n_samples),
          "msda_bwd_generic_kernel");
      if (st != BEVK_OK) return st;
    }
  }
  if (!f32 && n_value > 0) {
    const int sms = device_info(current_device()).sm_count;
    const int64_t blocks = std::min<int64_t>((n_value + 255) / 256, static_cast<int64_t>(sms > 0 ? sms : 148) * 16);
    return launched(launch_dependent(narrow_kernel<T>, dim3(static_cast<unsigned>(blocks)),
                                     dim3(256), 0, stream, static_cast<const float *>(gv),
                                     static_cast<T *>(grad_value), n_value),
                    "msda narrow_kernel");
  }
  return BEVK_OK;
}

}  // namespace

size_t msda_backward_workspace_bytes(int B, int S, int heads, int C, int dtype) {
  if (dtype == BEVK_DTYPE_F32 || B <= 0 || S <= 0 || heads <= 0 || C <= 0) return 0;
  return static_cast<size_t>(B) * S * heads * C * 4;
}

int launch_msda_backward(const void *value, const int64_t *shapes, const int64_t *lsi,
                         const void *loc, const void *attn, const void *grad_out,
                         void *grad_value, void *grad_loc, void *grad_attn, int B, int S,
                         int heads, int C, int L, int Q, int P, void *workspace,
                         size_t workspace_bytes, int dtype, cudaStream_t stream) {
  switch (dtype) {
    case BEVK_DTYPE_F32:
      return launch_bwd_typed<float>(value, shapes, lsi, loc, attn, grad_out, grad_value,
                                     grad_loc, grad_attn, B, S, heads, C, L, Q, P, workspace,
                                     workspace_bytes, stream);
    case BEVK_DTYPE_F16:
      return launch_bwd_typed<__half>(value, shapes, lsi, loc, attn, grad_out, grad_value,
                                      grad_loc, grad_attn, B, S, heads, C, L, Q, P, workspace,
                                      workspace_bytes, stream);
    case BEVK_DTYPE_BF16:
      return launch_bwd_typed<__nv_bfloat16>(value, shapes, lsi, loc, attn, grad_out,
                                             grad_value, grad_loc, grad_attn, B, S, heads, C,
                                             L, Q, P, workspace, workspace_bytes, stream);
    default:
      return fail(BEVK_ERR_UNSUPPORTED, "msda backward: dtype %d not supported (f32, f16, bf16)",
                  dtype);
  }
}

}  // namespace bevk
