// dcn_simt.cu -- exact DCNv2 forward on CUDA cores, plus the layout helpers
// shared by every DCN path (weight packing, NCHW -> NHWC) and the
// reference-compatible column-matrix ops.
//
// The SIMT forward is an implicit GEMM: a CTA owns 64 output pixels x 64
// output channels of one convolution group and walks the reduction as
// (tap t, chunk of <= 16 input channels that stays inside one deformable
// group).  Per chunk it computes the tap geometry of its 64 pixels once,
// gathers the modulated bilinear samples into shared memory, stages the packed
// weights next to them and runs a 4x4-per-thread register-blocked FMA loop.
// fp32/f16/bf16 accumulate in fp32, fp64 in fp64.  It covers every geometry
// the reference accepts (groups, deformable groups, any kernel/stride/pad/
// dilation, any strides) and is the exact path for fp32 inputs, where the
// reference's 1e-5 tolerance rules out tf32/bf16 tensor-core arithmetic.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "bevk_internal.h"
#include "bevk_ptx.cuh"

namespace bevk {
namespace {

template <typename T>
__device__ __forceinline__ float ld_f(const T *p) { return static_cast<float>(*p); }
template <>
__device__ __forceinline__ float ld_f<__half>(const __half *p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16 *p) {
  return __bfloat162float(*p);
}

template <typename Acc, typename T>
__device__ __forceinline__ Acc ld_acc(const T *p) { return static_cast<Acc>(ld_f<T>(p)); }
template <>
__device__ __forceinline__ double ld_acc<double, double>(const double *p) { return *p; }

template <typename T, typename Acc>
__device__ __forceinline__ T store_cast(Acc v) { return static_cast<T>(v); }
template <>
__device__ __forceinline__ __half store_cast<__half, float>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 store_cast<__nv_bfloat16, float>(float v) {
  return __float2bfloat16_rn(v);
}

// Scalar-type helpers for the sampling math (fp64 problems sample in fp64,
// everything else in fp32 like the reference kernels).
template <typename Acc> __device__ __forceinline__ Acc floor_(Acc v);
template <> __device__ __forceinline__ float floor_<float>(float v) { return floorf(v); }
template <> __device__ __forceinline__ double floor_<double>(double v) { return floor(v); }
template <typename Acc> __device__ __forceinline__ Acc sigmoid_(Acc v);
template <> __device__ __forceinline__ float sigmoid_<float>(float v) { return 1.f / (1.f + __expf(-v)); }
template <> __device__ __forceinline__ double sigmoid_<double>(double v) { return 1.0 / (1.0 + exp(-v)); }

struct SimtParams {
  int B, Cin, H, W, Cout, kH, kW, T, sh, sw, ph, pw, dh, dw;
  int Ho, Wo, Cin_g, Cout_g, Cin_g_pad, cpdg, groups;
  int64_t M;
  int64_t xs[4], os[4], ms[4], ys[4];
  int mask_is_logit, has_bias, act_relu;
};

// Tap geometry of one (pixel, tap, deformable group): element offsets of the
// four corners (channel 0 of the pixel) and their weights (mask folded in).
template <typename Acc>
struct TapGeom {
  int64_t off[4];
  Acc w[4];
};

template <typename Acc, typename T>
__device__ __forceinline__ TapGeom<Acc> tap_geometry(const SimtParams &p, const T *off,
                                                     const T *msk, int64_t m, int t, int dgi) {
  TapGeom<Acc> g;
#pragma unroll
  for (int q = 0; q < 4; ++q) { g.off[q] = 0; g.w[q] = Acc(0); }
  if (m >= p.M) return g;
  const int64_t HoWo = static_cast<int64_t>(p.Ho) * p.Wo;
  const int b = static_cast<int>(m / HoWo);
  const int rem = static_cast<int>(m - b * HoWo);
  const int oh = rem / p.Wo, ow = rem - (rem / p.Wo) * p.Wo;
  const int ki = t / p.kW, kj = t - (t / p.kW) * p.kW;
  const int taps = p.T;
  const T *ob = off + b * p.os[0] + oh * p.os[2] + ow * p.os[3];
  const Acc off_h = ld_acc<Acc>(ob + (static_cast<int64_t>(dgi) * 2 * taps + 2 * t) * p.os[1]);
  const Acc off_w = ld_acc<Acc>(ob + (static_cast<int64_t>(dgi) * 2 * taps + 2 * t + 1) * p.os[1]);
  Acc mk = ld_acc<Acc>(msk + b * p.ms[0] + (static_cast<int64_t>(dgi) * taps + t) * p.ms[1] +
                       oh * p.ms[2] + ow * p.ms[3]);
  if (p.mask_is_logit) mk = sigmoid_<Acc>(mk);
  const Acc h_im = static_cast<Acc>(oh * p.sh - p.ph + ki * p.dh) + off_h;
  const Acc w_im = static_cast<Acc>(ow * p.sw - p.pw + kj * p.dw) + off_w;
  if (!(h_im > Acc(-1) && w_im > Acc(-1) && h_im < static_cast<Acc>(p.H) &&
        w_im < static_cast<Acc>(p.W)))
    return g;
  const int h_low = static_cast<int>(floor_<Acc>(h_im));
  const int w_low = static_cast<int>(floor_<Acc>(w_im));
  const Acc lh = h_im - static_cast<Acc>(h_low), lw = w_im - static_cast<Acc>(w_low);
  const Acc hh = Acc(1) - lh, hw = Acc(1) - lw;
  const int64_t xb = b * p.xs[0];
  const bool y0 = h_low >= 0, y1 = h_low + 1 <= p.H - 1;
  const bool x0 = w_low >= 0, x1 = w_low + 1 <= p.W - 1;
  if (y0 && x0) { g.off[0] = xb + h_low * p.xs[2] + w_low * p.xs[3];             g.w[0] = hh * hw * mk; }
  if (y0 && x1) { g.off[1] = xb + h_low * p.xs[2] + (w_low + 1) * p.xs[3];       g.w[1] = hh * lw * mk; }
  if (y1 && x0) { g.off[2] = xb + (h_low + 1) * p.xs[2] + w_low * p.xs[3];       g.w[2] = lh * hw * mk; }
  if (y1 && x1) { g.off[3] = xb + (h_low + 1) * p.xs[2] + (w_low + 1) * p.xs[3]; g.w[3] = lh * lw * mk; }
  return g;
}

constexpr int BM = 64, BN = 64, BK = 16, NT = 256;

template <typename T, typename Acc>
__global__ void __launch_bounds__(NT)
dcn_fwd_simt_kernel(SimtParams p, const T *__restrict__ x, const T *__restrict__ off,
                    const T *__restrict__ msk, const T *__restrict__ wpk,
                    const T *__restrict__ bias, T *__restrict__ y) {
  __shared__ TapGeom<Acc> s_geo[BM];
  __shared__ Acc s_a[BK][BM + 4];
  __shared__ Acc s_b[BK][BN + 4];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * BM;
  const int n_tiles_g = (p.Cout_g + BN - 1) / BN;
  const int grp = blockIdx.y / n_tiles_g;
  const int n0 = (blockIdx.y - grp * n_tiles_g) * BN;  // within the group
  const int c_base = grp * p.Cin_g;                    // first input channel of the group

  Acc acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) acc[i][jj] = Acc(0);

  for (int t = 0; t < p.T; ++t) {
    for (int c0 = 0; c0 < p.Cin_g;) {
      // chunk [c0, c1): at most BK channels, never crossing a deformable group
      const int cg = c_base + c0;
      const int dgi = cg / p.cpdg;
      const int dg_end = (dgi + 1) * p.cpdg - c_base;
      const int c1 = min(min(c0 + BK, p.Cin_g), dg_end);
      const int clen = c1 - c0;
      if (tid < BM) s_geo[tid] = tap_geometry<Acc>(p, off, msk, m0 + tid, t, dgi);
      __syncthreads();
      // gather: 64 pixels x 16 channels, channel fastest
#pragma unroll
      for (int i = 0; i < (BM * BK) / NT; ++i) {
        const int e = tid + i * NT;
        const int r = e / BK, ci = e - (e / BK) * BK;
        Acc v = Acc(0);
        if (ci < clen) {
          const TapGeom<Acc> &g = s_geo[r];
          const int64_t co = static_cast<int64_t>(cg + ci) * p.xs[1];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (g.w[q] != Acc(0)) v += g.w[q] * ld_acc<Acc>(x + g.off[q] + co);
        }
        s_a[ci][r] = v;
      }
      // packed weights [Cout][T][Cin_g_pad]: 64 output channels x 16 channels
#pragma unroll
      for (int i = 0; i < (BN * BK) / NT; ++i) {
        const int e = tid + i * NT;
        const int n = e / BK, ci = e - (e / BK) * BK;
        const int co = n0 + n;
        Acc v = Acc(0);
        if (ci < clen && co < p.Cout_g)
          v = ld_acc<Acc>(wpk + (static_cast<int64_t>(grp) * p.Cout_g + co) * p.T * p.Cin_g_pad +
                          static_cast<int64_t>(t) * p.Cin_g_pad + c0 + ci);
        s_b[ci][n] = v;
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < BK; ++k) {
        Acc a[4], bb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = s_a[k][ty * 4 + i];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) bb[jj] = s_b[k][tx * 4 + jj];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) acc[i][jj] += a[i] * bb[jj];
      }
      __syncthreads();
      c0 = c1;
    }
  }

  const int64_t HoWo = static_cast<int64_t>(p.Ho) * p.Wo;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= p.M) continue;
    const int b = static_cast<int>(m / HoWo);
    const int rem = static_cast<int>(m - b * HoWo);
    const int oh = rem / p.Wo, ow = rem - (rem / p.Wo) * p.Wo;
    T *yb = y + b * p.ys[0] + oh * p.ys[2] + ow * p.ys[3];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int co = n0 + tx * 4 + jj;
      if (co >= p.Cout_g) continue;
      const int cog = grp * p.Cout_g + co;
      Acc v = acc[i][jj];
      if (p.has_bias) v += ld_acc<Acc>(bias + cog);
      if (p.act_relu && v < Acc(0)) v = Acc(0);
      yb[static_cast<int64_t>(cog) * p.ys[1]] = store_cast<T, Acc>(v);
    }
  }
}

// ---------------------------------------------------------------- small problems
// Small problems (few 64 x 64 tiles, e.g. 1 x 64 x 32 x 32): a CTA owns SBM = 16
// output pixels x 64 output channels, so four times as many CTAs run; the
// reduction walks chunks of up to SBK = 64 channels (one chunk a tap when
// Cin_g <= 64); the geometry of every (tap, deformable group) of the CTA's
// pixels is computed once up front; and the next chunk's samples and weights
// are loaded into registers while the current chunk's products accumulate, so
// each chunk costs about one global-memory latency.  With three or more taps
// and few tiles, the taps are split over a cluster of 3 CTAs (grid z), each
// walking a third of the chunks; rank 0 adds the other two partial tiles,
// read through distributed shared memory in rank order, before the epilogue.
// Same sampling arithmetic as the large kernel (fp32/fp64, Acc accumulation);
// the sum over the taps is grouped in thirds.
constexpr int SBM = 16, SBK = 64;
constexpr int kSmallA = SBM * SBK / NT;   // gathered samples a thread loads per chunk
constexpr int kSmallB = BN * SBK / NT;    // weights a thread loads per chunk

template <typename T, typename Acc>
__global__ void __launch_bounds__(NT)
dcn_fwd_simt_small_kernel(SimtParams p, const T *__restrict__ x, const T *__restrict__ off,
                          const T *__restrict__ msk, const T *__restrict__ wpk,
                          const T *__restrict__ bias, T *__restrict__ y) {
  // dynamic shared memory: the double-buffered A / B chunks, then the
  // geometry [T * dg][SBM]
  extern __shared__ __align__(16) unsigned char simt_small_smem[];
  using ATile = Acc[SBK][SBM + 1];
  using BTile = Acc[SBK][BN + 4];
  ATile *s_a = reinterpret_cast<ATile *>(simt_small_smem);
  BTile *s_b = reinterpret_cast<BTile *>(simt_small_smem + 2 * sizeof(ATile));
  TapGeom<Acc> *s_geo =
      reinterpret_cast<TapGeom<Acc> *>(simt_small_smem + 2 * sizeof(ATile) + 2 * sizeof(BTile));

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * SBM;
  const int n_tiles_g = (p.Cout_g + BN - 1) / BN;
  const int grp = blockIdx.y / n_tiles_g;
  const int n0 = (blockIdx.y - grp * n_tiles_g) * BN;
  const int c_base = grp * p.Cin_g;
  const bool cl = p.xs[1] == 1;   // channel-contiguous input: channels fastest across threads

  // K split across a cluster of gridDim.z CTAs: CTA z walks taps
  // [t_lo, t_hi) and the cluster's partial tiles are summed at the end
  const int ks = static_cast<int>(gridDim.z);
  const int t_lo = p.T * static_cast<int>(blockIdx.z) / ks;
  const int t_hi = p.T * (static_cast<int>(blockIdx.z) + 1) / ks;

  // geometry of every (tap, deformable group) x pixel of this tile (of the
  // CTA's taps)
  const int n_geo = p.T * (p.Cin / p.cpdg);   // taps x deformable groups
  for (int e = tid; e < n_geo * SBM; e += NT) {
    const int tg = e / SBM, r = e - (e / SBM) * SBM;
    const int t = tg % p.T, dgi = tg / p.T;
    if (t >= t_lo && t < t_hi) s_geo[e] = tap_geometry<Acc>(p, off, msk, m0 + r, t, dgi);
  }
  __syncthreads();

  // chunk k -> (tap t, channels [c0, c1) of the group, never crossing a
  // deformable group); chunks are walked tap-major like the large kernel
  struct Chunk {
    int t, c0, c1, dgi;
  };
  auto chunk_at = [&](int t, int c0) {
    const int cg = c_base + c0;
    const int dgi = cg / p.cpdg;
    const int dg_end = (dgi + 1) * p.cpdg - c_base;
    return Chunk{t, c0, min(min(c0 + SBK, p.Cin_g), dg_end), dgi};
  };
  auto next_chunk = [&](Chunk c, bool &more) {
    if (c.c1 < p.Cin_g) return chunk_at(c.t, c.c1);
    if (c.t + 1 < t_hi) return chunk_at(c.t + 1, 0);
    more = false;
    return c;
  };
  Acc ra[kSmallA], rb[kSmallB];
  auto load = [&](const Chunk &c) {
    const int clen = c.c1 - c.c0;
    const TapGeom<Acc> *geo = s_geo + (c.dgi * p.T + c.t) * SBM;
    // every corner load is issued before any is used: a dropped corner has
    // offset 0 (a valid address) and weight 0, and is skipped in the sum
    Acc raw[kSmallA][4];
#pragma unroll
    for (int i = 0; i < kSmallA; ++i) {
      const int e = tid + i * NT;
      const int r = cl ? e / SBK : e % SBM;
      const int ci = cl ? e % SBK : e / SBM;
      const TapGeom<Acc> &g = geo[r];
      const int64_t co = static_cast<int64_t>(c_base + c.c0 + min(ci, clen - 1)) * p.xs[1];
#pragma unroll
      for (int q = 0; q < 4; ++q) raw[i][q] = ld_acc<Acc>(x + g.off[q] + co);
    }
#pragma unroll
    for (int i = 0; i < kSmallA; ++i) {
      const int e = tid + i * NT;
      const int r = cl ? e / SBK : e % SBM;
      const int ci = cl ? e % SBK : e / SBM;
      const TapGeom<Acc> &g = geo[r];
      Acc v = Acc(0);
      if (ci < clen) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (g.w[q] != Acc(0)) v += g.w[q] * raw[i][q];
      }
      ra[i] = v;
    }
#pragma unroll
    for (int i = 0; i < kSmallB; ++i) {
      const int e = tid + i * NT;
      const int n = e / SBK, ci = e - (e / SBK) * SBK;
      const int co = n0 + n;
      Acc v = Acc(0);
      if (ci < clen && co < p.Cout_g)
        v = ld_acc<Acc>(wpk + (static_cast<int64_t>(grp) * p.Cout_g + co) * p.T * p.Cin_g_pad +
                        static_cast<int64_t>(c.t) * p.Cin_g_pad + c.c0 + ci);
      rb[i] = v;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int i = 0; i < kSmallA; ++i) {
      const int e = tid + i * NT;
      const int r = cl ? e / SBK : e % SBM;
      const int ci = cl ? e % SBK : e / SBM;
      s_a[buf][ci][r] = ra[i];
    }
#pragma unroll
    for (int i = 0; i < kSmallB; ++i) {
      const int e = tid + i * NT;
      s_b[buf][e % SBK][e / SBK] = rb[i];
    }
  };

  Acc acc[4] = {Acc(0), Acc(0), Acc(0), Acc(0)};
  Chunk cur = chunk_at(t_lo, 0);
  load(cur);
  store(0);
  __syncthreads();
  int buf = 0;
  bool more = true;
  while (true) {
    const Chunk nxt = next_chunk(cur, more);
    if (more) load(nxt);          // in flight while this chunk accumulates
    const int clen = cur.c1 - cur.c0;
    for (int k = 0; k < clen; ++k) {
      const Acc a = s_a[buf][k][ty];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) acc[jj] += a * s_b[buf][k][tx * 4 + jj];
    }
    if (!more) break;
    store(buf ^ 1);
    __syncthreads();
    buf ^= 1;
    cur = nxt;
  }

  if (ks > 1) {
    // partial tiles through distributed shared memory: every CTA leaves its
    // sums in its A buffers, rank 0 adds the others' in rank order (so the
    // result does not depend on timing) and writes the output; the second
    // barrier keeps the other CTAs resident until rank 0 has read them
    Acc *part = reinterpret_cast<Acc *>(simt_small_smem);
    static_assert(SBM * BN * sizeof(Acc) <= 2 * sizeof(ATile), "partial tile fits the A buffers");
    __syncthreads();  // every thread is done reading the chunk buffers
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) part[ty * BN + tx * 4 + jj] = acc[jj];
    ptx::cluster_sync();
    if (ptx::cluster_ctarank() == 0) {
      for (int r = 1; r < ks; ++r) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const uint32_t a = ptx::mapa_shared(ptx::smem_u32(&part[ty * BN + tx * 4 + jj]),
                                              static_cast<uint32_t>(r));
          Acc v;
          if constexpr (sizeof(Acc) == 8) {
            asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(a) : "memory");
          } else {
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
          }
          acc[jj] += v;
        }
      }
    }
    ptx::cluster_sync();
    if (ptx::cluster_ctarank() != 0) return;
  }

  const int64_t m = m0 + ty;
  if (m >= p.M) return;
  const int64_t HoWo = static_cast<int64_t>(p.Ho) * p.Wo;
  const int b = static_cast<int>(m / HoWo);
  const int rem = static_cast<int>(m - b * HoWo);
  const int oh = rem / p.Wo, ow = rem - (rem / p.Wo) * p.Wo;
  T *yb = y + b * p.ys[0] + oh * p.ys[2] + ow * p.ys[3];
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const int co = n0 + tx * 4 + jj;
    if (co >= p.Cout_g) continue;
    const int cog = grp * p.Cout_g + co;
    Acc v = acc[jj];
    if (p.has_bias) v += ld_acc<Acc>(bias + cog);
    if (p.act_relu && v < Acc(0)) v = Acc(0);
    yb[static_cast<int64_t>(cog) * p.ys[1]] = store_cast<T, Acc>(v);
  }
}

// ---------------------------------------------------------------- packing
// wpk[co][t][c] = weight[co][c][t] for c < Cin_g, 0 for the padding.
template <typename T>
__global__ void pack_weight_kernel(const T *__restrict__ w, T *__restrict__ wpk, int Cout,
                                   int Cin_g, int T_, int Cin_g_pad) {
  const int64_t n = static_cast<int64_t>(Cout) * T_ * Cin_g_pad;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % Cin_g_pad);
    const int64_t r = i / Cin_g_pad;
    const int t = static_cast<int>(r % T_);
    const int64_t co = r / T_;
    wpk[i] = c < Cin_g ? w[(co * Cin_g + c) * T_ + t] : T(0);
  }
}

// dst[b][h][w][c] = src[b, c, h, w] (any strides) through a 32x32 smem tile
// per (b, c-block, hw-block).
template <typename T>
__global__ void nchw_to_nhwc_kernel(const T *__restrict__ src, T *__restrict__ dst, int C,
                                    int H, int W, int64_t s0, int64_t s1, int64_t s2,
                                    int64_t s3) {
  __shared__ T tile[32][33];
  const int HW = H * W;
  const int b = blockIdx.z;
  const int c0 = blockIdx.y * 32, p0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, pix = p0 + threadIdx.x;
    if (c < C && pix < HW) {
      const int hh = pix / W, ww = pix - (pix / W) * W;
      tile[i][threadIdx.x] = src[b * s0 + c * s1 + hh * s2 + ww * s3];
    }
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int pix = p0 + i, c = c0 + threadIdx.x;
    if (c < C && pix < HW) dst[(static_cast<int64_t>(b) * HW + pix) * C + c] = tile[threadIdx.x][i];
  }
}

// ---------------------------------------------------------------- columns
// Column matrix of the reference ops: one thread per (pixel, tap, channel
// block), geometry once, then the channel loop.  Layout 0 writes
// col[(c*T + t), m] (coalesced across pixels), layout 1 writes col[m, t*C + c].
template <typename T>
__global__ void __launch_bounds__(256)
im2col_kernel(SimtParams p, const T *__restrict__ x, const T *__restrict__ off,
              const T *__restrict__ msk, T *__restrict__ col, int layout, int cblock) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t MT = p.M * p.T;
  if (i >= MT) return;
  const int t = static_cast<int>(i / p.M);
  const int64_t m = i - t * p.M;
  const int c_begin = blockIdx.y * cblock;
  const int c_end = min(p.Cin, c_begin + cblock);
  int dgi = -1;
  TapGeom<float> g;
  for (int c = c_begin; c < c_end; ++c) {
    const int d = c / p.cpdg;
    if (d != dgi) { g = tap_geometry<float>(p, off, msk, m, t, d); dgi = d; }
    const int64_t co = static_cast<int64_t>(c) * p.xs[1];
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (g.w[q] != 0.f) v += g.w[q] * ld_f<T>(x + g.off[q] + co);
    const int64_t dst = layout == 0 ? (static_cast<int64_t>(c) * p.T + t) * p.M + m
                                    : m * p.T * p.Cin + static_cast<int64_t>(t) * p.Cin + c;
    col[dst] = store_cast<T, float>(v);
  }
}

// NHWC column matrix col[m, t*C + c] from channel-contiguous input (one
// deformable group): one warp per (pixel, tap), lanes over the channels in
// 16-byte vectors, so corner reads and column writes are whole-warp
// contiguous segments.  Units run taps fastest, so consecutive warps write
// consecutive parts of a pixel's column row.
template <typename T>
__global__ void __launch_bounds__(256)
im2col_nhwc_vec_kernel(SimtParams p, const T *__restrict__ x, const T *__restrict__ off,
                       const T *__restrict__ msk, T *__restrict__ col) {
  constexpr int V = 16 / sizeof(T);
  const int64_t unit = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (unit >= p.M * p.T) return;
  const int lane = threadIdx.x & 31;
  const int t = static_cast<int>(unit % p.T);
  const int64_t m = unit / p.T;
  const TapGeom<float> g = tap_geometry<float>(p, off, msk, m, t, 0);
  T *dst = col + m * p.T * p.Cin + static_cast<int64_t>(t) * p.Cin;
  for (int c = lane * V; c < p.Cin; c += 32 * V) {
    float acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (g.w[q] == 0.f) continue;
      const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(x + g.off[q] + c));
      const T *e = reinterpret_cast<const T *>(&raw);
#pragma unroll
      for (int v = 0; v < V; ++v) acc[v] = fmaf(g.w[q], ld_f<T>(e + v), acc[v]);
    }
    uint4 outv;
    T *o = reinterpret_cast<T *>(&outv);
#pragma unroll
    for (int v = 0; v < V; ++v) o[v] = store_cast<T, float>(acc[v]);
    *reinterpret_cast<uint4 *>(dst + c) = outv;
  }
}

template <>
__global__ void __launch_bounds__(256)
im2col_kernel<double>(SimtParams p, const double *__restrict__ x, const double *__restrict__ off,
                      const double *__restrict__ msk, double *__restrict__ col, int layout,
                      int cblock) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t MT = p.M * p.T;
  if (i >= MT) return;
  const int t = static_cast<int>(i / p.M);
  const int64_t m = i - t * p.M;
  const int c_begin = blockIdx.y * cblock;
  const int c_end = min(p.Cin, c_begin + cblock);
  int dgi = -1;
  TapGeom<double> g;
  for (int c = c_begin; c < c_end; ++c) {
    const int d = c / p.cpdg;
    if (d != dgi) { g = tap_geometry<double>(p, off, msk, m, t, d); dgi = d; }
    const int64_t co = static_cast<int64_t>(c) * p.xs[1];
    double v = 0.0;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (g.w[q] != 0.0) v += g.w[q] * x[g.off[q] + co];
    const int64_t dst = layout == 0 ? (static_cast<int64_t>(c) * p.T + t) * p.M + m
                                    : m * p.T * p.Cin + static_cast<int64_t>(t) * p.Cin + c;
    col[dst] = v;
  }
}

SimtParams make_params(const bevk_dcn_problem *pr, const DcnDims &d) {
  SimtParams p;
  p.B = d.B; p.Cin = d.Cin; p.H = d.H; p.W = d.W; p.Cout = d.Cout;
  p.kH = d.kH; p.kW = d.kW; p.T = d.T;
  p.sh = d.sh; p.sw = d.sw; p.ph = d.ph; p.pw = d.pw; p.dh = d.dh; p.dw = d.dw;
  p.Ho = d.Ho; p.Wo = d.Wo; p.Cin_g = d.Cin_g; p.Cout_g = d.Cout_g; p.Cin_g_pad = d.Cin_g_pad;
  p.cpdg = d.cpdg; p.groups = d.groups; p.M = d.M;
  for (int i = 0; i < 4; ++i) {
    p.xs[i] = pr->input_strides[i];
    p.os[i] = pr->offset_strides[i];
    p.ms[i] = pr->mask_strides[i];
    p.ys[i] = pr->output_strides[i];
  }
  p.mask_is_logit = pr->mask_is_logit;
  p.has_bias = pr->has_bias;
  p.act_relu = pr->act_relu;
  return p;
}

template <typename T, typename Acc>
int launch_simt_typed(const bevk_dcn_problem *pr, const DcnDims &d, const void *x,
                      const void *off, const void *msk, const void *wpk, const void *bias,
                      void *y, cudaStream_t stream) {
  const SimtParams p = make_params(pr, d);
  const int64_t mt = (d.M + BM - 1) / BM;
  const int64_t nt = static_cast<int64_t>(d.groups) * ((d.Cout_g + BN - 1) / BN);
  if (mt > 0x7FFFFFFF || nt > 65535)
    return fail(BEVK_ERR_INDEX_OVERFLOW, "dcn simt: grid (%lld x %lld) too large",
                static_cast<long long>(mt), static_cast<long long>(nt));
  // Fewer 64 x 64 tiles than two per SM: the small-tile kernel (its up-front
  // geometry of every (tap, deformable group) must fit in 48 KB).
  const int sms = device_info(current_device()).sm_count > 0
                      ? device_info(current_device()).sm_count : 148;
  const size_t geo_bytes = sizeof(TapGeom<Acc>) * SBM * d.T * d.dg;
  if (mt * nt < 2 * sms && geo_bytes <= 48 * 1024) {
    const size_t tiles = 2 * sizeof(Acc) * SBK * ((SBM + 1) + (BN + 4));
    const size_t smem = tiles + geo_bytes;
    constexpr int kMaxDevices = 64;
    static std::atomic<bool> sized[kMaxDevices];
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices || !sized[dev].load(std::memory_order_relaxed)) {
      if (cudaFuncSetAttribute(dcn_fwd_simt_small_kernel<T, Acc>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(tiles + 48 * 1024)) != cudaSuccess) {
        (void)cudaGetLastError();
        return fail(BEVK_ERR_CUDA, "dcn simt: cannot size shared memory");
      }
      if (dev >= 0 && dev < kMaxDevices) sized[dev].store(true, std::memory_order_relaxed);
    }
    const int64_t smt = (d.M + SBM - 1) / SBM;
    // The taps are split over a cluster of 3 CTAs when the tiles are few:
    // each CTA's chain of dependent chunks (one global round trip each) is
    // then a third as long (1 x 64 x 32 x 32 fp32: 64 tiles x 9 taps, 35.5 ->
    // 22.3 us on B200); the partial tiles are summed over distributed shared
    // memory in a fixed order
    constexpr int kSplit = 3;
    const int ks = d.T >= kSplit && smt * nt * kSplit <= 4 * static_cast<int64_t>(sms) ? kSplit : 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(smt), static_cast<unsigned>(nt), static_cast<unsigned>(ks));
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = static_cast<unsigned>(ks);
    cfg.attrs = attr;
    cfg.numAttrs = ks > 1 ? 1 : 0;
    return launched(cudaLaunchKernelEx(&cfg, dcn_fwd_simt_small_kernel<T, Acc>, p,
                                       static_cast<const T *>(x), static_cast<const T *>(off),
                                       static_cast<const T *>(msk), static_cast<const T *>(wpk),
                                       static_cast<const T *>(bias), static_cast<T *>(y)),
                    "dcn_fwd_simt_small_kernel");
  }
  dim3 grid(static_cast<unsigned>(mt), static_cast<unsigned>(nt));
  dcn_fwd_simt_kernel<T, Acc><<<grid, NT, 0, stream>>>(
      p, static_cast<const T *>(x), static_cast<const T *>(off), static_cast<const T *>(msk),
      static_cast<const T *>(wpk), static_cast<const T *>(bias), static_cast<T *>(y));
  return check_launch("dcn_fwd_simt_kernel");
}

template <typename T>
int launch_im2col_typed(const bevk_dcn_problem *pr, const DcnDims &d, const void *x,
                        const void *off, const void *msk, void *col, int layout,
                        cudaStream_t stream) {
  const SimtParams p = make_params(pr, d);
  const int64_t MT = d.M * d.T;
  if constexpr (sizeof(T) <= 4) {
    constexpr int V = 16 / sizeof(T);
    const bool vec = layout == 1 && d.dg == 1 && d.Cin % V == 0 && pr->input_strides[1] == 1 &&
                     pr->input_strides[0] % V == 0 && pr->input_strides[2] % V == 0 &&
                     pr->input_strides[3] % V == 0 && aligned(x, 16) && aligned(col, 16);
    if (vec) {
      const int64_t blocks = (MT * 32 + 255) / 256;
      if (blocks > 0x7FFFFFFF) return fail(BEVK_ERR_INDEX_OVERFLOW, "im2col: grid too large");
      im2col_nhwc_vec_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
          p, static_cast<const T *>(x), static_cast<const T *>(off), static_cast<const T *>(msk),
          static_cast<T *>(col));
      return check_launch("im2col_nhwc_vec_kernel");
    }
  }
  const int cblock = 64;
  const int64_t bx = (MT + 255) / 256;
  const int by = (d.Cin + cblock - 1) / cblock;
  if (bx > 0x7FFFFFFF || by > 65535) return fail(BEVK_ERR_INDEX_OVERFLOW, "im2col: grid too large");
  dim3 grid(static_cast<unsigned>(bx), by);
  im2col_kernel<T><<<grid, 256, 0, stream>>>(p, static_cast<const T *>(x),
                                             static_cast<const T *>(off),
                                             static_cast<const T *>(msk), static_cast<T *>(col),
                                             layout, cblock);
  return check_launch("im2col_kernel");
}

}  // namespace

int launch_dcn_forward_simt(const bevk_dcn_problem *p, const DcnDims &d, const void *x,
                            const void *off, const void *msk, const void *wpk,
                            const void *bias, void *out, cudaStream_t stream) {
  switch (p->dtype) {
    case BEVK_DTYPE_F32: return launch_simt_typed<float, float>(p, d, x, off, msk, wpk, bias, out, stream);
    case BEVK_DTYPE_F64: return launch_simt_typed<double, double>(p, d, x, off, msk, wpk, bias, out, stream);
    case BEVK_DTYPE_F16: return launch_simt_typed<__half, float>(p, d, x, off, msk, wpk, bias, out, stream);
    case BEVK_DTYPE_BF16: return launch_simt_typed<__nv_bfloat16, float>(p, d, x, off, msk, wpk, bias, out, stream);
    default: return fail(BEVK_ERR_UNSUPPORTED, "dcn: dtype %d not supported", p->dtype);
  }
}

int launch_dcn_pack_weight(const DcnDims &d, const void *w, void *wpk, int dtype,
                           cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>(d.Cout) * d.T * d.Cin_g_pad;
  const int blocks = static_cast<int>(n / 256 + 1 < 65535 ? n / 256 + 1 : 65535);
  switch (dtype_size(dtype)) {
    case 2:
      pack_weight_kernel<uint16_t><<<blocks, 256, 0, stream>>>(
          static_cast<const uint16_t *>(w), static_cast<uint16_t *>(wpk), d.Cout, d.Cin_g, d.T,
          d.Cin_g_pad);
      break;
    case 4:
      pack_weight_kernel<uint32_t><<<blocks, 256, 0, stream>>>(
          static_cast<const uint32_t *>(w), static_cast<uint32_t *>(wpk), d.Cout, d.Cin_g, d.T,
          d.Cin_g_pad);
      break;
    case 8:
      pack_weight_kernel<uint64_t><<<blocks, 256, 0, stream>>>(
          static_cast<const uint64_t *>(w), static_cast<uint64_t *>(wpk), d.Cout, d.Cin_g, d.T,
          d.Cin_g_pad);
      break;
    default:
      return fail(BEVK_ERR_UNSUPPORTED, "pack_weight: dtype %d", dtype);
  }
  return check_launch("pack_weight_kernel");
}

int launch_nchw_to_nhwc(const void *src, void *dst, int B, int C, int H, int W,
                        const int64_t s[4], int dtype, cudaStream_t stream) {
  dim3 grid((H * W + 31) / 32, (C + 31) / 32, B);
  dim3 block(32, 8);
  if (grid.y > 65535 || grid.z > 65535) return fail(BEVK_ERR_INDEX_OVERFLOW, "transpose: grid too large");
  switch (dtype_size(dtype)) {
    case 2:
      nchw_to_nhwc_kernel<uint16_t><<<grid, block, 0, stream>>>(
          static_cast<const uint16_t *>(src), static_cast<uint16_t *>(dst), C, H, W, s[0], s[1],
          s[2], s[3]);
      break;
    case 4:
      nchw_to_nhwc_kernel<uint32_t><<<grid, block, 0, stream>>>(
          static_cast<const uint32_t *>(src), static_cast<uint32_t *>(dst), C, H, W, s[0], s[1],
          s[2], s[3]);
      break;
    case 8:
      nchw_to_nhwc_kernel<uint64_t><<<grid, block, 0, stream>>>(
          static_cast<const uint64_t *>(src), static_cast<uint64_t *>(dst), C, H, W, s[0], s[1],
          s[2], s[3]);
      break;
    default:
      return fail(BEVK_ERR_UNSUPPORTED, "transpose: dtype %d", dtype);
  }
  return check_launch("nchw_to_nhwc_kernel");
}

int launch_dcn_im2col(const bevk_dcn_problem *p, const DcnDims &d, const void *x,
                      const void *off, const void *msk, void *col, int layout,
                      cudaStream_t stream) {
  switch (p->dtype) {
    case BEVK_DTYPE_F32: return launch_im2col_typed<float>(p, d, x, off, msk, col, layout, stream);
    case BEVK_DTYPE_F64: return launch_im2col_typed<double>(p, d, x, off, msk, col, layout, stream);
    case BEVK_DTYPE_F16: return launch_im2col_typed<__half>(p, d, x, off, msk, col, layout, stream);
    case BEVK_DTYPE_BF16: return launch_im2col_typed<__nv_bfloat16>(p, d, x, off, msk, col, layout, stream);
    default: return fail(BEVK_ERR_UNSUPPORTED, "im2col: dtype %d not supported", p->dtype);
  }
}

}  // namespace bevk
