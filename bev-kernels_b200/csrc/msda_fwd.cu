// msda_fwd.cu -- multi-scale deformable attention forward for sm_100a.
//
// Semantics follow csrc_musa/msda/ms_deform_attn_kernels.cuh:559-623 (generic
// im2col) and :51-284 (spec warp kernel):
//   out[b, q, m*C + c] = sum_{l,p} attn[b,q,m,l,p] * bilinear(value_l[b, :, m, c],
//                        h = loc_y*H_l - 0.5, w = loc_x*W_l - 0.5)
// with a sample dropped unless -1 < h < H_l and -1 < w < W_l and each of the
// four corners zeroed outside [0, H_l-1] x [0, W_l-1].  h and w are one fused
// multiply-add each (__fmaf_rn), which is how nvcc compiles the reference's
// `loc * H - 0.5f`; the bilinear derivative in the backward jumps at integer
// coordinates, so the rounding of this expression is part of the contract.
//
// Design (C == 32, the BEVFormer head dim; L*P samples per (b, q, head) unit):
// * Pass kernel (L*P = 4, 8, 16): a warp takes passes of 32 samples (32/(L*P)
//   units).  Lane s computes the geometry of sample s -- four corner line
//   indices and the four bilinear weights with the attention weight folded in
//   -- into shared memory; the next pass's locations and weights are already
//   being loaded.  Each sample then costs the warp ONE load instruction
//   covering all four corners: lanes 8g..8g+7 read corner g's 32-channel line
//   as 4-channel vectors, predicated (no branches), in batches.  Each lane
//   keeps a 4-channel partial sum for its corner slot; the slots of two
//   consecutive units are folded together when the second one is done.  Passes are dealt
//   round-robin over a grid of exactly the resident CTAs, so the grid walks
//   the units in (batch, head, query) order together.  A warp's passes are a
//   fixed number of units apart, so each lane advances its (batch, head,
//   query) by that stride with carries instead of dividing per pass.
// * Warp-per-unit kernel (other L*P): the same corner-slot mapping, one unit
//   per warp, its samples in rounds of 32.  Its geometry table is corner-major
//   with two samples' (line, weight) entries per 16-byte word, so the slot's
//   lanes read two samples' geometry in one shared-memory load (about 1.2
//   shared-memory wavefronts per sample against 2.1 for separate line and
//   weight reads), and a batch's corner loads are predicated, not branched.
// * Any other head dim: one thread per output element.
// The gather is bound by the 16-byte loads a warp can keep in flight, which
// the register file caps; batch sizes and CTAs per SM are the measured best.
// No tensor cores: this is a gather, not a contraction.
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

template <typename T>
struct Vec4;  // 4 channels of T, loaded as one vector
template <>
struct Vec4<float> {
  using type = float4;
  __device__ static float4 to_f32(float4 v) { return v; }
  __device__ static float4 from_f32(float4 v) { return v; }
};
template <>
struct Vec4<__half> {
  using type = uint2;
  __device__ static float4 to_f32(uint2 v) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&v.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&v.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  __device__ static uint2 from_f32(float4 f) {
    __half2 a = __floats2half2_rn(f.x, f.y), b = __floats2half2_rn(f.z, f.w);
    return make_uint2(*reinterpret_cast<uint32_t *>(&a), *reinterpret_cast<uint32_t *>(&b));
  }
};
template <>
struct Vec4<__nv_bfloat16> {
  using type = uint2;
  __device__ static float4 to_f32(uint2 v) {
    return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                       __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
  }
  __device__ static uint2 from_f32(float4 f) {
    __nv_bfloat162 a = __floats2bfloat162_rn(f.x, f.y), b = __floats2bfloat162_rn(f.z, f.w);
    return make_uint2(*reinterpret_cast<uint32_t *>(&a), *reinterpret_cast<uint32_t *>(&b));
  }
};

template <typename T>
__device__ __forceinline__ float to_f32(T v) { return static_cast<float>(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v) { return static_cast<T>(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

constexpr int kWarps = 8;
// Per-warp geometry table of one round of 32 samples, corner-major: corner k's
// entries are 16 pairs of samples x {line, weight, line, weight}, with a
// 4-word pad between corners.  Lane s writes its sample's four corners with
// conflict-free 8-byte stores; the 8 lanes of corner slot g then read two
// samples' entries in one 16-byte load, the four slots hitting distinct banks.
constexpr int kGeoCornerWords = 16 * 4 + 4;
constexpr int kGeoWords = 4 * kGeoCornerWords;

// Predicated vector loads of 4 channels (zeros when `pred` is 0).
__device__ __forceinline__ uint4 ld_pred16(const void *p, uint32_t pred);
__device__ __forceinline__ uint2 ld_pred8(const void *p, uint32_t pred);
template <typename T>
struct RawVec4;

template <typename T, int BATCH>
__global__ void __launch_bounds__(kWarps * 32)
msda_fwd_c32_kernel(const T *__restrict__ value, const int64_t *__restrict__ shapes,
                    const int64_t *__restrict__ lsi, const T *__restrict__ loc,
                    const T *__restrict__ attn, T *__restrict__ out, int S, int heads,
                    int L, int Q, int P, int64_t units) {
  static_assert(BATCH % 2 == 0 && 32 % BATCH == 0, "BATCH: an even divisor of 32");
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  using R = RawVec4<T>;
  using RT = typename R::type;
  using V = Vec4<T>;
  using VT = typename V::type;
  constexpr int C = 32;
  __shared__ int s_lvl[kMaxLevels][3];  // H, W, start
  __shared__ __align__(16) uint32_t s_geo[kWarps][kGeoWords];

  if (threadIdx.x < L) {
    s_lvl[threadIdx.x][0] = static_cast<int>(shapes[2 * threadIdx.x]);
    s_lvl[threadIdx.x][1] = static_cast<int>(shapes[2 * threadIdx.x + 1]);
    s_lvl[threadIdx.x][2] = static_cast<int>(lsi[threadIdx.x]);
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (unit >= units) return;

  const int m = static_cast<int>(unit % heads);
  const int64_t b = unit / (static_cast<int64_t>(Q) * heads);
  const T *vbase = value + b * S * heads * C;
  const int LP = L * P;
  const T *uloc = loc + unit * LP * 2;
  const T *uattn = attn + unit * LP;

  const int g = lane >> 3;  // corner slot
  const int j = lane & 7;   // 4-channel vector within the head's 32 channels
  const uint32_t geo_s = ptx::smem_u32(&s_geo[warp][0]);
  const uint32_t my_geo = geo_s + 4u * (g * kGeoCornerWords);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);

  for (int s0 = 0; s0 < LP; s0 += 32) {
    const int s = s0 + lane;
    int idx[4] = {0, 0, 0, 0};
    float wk[4] = {0.f, 0.f, 0.f, 0.f};
    if (s < LP) {
      const int l = s / P;
      const int Hl = s_lvl[l][0], Wl = s_lvl[l][1], start = s_lvl[l][2];
      const float lx = to_f32(uloc[2 * s]);
      const float ly = to_f32(uloc[2 * s + 1]);
      const float a = to_f32(uattn[s]);
      const float h_im = __fmaf_rn(ly, static_cast<float>(Hl), -0.5f);
      const float w_im = __fmaf_rn(lx, static_cast<float>(Wl), -0.5f);
      if (h_im > -1.f && w_im > -1.f && h_im < static_cast<float>(Hl) &&
          w_im < static_cast<float>(Wl)) {
        const int h_low = static_cast<int>(floorf(h_im));
        const int w_low = static_cast<int>(floorf(w_im));
        const float lh = h_im - static_cast<float>(h_low);
        const float lw = w_im - static_cast<float>(w_low);
        const float hh = 1.f - lh, hw = 1.f - lw;
        const bool y0 = h_low >= 0, y1 = h_low + 1 <= Hl - 1;
        const bool x0 = w_low >= 0, x1 = w_low + 1 <= Wl - 1;
        const int base = start + h_low * Wl + w_low;  // pixel of corner (y0, x0)
        if (y0 && x0) { idx[0] = base * heads + m;            wk[0] = hh * hw * a; }
        if (y0 && x1) { idx[1] = (base + 1) * heads + m;      wk[1] = hh * lw * a; }
        if (y1 && x0) { idx[2] = (base + Wl) * heads + m;     wk[2] = lh * hw * a; }
        if (y1 && x1) { idx[3] = (base + Wl + 1) * heads + m; wk[3] = lh * lw * a; }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t a_s =
          geo_s + 4u * (k * kGeoCornerWords + (lane >> 1) * 4 + (lane & 1) * 2);
      asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(a_s), "r"(idx[k]),
                   "r"(__float_as_uint(wk[k]))
                   : "memory");
    }
    __syncwarp();
    // samples in batches of BATCH: a batch's corner loads are issued together
    // (predicated off for dropped corners and for entries past the round's
    // last sample, whose weights are 0), then consumed
    const int nb = (min(32, LP - s0) + BATCH - 1) / BATCH;
    for (int bt = 0; bt < nb; ++bt) {
      RT vb[BATCH];
      float w[BATCH];
#pragma unroll
      for (int k = 0; k < BATCH; k += 2) {
        const uint4 e = ptx::ld_shared_v4(my_geo + 16u * ((bt * BATCH + k) >> 1));
        w[k] = __uint_as_float(e.y);
        w[k + 1] = __uint_as_float(e.w);
        vb[k] = R::load(vbase + static_cast<int64_t>(static_cast<int>(e.x)) * C + j * 4,
                        w[k] != 0.f);
        vb[k + 1] = R::load(vbase + static_cast<int64_t>(static_cast<int>(e.z)) * C + j * 4,
                            w[k + 1] != 0.f);
      }
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        ptx::reg_fence(vb[k]);
        ptx::reg_fence(w[k]);
      }
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        const float4 v = R::f32(vb[k]);
        acc.x = fmaf(w[k], v.x, acc.x);
        acc.y = fmaf(w[k], v.y, acc.y);
        acc.z = fmaf(w[k], v.z, acc.z);
        acc.w = fmaf(w[k], v.w, acc.w);
      }
      ptx::reg_fence(acc.x);
      ptx::reg_fence(acc.y);
      ptx::reg_fence(acc.z);
      ptx::reg_fence(acc.w);
    }
    __syncwarp();
  }
#pragma unroll
  for (int o = 8; o <= 16; o <<= 1) {
    acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
    acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
    acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
    acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
  }
  if (lane < 8) reinterpret_cast<VT *>(out + unit * C)[j] = V::from_f32(acc);
}

// Predicated vector loads of 4 channels (zeros when `pred` is 0).
__device__ __forceinline__ uint4 ld_pred16(const void *p, uint32_t pred) {
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %4, 0;\n\t"
      "@q ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%5];\n\t}"
      : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w)
      : "r"(pred), "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ld_pred8(const void *p, uint32_t pred) {
  uint2 v = make_uint2(0u, 0u);
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t"
      "@q ld.global.nc.v2.u32 {%0, %1}, [%3];\n\t}"
      : "+r"(v.x), "+r"(v.y)
      : "r"(pred), "l"(p));
  return v;
}
template <typename T>
struct RawVec4;  // raw bits of 4 channels
template <>
struct RawVec4<float> {
  using type = uint4;
  __device__ static uint4 load(const void *p, uint32_t pred) { return ld_pred16(p, pred); }
  __device__ static float4 f32(uint4 v) {
    return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z),
                       __uint_as_float(v.w));
  }
};
template <>
struct RawVec4<__half> {
  using type = uint2;
  __device__ static uint2 load(const void *p, uint32_t pred) { return ld_pred8(p, pred); }
  __device__ static float4 f32(uint2 v) { return Vec4<__half>::to_f32(v); }
};
template <>
struct RawVec4<__nv_bfloat16> {
  using type = uint2;
  __device__ static uint2 load(const void *p, uint32_t pred) { return ld_pred8(p, pred); }
  __device__ static float4 f32(uint2 v) { return Vec4<__nv_bfloat16>::to_f32(v); }
};

struct CornerGeom {
  int idx;   // line index (pixel * heads + head) relative to the camera's value base
  float w;   // bilinear weight * attention weight; 0 for a dropped corner
};
constexpr int kPassWarps = 16;

// LP = L*P samples per unit (a divisor of 32).  Loads go out in batches of
// BATCH samples; with DB the next batch is issued before the current one is
// consumed.  MINB is the number of CTAs per SM the register budget is cut for.
template <typename T, int LP, int BATCH, bool DB, int MINB, bool GIDX>
__global__ void __launch_bounds__(kPassWarps * 32, MINB)
msda_fwd_pass_kernel(const T *__restrict__ value, const int64_t *__restrict__ shapes,
                     const int64_t *__restrict__ lsi, const T *__restrict__ loc,
                     const T *__restrict__ attn, T *__restrict__ out, int S, int heads, int L,
                     int Q, int P, int64_t passes) {
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  static_assert(32 % LP == 0, "LP must divide 32");
  constexpr int C = 32;
  constexpr int UPP = 32 / LP;  // units per pass
  static_assert(UPP % 2 == 0, "units are folded in pairs");
  using R = RawVec4<T>;
  using RT = typename R::type;
  using V = Vec4<T>;
  using VT = typename V::type;
  __shared__ int s_lvl[kMaxLevels][3];
  __shared__ CornerGeom s_geo[kPassWarps][32][4];
  __shared__ int64_t s_vbase[kPassWarps][UPP];   // value element offset of the unit's camera
  __shared__ int64_t s_obase[kPassWarps][UPP];   // output element offset of the unit

  if (threadIdx.x < L) {
    s_lvl[threadIdx.x][0] = static_cast<int>(shapes[2 * threadIdx.x]);
    s_lvl[threadIdx.x][1] = static_cast<int>(shapes[2 * threadIdx.x + 1]);
    s_lvl[threadIdx.x][2] = static_cast<int>(lsi[threadIdx.x]);
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 3;  // corner slot
  const int j = lane & 7;   // 4-channel chunk of the head's 32 channels
  // Passes are dealt round-robin to the warps of all CTAs, so the grid walks the
  // units in (b, h, q) order together and the value lines in use at any moment
  // are those of about one (camera, head) slice -- small enough to stay in L2
  // even when the whole value tensor is not.
  const int64_t p_stride = static_cast<int64_t>(gridDim.x) * kPassWarps;
  const int64_t p_first = static_cast<int64_t>(blockIdx.x) * kPassWarps + warp;
  const int64_t HQ = static_cast<int64_t>(heads) * Q;
  const int my_l = (lane % LP) / P;  // level of this lane's sample (fixed across passes)

  // Unit (b, h, q) of this lane's sample, in (b, h, q) order.  A warp's
  // passes are p_stride apart, i.e. a fixed number of units, so the position
  // of the next pass is the current one plus that stride's (b, h, q) with
  // carries: one division per thread at the start instead of two 64-bit
  // divisions per pass.
  struct UPos {
    int b, h, q;
  };
  auto decompose = [&](int64_t v) {
    UPos r;
    r.b = static_cast<int>(v / HQ);
    const int64_t rr = v - static_cast<int64_t>(r.b) * HQ;
    r.h = static_cast<int>(rr / Q);
    r.q = static_cast<int>(rr - static_cast<int64_t>(r.h) * Q);
    return r;
  };
  const UPos step = decompose(p_stride * UPP);
  auto advance = [&](UPos &u) {
    u.q += step.q;
    int c = u.q >= Q ? 1 : 0;
    u.q -= c ? Q : 0;
    u.h += step.h + c;
    c = u.h >= heads ? 1 : 0;
    u.h -= c ? heads : 0;
    u.b += step.b + c;
  };
  // raw location / attention of this lane's sample at unit position `up`
  auto fetch = [&](const UPos &up, float &lx, float &ly, float &a) {
    const int64_t u = (static_cast<int64_t>(up.b) * Q + up.q) * heads + up.h;  // memory order (b, q, h)
    const int i = lane % LP;
    lx = to_f32(loc[(u * LP + i) * 2]);
    ly = to_f32(loc[(u * LP + i) * 2 + 1]);
    a = to_f32(attn[u * LP + i]);
  };

  float lx = 0.f, ly = 0.f, a = 0.f;
  UPos nxt = decompose(p_first * UPP + lane / LP);
  if (p_first < passes) fetch(nxt, lx, ly, a);
  for (int64_t ps = p_first; ps < passes; ps += p_stride) {
    // ---- geometry of this pass (lane = sample)
    const UPos cur = nxt;
    advance(nxt);
    const int64_t b = cur.b, q = cur.q;
    const int h = cur.h;
    {
      const int Hl = s_lvl[my_l][0], Wl = s_lvl[my_l][1], start = s_lvl[my_l][2];
      CornerGeom cg[4] = {{0, 0.f}, {0, 0.f}, {0, 0.f}, {0, 0.f}};
      const float h_im = __fmaf_rn(ly, static_cast<float>(Hl), -0.5f);
      const float w_im = __fmaf_rn(lx, static_cast<float>(Wl), -0.5f);
      if (h_im > -1.f && w_im > -1.f && h_im < static_cast<float>(Hl) &&
          w_im < static_cast<float>(Wl)) {
        const int h_low = static_cast<int>(floorf(h_im));
        const int w_low = static_cast<int>(floorf(w_im));
        const float lh = h_im - static_cast<float>(h_low);
        const float lw = w_im - static_cast<float>(w_low);
        const float hh = 1.f - lh, hw = 1.f - lw;
        const bool y0 = h_low >= 0, y1 = h_low + 1 <= Hl - 1;
        const bool x0 = w_low >= 0, x1 = w_low + 1 <= Wl - 1;
        // GIDX: line index over all cameras (the launcher checks it fits
        // 32 bits), so the gather needs no per-unit camera base
        const int base = (GIDX ? static_cast<int>(b) * S : 0) + start + h_low * Wl + w_low;
        if (y0 && x0) cg[0] = {base * heads + h, hh * hw * a};
        if (y0 && x1) cg[1] = {(base + 1) * heads + h, hh * lw * a};
        if (y1 && x0) cg[2] = {(base + Wl) * heads + h, lh * hw * a};
        if (y1 && x1) cg[3] = {(base + Wl + 1) * heads + h, lh * lw * a};
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) s_geo[warp][lane][k] = cg[k];
      if (lane % LP == 0) {
        if (!GIDX) s_vbase[warp][lane / LP] = b * S * heads * C;
        s_obase[warp][lane / LP] = ((b * Q + q) * heads + h) * C;
      }
    }
    __syncwarp();
    // next pass's raw inputs are loaded while this pass gathers
    if (ps + p_stride < passes) fetch(nxt, lx, ly, a);

    // ---- gather: batches of BATCH samples
    RT buf[DB ? 2 : 1][BATCH];
    float wbuf[DB ? 2 : 1][BATCH];
    auto issue = [&](int bt, RT (&vb)[BATCH], float (&wb)[BATCH]) {
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        const int smp = bt * BATCH + k;
        const CornerGeom cgk = s_geo[warp][smp][g];
        // camera of this sample's unit (units of a pass may straddle cameras)
        const T *vb_ptr = value + (GIDX ? int64_t(0) : s_vbase[warp][smp / LP]) +
                          static_cast<int64_t>(cgk.idx) * C + j * 4;
        wb[k] = cgk.w;
        vb[k] = R::load(vb_ptr, cgk.w != 0.f);
      }
    };
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    // The corner slots of two consecutive units are folded together: the
    // lane halves exchange one unit each (xor 16), then the quarters finish
    // (xor 8) -- 8 shuffles for two units where folding each alone takes 16;
    // slots 0 and 2 then hold units 0 and 1 (cfg4 fp32 102 -> 96 us, fp16 92
    // -> 81 us on B200; folding four units at once spilled and took 97 / 85).
    float4 held[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    auto fold_store = [&](int u0) {
      const bool hi = (g & 2) != 0;
      auto xr = [](float4 v, int o) {
        return make_float4(__shfl_xor_sync(0xffffffffu, v.x, o), __shfl_xor_sync(0xffffffffu, v.y, o),
                           __shfl_xor_sync(0xffffffffu, v.z, o), __shfl_xor_sync(0xffffffffu, v.w, o));
      };
      auto add = [](float4 a, float4 b) {
        return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
      };
      float4 r = add(hi ? held[1] : held[0], xr(hi ? held[0] : held[1], 16));
      r = add(r, xr(r, 8));
      if ((g & 1) == 0)
        reinterpret_cast<VT *>(out + s_obase[warp][u0 + (hi ? 1 : 0)])[j] = V::from_f32(r);
    };
    auto consume = [&](int bt, RT (&vb)[BATCH], float (&wb)[BATCH]) {
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        ptx::reg_fence(vb[k]);
        ptx::reg_fence(wb[k]);
      }
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        const int smp = bt * BATCH + k;
        const float4 v = R::f32(vb[k]);
        acc.x = fmaf(wb[k], v.x, acc.x);
        acc.y = fmaf(wb[k], v.y, acc.y);
        acc.z = fmaf(wb[k], v.z, acc.z);
        acc.w = fmaf(wb[k], v.w, acc.w);
        if ((smp + 1) % LP == 0) {  // last sample of a unit
          const int uu = smp / LP;   // unit within the pass (compile-time after unrolling)
          held[uu % 2] = acc;
          acc = make_float4(0.f, 0.f, 0.f, 0.f);
          if (uu % 2 == 1) fold_store(uu - 1);
        }
      }
    };
    if constexpr (DB) {
      issue(0, buf[0], wbuf[0]);
#pragma unroll
      for (int bt = 0; bt < 32 / BATCH; ++bt) {
        if (bt + 1 < 32 / BATCH) issue(bt + 1, buf[(bt + 1) & 1], wbuf[(bt + 1) & 1]);
        consume(bt, buf[bt & 1], wbuf[bt & 1]);
      }
    } else {
#pragma unroll
      for (int bt = 0; bt < 32 / BATCH; ++bt) {
        issue(bt, buf[0], wbuf[0]);
        consume(bt, buf[0], wbuf[0]);
      }
    }
    __syncwarp();
  }
}

// Any head dim: one thread per output element (b, q, m, c).
template <typename T>
__global__ void __launch_bounds__(256)
msda_fwd_generic_kernel(const T *__restrict__ value, const int64_t *__restrict__ shapes,
                        const int64_t *__restrict__ lsi, const T *__restrict__ loc,
                        const T *__restrict__ attn, T *__restrict__ out, int S, int heads,
                        int C, int L, int Q, int P, int64_t n) {
  ptx::grid_launch_dependents();
  ptx::grid_wait_prerequisites();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int c = static_cast<int>(i % C);
  const int64_t unit = i / C;
  const int m = static_cast<int>(unit % heads);
  const int64_t b = unit / (static_cast<int64_t>(Q) * heads);
  const int LP = L * P;
  const T *uloc = loc + unit * LP * 2;
  const T *uattn = attn + unit * LP;
  float acc = 0.f;
  for (int l = 0; l < L; ++l) {
    const int Hl = static_cast<int>(shapes[2 * l]), Wl = static_cast<int>(shapes[2 * l + 1]);
    const T *vl = value + (b * S + lsi[l]) * heads * C + static_cast<int64_t>(m) * C + c;
    const int64_t ws = static_cast<int64_t>(heads) * C, hs = Wl * ws;
    for (int p = 0; p < P; ++p) {
      const int s = l * P + p;
      const float h_im = __fmaf_rn(to_f32(uloc[2 * s + 1]), static_cast<float>(Hl), -0.5f);
      const float w_im = __fmaf_rn(to_f32(uloc[2 * s]), static_cast<float>(Wl), -0.5f);
      if (!(h_im > -1.f && w_im > -1.f && h_im < static_cast<float>(Hl) &&
            w_im < static_cast<float>(Wl)))
        continue;
      const int h_low = static_cast<int>(floorf(h_im)), w_low = static_cast<int>(floorf(w_im));
      const float lh = h_im - h_low, lw = w_im - w_low, hh = 1.f - lh, hw = 1.f - lw;
      float v1 = 0.f, v2 = 0.f, v3 = 0.f, v4 = 0.f;
      if (h_low >= 0 && w_low >= 0) v1 = to_f32(vl[h_low * hs + w_low * ws]);
      if (h_low >= 0 && w_low + 1 <= Wl - 1) v2 = to_f32(vl[h_low * hs + (w_low + 1) * ws]);
      if (h_low + 1 <= Hl - 1 && w_low >= 0) v3 = to_f32(vl[(h_low + 1) * hs + w_low * ws]);
      if (h_low + 1 <= Hl - 1 && w_low + 1 <= Wl - 1)
        v4 = to_f32(vl[(h_low + 1) * hs + (w_low + 1) * ws]);
      acc += (hh * hw * v1 + hh * lw * v2 + lh * hw * v3 + lh * lw * v4) * to_f32(uattn[s]);
    }
  }
  out[i] = from_f32<T>(acc);
}

// Resident CTAs per SM of one pass-kernel instantiation, computed once per
// device; the grid is exactly that many CTAs per SM (the kernel loops).
template <typename T, int LP, int BATCH, bool DB, int MINB, bool GIDX>
int launch_pass(const void *value, const int64_t *shapes, const int64_t *lsi, const void *loc,
                const void *attn, int S, int heads, int L, int Q, int P, void *out,
                int64_t passes, cudaStream_t stream) {
  constexpr int kMaxDevices = 64;
  static std::atomic<int> resident[kMaxDevices];
  const int dev = current_device();
  const auto kern = msda_fwd_pass_kernel<T, LP, BATCH, DB, MINB, GIDX>;
  int per_sm = (dev >= 0 && dev < kMaxDevices) ? resident[dev].load(std::memory_order_relaxed) : 0;
  if (per_sm <= 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kPassWarps * 32, 0) !=
            cudaSuccess ||
        per_sm <= 0)
      return fail(BEVK_ERR_CUDA, "msda: occupancy query failed");
    if (dev >= 0 && dev < kMaxDevices) resident[dev].store(per_sm, std::memory_order_relaxed);
  }
  const int sms = device_info(dev).sm_count;
  const int64_t ctas =
      std::min<int64_t>(passes, static_cast<int64_t>(sms > 0 ? sms : 148) * per_sm);
  return launched(launch_dependent(kern, dim3(static_cast<unsigned>(ctas)), dim3(kPassWarps * 32),
                                   0, stream, static_cast<const T *>(value), shapes, lsi,
                                   static_cast<const T *>(loc), static_cast<const T *>(attn),
                                   static_cast<T *>(out), S, heads, L, Q, P, passes),
                  "msda_fwd_pass_kernel");
}

template <typename T>
int launch_typed(const void *value, const int64_t *shapes, const int64_t *lsi, const void *loc,
                 const void *attn, int B, int S, int heads, int C, int L, int Q, int P,
                 void *out, cudaStream_t stream) {
  const int64_t units = static_cast<int64_t>(B) * Q * heads;
  if (units == 0) return BEVK_OK;
  const size_t vec_bytes = sizeof(T) * 4;
  const bool fast = C == 32 && L <= kMaxLevels && aligned(value, vec_bytes) &&
                    aligned(out, vec_bytes);
  const int LP = L * P;
  // Batch sizes and CTAs per SM measured on B200 (1 level, P=4, Q=40000: 132 us
  // with batches of 4 at 2 CTAs/SM against 158 us with double-buffered batches of
  // 8 at 1 CTA/SM).  At L*P = 32 the warp-per-unit kernel is faster (499 us
  // against 532 us on the 4-level, P=8 encoder workload), so it keeps that case.
  if (fast && LP >= 4 && LP <= 16 && 32 % LP == 0 && units % (32 / LP) == 0) {
    const int64_t passes = units / (32 / LP);
    // fp16/bf16 values with line indices over all cameras that fit 32 bits:
    // no per-unit camera base (cfg4 fp16 104.3 -> 98.9 us on B200; for fp32
    // the same change measured 110.1 -> 118.6 us, so fp32 keeps the base)
    const bool gidx = sizeof(T) == 2 &&
                      static_cast<int64_t>(B) * S * heads < (int64_t(1) << 31);
#define BEVK_PASS(LPV, MB)                                                                     \
  case LPV:                                                                                    \
    return gidx ? launch_pass<T, LPV, 4, false, MB, true>(value, shapes, lsi, loc, attn, S,    \
                                                           heads, L, Q, P, out, passes, stream) \
                : launch_pass<T, LPV, 4, false, MB, false>(value, shapes, lsi, loc, attn, S,   \
                                                            heads, L, Q, P, out, passes, stream);
    switch (LP) {
      BEVK_PASS(4, 2)
      BEVK_PASS(8, 2)
      BEVK_PASS(16, 3)
#undef BEVK_PASS
      default:
        break;
    }
  }
  if (fast) {
    const int64_t blocks = (units + kWarps - 1) / kWarps;
    if (blocks > 0x7FFFFFFF) return fail(BEVK_ERR_INDEX_OVERFLOW, "msda: grid too large");
    // loads in flight per warp: 16 fp32 or 8 half-width samples (cfg5 on B200:
    // fp32 480 -> 440 us against the earlier per-corner table, fp16 436 -> 402 us;
    // fp32 batches of 8 took 458 us, fp16 batches of 16 407 us)
    const auto kern = sizeof(T) == 4 ? msda_fwd_c32_kernel<T, 16> : msda_fwd_c32_kernel<T, 8>;
    return launched(launch_dependent(kern, dim3(static_cast<unsigned>(blocks)),
                                     dim3(kWarps * 32), 0, stream, static_cast<const T *>(value),
                                     shapes, lsi, static_cast<const T *>(loc),
                                     static_cast<const T *>(attn), static_cast<T *>(out), S,
                                     heads, L, Q, P, units),
                    "msda_fwd_c32_kernel");
  }
  const int64_t n = units * C;
  const int64_t blocks = (n + 255) / 256;
  if (blocks > 0x7FFFFFFF) return fail(BEVK_ERR_INDEX_OVERFLOW, "msda: grid too large");
  return launched(launch_dependent(msda_fwd_generic_kernel<T>, dim3(static_cast<unsigned>(blocks)),
                                   dim3(256), 0, stream, static_cast<const T *>(value), shapes,
                                   lsi, static_cast<const T *>(loc), static_cast<const T *>(attn),
                                   static_cast<T *>(out), S, heads, C, L, Q, P, n),
                  "msda_fwd_generic_kernel");
}

}  // namespace

int launch_msda_forward(const void *value, const int64_t *shapes, const int64_t *lsi,
                        const void *loc, const void *attn, int B, int S, int heads, int C,
                        int L, int Q, int P, void *out, int dtype, cudaStream_t stream) {
  switch (dtype) {
    case BEVK_DTYPE_F32:
      return launch_typed<float>(value, shapes, lsi, loc, attn, B, S, heads, C, L, Q, P, out,
                                 stream);
    case BEVK_DTYPE_F16:
      return launch_typed<__half>(value, shapes, lsi, loc, attn, B, S, heads, C, L, Q, P, out,
                                  stream);
    case BEVK_DTYPE_BF16:
      return launch_typed<__nv_bfloat16>(value, shapes, lsi, loc, attn, B, S, heads, C, L, Q, P,
                                         out, stream);
    default:
      return fail(BEVK_ERR_UNSUPPORTED, "msda: dtype %d not supported (f32, f16, bf16)", dtype);
  }
}

}  // namespace bevk
