// dcn_tc.cu -- fused DCNv2 forward on the sm_100a tensor cores (tcgen05/TMEM).
//
// out[m, co] = bias[co] + sum_{t, c} A[m, (t, c)] * W[co, t, c]
// A[m, (t, c)] = mask(m, t) * bilinear(x[b(m)], p(m) + tap(t) + offset(m, t))[c]
//
// One CTA computes a 128-pixel x BN-output-channel tile.  The reduction runs
// over (tap, 64-channel chunk) stages:
//   * 16 gather warps build the A stage in shared memory directly in the
//     canonical K-major 128-byte-swizzled UMMA layout: 8 lanes cover one
//     pixel's 64 channels (16-byte vector loads from NHWC input, one load per
//     bilinear corner), interpolate (packed half2 / bf16x2 FMA chains, each
//     step rounded to the input type), and st.shared the
//     result -- the column matrix never touches HBM;
//   * 1 TMA warp streams the matching [BN x 64] tile of the packed weights
//     ([Cout][tap][Cin_pad], K-major, 128-byte swizzle) into shared memory;
//   * 1 MMA warp allocates the TMEM accumulator and issues, from one thread,
//     tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) x 4 per stage,
//     committing each stage back to its "empty" barrier;
//   * warps 0-15 then drain TMEM (tcgen05.ld 32x32b), add bias and
//     store fp16/bf16 to any output layout.
// Pipelining uses full/empty mbarrier rings.  Every wait is bounded (2 s);
// a wait that gives up records its site in g_bevk_watchdog, raises a CTA-wide
// abort flag so the other roles unwind, and the CTA still frees its TMEM.
//
// The per-(pixel, tap) geometry (corner base offset + four corner weights with
// the mask folded in) is computed once per tile into shared memory; offset and
// mask tensors may have any strides (NCHW as in
// ModulatedDeformConv2dFunction, NHWC / fused logits as in
// DCNSplitNHWCFunction), matching csrc/modulated_deform_conv_cuda_kernel.cuh
// :403-470 and csrc/dcn_fused_nhwc_kernel.cuh:85-194 semantics.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>

#include "bevk_internal.h"
#include "bevk_ptx.cuh"

namespace bevk {

// Device watchdog word: set by a bounded wait that expired (see bevk.h).
__device__ unsigned int g_bevk_watchdog = 0;

namespace {
// 128 bytes of zeros: corner reads that fall outside the image load from here
// (never written; static device memory starts zeroed).
__device__ __align__(128) uint32_t g_dcn_zero_line[32];
}  // namespace

namespace {

constexpr int kBM = 128;           // pixels per tile (UMMA M)
constexpr int kBK = 64;            // channels per stage (128 B of fp16/bf16)
constexpr int kGatherWarps = 16;
constexpr int kEpilogueWarps = 16;  // warps 0-15: four per TMEM lane quadrant (w % 4)
constexpr int kMaxTaps = 9;
constexpr int kSplitCols = 256;     // K split: accumulator columns each half finishes

// Watchdog sites (low byte) -- identify which wait expired.
enum : unsigned int {
  kSiteGatherEmpty = 0xB0C1,
  kSiteTmaEmpty = 0xB0C2,
  kSiteMmaFull = 0xB0C3,
  kSiteEpilogue = 0xB0C4,
  kSiteSplitK = 0xB0C5,
};

struct TcParams {
  int Cin, H, W, Ho, Wo, Cout, kW, T;
  int sh, sw, ph, pw, dh, dw;
  int tap_dy[kMaxTaps], tap_dx[kMaxTaps];   // ki * dh - ph, kj * dw - pw of tap t
  int M, Cin_pad, n_cc, n_k, n_tiles_n;
  int mask_is_logit, has_bias, act_relu;
  int xs0, xs2, xs3;        // input strides (channel stride is 1)
  int64_t os[4], ms[4], ys[4];
  unsigned long long wait_limit_ns;  // pipeline barrier waits (bevk_set_wait_limit_ns)
  // K split (kModePairN2): clusters [tile][k_split] each run stages
  // [k_part * k_len, ...) of the tile; the two halves of a tile exchange half
  // of their fp32 accumulators through `part` (per (tile, rank, half):
  // [kSplitCols / 4][kBM][4] floats) and meet on `tickets` (two words per
  // (tile, rank): arrival, release).
  int k_split, k_len;
  float *part;
  unsigned long long *tickets;
};

// Tile schedules of the fused kernel.
enum : int {
  kModeSingle = 0,  // one CTA per 128-pixel x BN tile, M=128 MMA
  kModePair = 1,    // 2-CTA cluster per 256-pixel x BN tile, M=256 cta_group::2 MMA
  kModeNSplit = 2,  // 2-CTA cluster per 128-pixel x 2*BN tile, A rows shared
  kModePairN2 = 3,  // 2-CTA cluster per 256-pixel x 2*BN tile: two M=256 accumulators
};

// Warp roles.  A warp issues on SM sub-partition (warp index mod 4).
// Isolated layout (21 warps): the TMA warp (7) and the MMA warp (3) have
// sub-partition 3 to themselves (with idle warps 11, 15, 19) and the 16
// gather warps fill sub-partitions 0-2.  A gather warp that shares a
// sub-partition with the thread issuing tcgen05.mma (which blocks while the
// tensor pipe is busy) or the TMA copies falls most of a stage behind the
// others, and the slowest gather warp sets the pace of the pipeline.  The
// price is the register budget: six warps on a sub-partition leave 80
// registers a thread.  Compact layout (18 warps, 96 registers): gather warps
// 0-15, TMA warp 16, MMA warp 17.
template <bool ISO>
struct Roles;
template <>
struct Roles<true> {
  static constexpr int kWarps = 21, kMma = 3, kTma = 7;
  __device__ static bool gather(int w) { return (w & 3) != 3; }
  __device__ static int gather_index(int w) { return w - ((w + 1) >> 2); }
};
template <>
struct Roles<false> {
  static constexpr int kWarps = kGatherWarps + 2, kMma = kGatherWarps + 1, kTma = kGatherWarps;
  __device__ static bool gather(int w) { return w < kGatherWarps; }
  __device__ static int gather_index(int w) { return w; }
};
// Measured on B200 (cfg2 N-split 53.1 -> 56.2 us, cfg3 pair 82.9 -> 130 us):
// the gather warps are issue-bound, so giving up a sub-partition costs more
// than the lag it removes, and every schedule uses the compact layout.  The
// isolated one is kept for experiments (BEVK_DCN_ISO_ROLES).
__host__ __device__ constexpr bool iso_roles(int mode) {
#ifdef BEVK_DCN_ISO_ROLES
  return mode >= 0;
#else
  return mode < 0;
#endif
}
template <int MODE>
__host__ __device__ constexpr int tc_threads() {
  return Roles<iso_roles(MODE)>::kWarps * 32;
}
// Gather warps that build one A stage: one row a thread, at most all of them
// (VB = bytes a lane loads per corner; N-split CTAs gather 64 rows a stage).
template <int MODE, int VB>
__host__ __device__ constexpr int warps_per_stage() {
  return ((MODE == kModeNSplit ? kBM / 2 : kBM) * 4 / VB) < kGatherWarps
             ? (MODE == kModeNSplit ? kBM / 2 : kBM) * 4 / VB
             : kGatherWarps;
}

template <int BN, int STAGES, bool PAIR, int NH = 1>
struct Smem {
  // In a CTA pair each CTA holds half of the B tile (BN/2 output channels) of
  // each of the NH accumulators.
  static constexpr int kBRows = PAIR ? NH * BN / 2 : BN;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = kBRows * kBK * 2;
  static constexpr int kA = 0;
  static constexpr int kB = kA + STAGES * kABytes;
  static constexpr int kGW = kB + STAGES * kBBytes;          // 4 16-bit weights [T][BM]
  static constexpr int kGB = kGW + kMaxTaps * kBM * 8;       // packed base + mask [T][BM]
  static constexpr int kBar = kGB + kMaxTaps * kBM * 4;      // full[S], empty[S], tmem_full
  static constexpr int kMisc = kBar + (2 * STAGES + 1) * 8;  // tmem slot, abort flag
  static constexpr int kTotal = kMisc + 16;
  static constexpr int kAlloc = kTotal + 1024;               // 1024-byte alignment slack
};

template <typename T>
struct GatherMath;

// Corner weights are kept in shared memory as four 16-bit values of the
// problem's type (uint2: corners 0,1 in .x, corners 2,3 in .y); prep() turns
// them into the operand form of lerp2().

// fp16: weights as half2 (w, w); packed half2 FMA chain.
template <>
struct GatherMath<__half> {
  static constexpr uint32_t kFmt = 0;
  __device__ static uint4 prep(uint2 wh) {
    return make_uint4(__byte_perm(wh.x, 0u, 0x1010), __byte_perm(wh.x, 0u, 0x3232),
                      __byte_perm(wh.y, 0u, 0x1010), __byte_perm(wh.y, 0u, 0x3232));
  }
  __device__ static uint32_t lerp2(uint4 w, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    const __half2 r0 = __hmul2(*reinterpret_cast<const __half2 *>(&w.x),
                               *reinterpret_cast<const __half2 *>(&a));
    const __half2 r1 = __hfma2(*reinterpret_cast<const __half2 *>(&w.y),
                               *reinterpret_cast<const __half2 *>(&b), r0);
    const __half2 r2 = __hfma2(*reinterpret_cast<const __half2 *>(&w.z),
                               *reinterpret_cast<const __half2 *>(&c), r1);
    __half2 r3 = __hfma2(*reinterpret_cast<const __half2 *>(&w.w),
                         *reinterpret_cast<const __half2 *>(&d), r2);
    return *reinterpret_cast<uint32_t *>(&r3);
  }
  __device__ static uint16_t store_bits(float v) {
    __half h = __float2half_rn(v);
    return *reinterpret_cast<uint16_t *>(&h);
  }
  // (lo, hi) rounded to the output type, lo in the low half
  __device__ static uint32_t pack2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
  }
  __device__ static float from_bits(uint16_t v) { return __half2float(__ushort_as_half(v)); }
};

// bf16: weights as bf16x2 (w, w); packed bf16x2 FMA chain, each step
// rounded to bf16 (as the fp16 path rounds each step to fp16).  On the cfg3
// data this moves the output 3.1e-3 relative L2 from the fp32 oracle, against
// 1.7e-3 for fp32 interpolation rounded once; the tolerance is 5e-3.  It takes
// the per-pair unpacking and fp32 arithmetic off the issue-bound gather warps.
template <>
struct GatherMath<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
  __device__ static uint4 prep(uint2 wh) {
    return make_uint4(__byte_perm(wh.x, 0u, 0x1010), __byte_perm(wh.x, 0u, 0x3232),
                      __byte_perm(wh.y, 0u, 0x1010), __byte_perm(wh.y, 0u, 0x3232));
  }
  __device__ static uint32_t lerp2(uint4 w, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    using B2 = __nv_bfloat162;
    const B2 r0 = __hmul2(*reinterpret_cast<const B2 *>(&w.x), *reinterpret_cast<const B2 *>(&a));
    const B2 r1 = __hfma2(*reinterpret_cast<const B2 *>(&w.y), *reinterpret_cast<const B2 *>(&b), r0);
    const B2 r2 = __hfma2(*reinterpret_cast<const B2 *>(&w.z), *reinterpret_cast<const B2 *>(&c), r1);
    B2 r3 = __hfma2(*reinterpret_cast<const B2 *>(&w.w), *reinterpret_cast<const B2 *>(&d), r2);
    return *reinterpret_cast<uint32_t *>(&r3);
  }
  __device__ static uint16_t store_bits(float v) {
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    return *reinterpret_cast<uint16_t *>(&h);
  }
  __device__ static uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
  }
  __device__ static float from_bits(uint16_t v) {
    return __uint_as_float(static_cast<uint32_t>(v) << 16);
  }
};

template <typename T>
__device__ __forceinline__ float ld_float(const T *p);
template <>
__device__ __forceinline__ float ld_float<__half>(const __half *p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ld_float<__nv_bfloat16>(const __nv_bfloat16 *p) {
  return __bfloat162float(*p);
}

// Geometry of output pixel m = (b, oh, ow) at tap t: `packed` = 2 * (element
// offset of corner (h_low, w_low)) | (in-range bits of corners 0..3) -- the
// offset is a multiple of 8 elements, so the low four bits are free and the
// offset comes back as (packed >> 1) & ~7 -- and `wh` = the four corner
// weights (mask folded in, 0 for dropped corners) as 16-bit values of type T.
// (dy, dx, mk) are the pixel's offsets and mask at tap t.
template <typename T>
__device__ __forceinline__ void tap_geometry(const TcParams &p, int b, int oh, int ow, int t,
                                             float dy, float dx, float mk, int &packed,
                                             uint2 &wh) {
  packed = 0;
  wh = make_uint2(0u, 0u);
  if (p.mask_is_logit) mk = 1.f / (1.f + __expf(-mk));
  const float h_im = static_cast<float>(oh * p.sh + p.tap_dy[t]) + dy;
  const float w_im = static_cast<float>(ow * p.sw + p.tap_dx[t]) + dx;
  if (!(h_im > -1.f && w_im > -1.f && h_im < static_cast<float>(p.H) &&
        w_im < static_cast<float>(p.W)))
    return;
  const int h_low = static_cast<int>(floorf(h_im));
  const int w_low = static_cast<int>(floorf(w_im));
  const float lh = h_im - static_cast<float>(h_low), lw = w_im - static_cast<float>(w_low);
  const float hh = 1.f - lh, hw = 1.f - lw;
  const bool y0 = h_low >= 0, y1 = h_low + 1 <= p.H - 1;
  const bool x0 = w_low >= 0, x1 = w_low + 1 <= p.W - 1;
  const int base = b * p.xs0 + h_low * p.xs2 + w_low * p.xs3;
  const int mask = (y0 && x0 ? 1 : 0) | (y0 && x1 ? 2 : 0) | (y1 && x0 ? 4 : 0) |
                   (y1 && x1 ? 8 : 0);
  packed = (base * 2) | mask;
  using GM = GatherMath<T>;
  const uint32_t w0 = (y0 && x0) ? GM::store_bits(hh * hw * mk) : 0u;
  const uint32_t w1 = (y0 && x1) ? GM::store_bits(hh * lw * mk) : 0u;
  const uint32_t w2 = (y1 && x0) ? GM::store_bits(lh * hw * mk) : 0u;
  const uint32_t w3 = (y1 && x1) ? GM::store_bits(lh * lw * mk) : 0u;
  wh = make_uint2(w0 | (w1 << 16), w2 | (w3 << 16));
}

// Kernel body.
// kModeSingle: one CTA per 128-pixel x BN tile, M=128 MMA.
// kModePair: a 2-CTA cluster per 256-pixel x BN tile; each CTA gathers its own
//   128 pixels and TMA-loads half of the weight tile, the leader (rank 0)
//   issues M=256 tcgen05.mma.cta_group::2 reading both CTAs' operands, and
//   each MMA commit releases the stage in both CTAs.  Both CTAs' gather warps
//   and TMA copies report to the leader's barriers.
// kModeNSplit: a 2-CTA cluster per 128-pixel x 2*BN tile; CTA c computes
//   output channels [c*BN, c*BN+BN) of the same 128 pixels with its own M=128
//   MMA.  Each CTA gathers only rows [c*64, c*64+64) of the A stage and a bulk
//   copy puts them into the other CTA's A stage too, so every pixel is
//   interpolated once for all 2*BN channels.  Each MMA commit is multicast to
//   both CTAs' empty barriers: a stage is refilled only when both are done.
template <typename T, int BN, int STAGES, int MODE, int VB>
__device__ __forceinline__ void dcn_fwd_tc_body(const CUtensorMap &tmap_w, const TcParams &p,
                                                const T *__restrict__ x,
                                                const T *__restrict__ off,
                                                const T *__restrict__ msk,
                                                const T *__restrict__ bias, T *__restrict__ y) {
  constexpr bool N2 = MODE == kModePairN2;
  constexpr bool PAIR = MODE == kModePair || N2;
  constexpr bool NSPLIT = MODE == kModeNSplit;
  constexpr int NH = N2 ? 2 : 1;        // accumulators (N halves) per tile
  constexpr int NCOLS = NH * BN;        // output channels per tile and TMEM columns
  constexpr bool CLUSTER = MODE != kModeSingle;
  constexpr int kGRows = NSPLIT ? kBM / 2 : kBM;   // A rows this CTA gathers per stage
  constexpr uint32_t kGBytes = kGRows * 128;       // their bytes in an A stage (copied
                                                   // to the other CTA under NSPLIT)
  using L = Smem<BN, STAGES, PAIR, NH>;
  using GM = GatherMath<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const uint32_t sA = sbase + L::kA, sB = sbase + L::kB;
  uint2 *s_gw = reinterpret_cast<uint2 *>(smem + L::kGW);
  int *s_gb = reinterpret_cast<int *>(smem + L::kGB);
  // full: one barrier per stage for everything the MMA reads -- an arrive
  // per gather warp (of both CTAs when paired) plus the TMA thread's
  // arrive.expect_tx, whose byte count covers the weight tile (NSPLIT: and
  // the other CTA's copied A rows).  The MMA thread waits on a single
  // barrier per stage: each wait it makes is a bubble in the tensor pipe.
  const uint32_t bar_full = sbase + L::kBar;
  const uint32_t bar_empty = bar_full + STAGES * 8;     // stage consumed (tcgen05.commit)
  const uint32_t bar_tmem = bar_empty + STAGES * 8;
  uint32_t *s_tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kMisc);
  volatile int *s_abort = reinterpret_cast<volatile int *>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  using R = Roles<iso_roles(MODE)>;
  const bool gather_warp = R::gather(warp);
  const int gw = R::gather_index(warp);      // gather warp index 0..15
  const uint32_t cr = CLUSTER ? ptx::cluster_ctarank() : 0u;   // rank in the CTA pair
  const bool leader = cr == 0;
  const int cl = CLUSTER ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  // K split: the clusters of one tile are adjacent, so they start together
  const int k_part = N2 ? cl % p.k_split : 0;
  const int tile = N2 ? cl / p.k_split : cl;
  const int k_begin = N2 ? k_part * p.k_len : 0;             // first stage of this cluster
  const int n_loc = N2 ? min(p.n_k - k_begin, p.k_len) : p.n_k;   // its stages (>= 1)
  const int n_tile = tile % p.n_tiles_n;
  const int m_tile = tile / p.n_tiles_n;
  // K order: stage kit covers tap kit % T of channel chunk kit / T.  Taps vary
  // fastest, so the corner lines of one channel chunk are re-read from L1
  // across consecutive stages.  (Starting each tile at a different K offset
  // spreads the weight-tile reads over L2 but measured slower on B200.)
  const int m0 = PAIR ? m_tile * 2 * kBM + static_cast<int>(cr) * kBM : m_tile * kBM;
  const int n0 = NSPLIT ? n_tile * 2 * BN + static_cast<int>(cr) * BN : n_tile * NCOLS;
  const int g_row0 = NSPLIT ? static_cast<int>(cr) * kGRows : 0;  // first tile row gathered here

  // The prologue below (barriers, TMEM, descriptor prefetch) touches no
  // global memory, so under a programmatic launch it overlaps the previous
  // kernel's tail; the next kernel may be placed as soon as SMs free up.
  ptx::grid_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // gather warps (of both CTAs when paired) + the TMA arrive with bytes
      ptx::mbar_init(bar_full + 8 * s, (PAIR ? 2 : 1) * warps_per_stage<MODE, VB>() + 1);
      ptx::mbar_init(bar_empty + 8 * s, NSPLIT ? 2 : 1);   // tcgen05.commit (of both CTAs)
    }
    ptx::mbar_init(bar_tmem, 1);
    *s_abort = 0;
    ptx::fence_mbar_init();
  }
  // Clustered CTAs: every barrier of both CTAs is initialised before any
  // cross-CTA arrive or copy can target it.
  if constexpr (CLUSTER) ptx::cluster_sync();
  if (warp == R::kMma) {
    if constexpr (PAIR) {
      ptx::tmem_alloc_pair(ptx::smem_u32(s_tmem_slot), NCOLS);
      ptx::tmem_relinquish_pair();
    } else {
      ptx::tmem_alloc(ptx::smem_u32(s_tmem_slot), BN);
      ptx::tmem_relinquish();
    }
  }
  if (warp == R::kTma && lane == 0) ptx::tma_prefetch_desc(&tmap_w);
  // every global read (input, offsets, mask, weights, bias) and write comes after
  ptx::grid_wait_prerequisites();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *s_tmem_slot;
  // Barriers the gather warps and TMA copies report to: the leader's.
  const uint32_t full_dst = PAIR ? ptx::mapa_shared(bar_full, 0) : bar_full;
  auto wait = [&](uint32_t bar, uint32_t parity, unsigned int site) -> bool {
    return ptx::mbar_wait_bounded(bar, parity, s_abort, &g_bevk_watchdog, site,
                                  p.wait_limit_ns);
  };

  bool ok = true;
  if (gather_warp) {
    // ---------------------------------------------------------- geometry
    // Entry e = t * kGRows + r for every tap t and tile row r.  A thread owns
    // one row (its pixel decoded once) and every kPerRow-th tap of it; the
    // lanes of a warp take consecutive rows, so each offset / mask load of a
    // warp is one contiguous run.  All of a thread's loads are issued before
    // any entry is computed.
    {
      constexpr int kPerRow = kGatherWarps * 32 / kGRows;
      constexpr int kMaxPer = (kMaxTaps + kPerRow - 1) / kPerRow;
      const int j = gw * 32 + lane;
      const int r = j % kGRows, t0 = j / kGRows;
      const int m = m0 + g_row0 + r;
      int b = 0, oh = 0, ow = 0;
      if (m < p.M) {
        const int HoWo = p.Ho * p.Wo;
        b = m / HoWo;
        const int rem = m - b * HoWo;
        oh = rem / p.Wo;
        ow = rem - oh * p.Wo;
      }
      // (entries past the last tap or pixel load element 0 and are dropped)
      const T *ob = off + b * p.os[0] + oh * p.os[2] + ow * p.os[3];
      const T *mb = msk + b * p.ms[0] + oh * p.ms[2] + ow * p.ms[3];
      uint16_t dy[kMaxPer], dx[kMaxPer], mk[kMaxPer];
#pragma unroll
      for (int i = 0; i < kMaxPer; ++i) {
        const int t = t0 + i * kPerRow < p.T ? t0 + i * kPerRow : 0;
        dy[i] = ptx::ld_global_nc_u16(ob + (2 * t) * p.os[1]);
        dx[i] = ptx::ld_global_nc_u16(ob + (2 * t + 1) * p.os[1]);
        mk[i] = ptx::ld_global_nc_u16(mb + t * p.ms[1]);
      }
#pragma unroll
      for (int i = 0; i < kMaxPer; ++i) {
        const int t = t0 + i * kPerRow;
        if (t < p.T) {
          int packed = 0;
          uint2 wh = make_uint2(0u, 0u);
          if (m < p.M)
            tap_geometry<T>(p, b, oh, ow, t, GM::from_bits(dy[i]), GM::from_bits(dx[i]),
                            GM::from_bits(mk[i]), packed, wh);
          s_gb[t * kGRows + r] = packed;
          s_gw[t * kGRows + r] = wh;
        }
      }
    }
    ptx::named_barrier_sync(1, kGatherWarps * 32);

    // ---------------------------------------------------------- gather
    // Each lane owns one VB-byte vector (VB/2 channels) of a 128-byte tile
    // row: kLanesPerRow lanes cover a row and one warp instruction covers
    // kRowsPerInstr rows.  kWarpsPerStage warps build a stage (each thread
    // owning kRowsPerThr rows of it); when that is fewer than the gather
    // warps, the warps form kGroups groups that take stages in turn (group g:
    // stages g, g + kGroups, ...).  The gather warps are issue-bound, so
    // 32-byte vectors -- half the address and predicate work per byte --
    // are worth the grouping.  The four corner loads of all its rows for a
    // warp's next stage are issued (into registers) before its current stage
    // is interpolated and stored, so a stage of corner reads is always in
    // flight per thread.  Stage coordinates advance incrementally (no
    // integer division in the loop).
    constexpr int kLanesPerRow = 128 / VB;
    constexpr int kRowsPerInstr = 32 / kLanesPerRow;
    constexpr int kWarpsPerStage = warps_per_stage<MODE, VB>();
    constexpr int kGroups = kGatherWarps / kWarpsPerStage;
    constexpr int kRowStride = kWarpsPerStage * kRowsPerInstr;  // between a thread's rows
    constexpr int kRowsPerThr = kGRows / kRowStride;
    // A gather warp waits for its stage's slot with a parity wait, which
    // tells two adjacent phases of the slot's barrier apart and no more: a
    // group's next stage may be at most STAGES stages ahead of its last one.
    static_assert(kRowsPerThr >= 1 && kGRows % kRowStride == 0 &&
                      kGroups * kWarpsPerStage == kGatherWarps && kGroups <= STAGES,
                  "gather lane layout");
    constexpr int kWords = VB / 4;
    using Vec = ptx::Words<kWords>;
    const int grp = gw / kWarpsPerStage;        // stage group of this warp
    const int gi = gw - grp * kWarpsPerStage;   // warp index within the group
    const int j = lane % kLanesPerRow;
    const int row0 = gi * kRowsPerInstr + lane / kLanesPerRow;
    const int xs2 = p.xs2, xs3 = p.xs3;
    const T *zline = reinterpret_cast<const T *>(g_dcn_zero_line) + j * (VB / 2);
    // NSPLIT: the other CTA's A stages and full barriers
    const uint32_t peer_sA = NSPLIT ? ptx::mapa_shared(sA, cr ^ 1u) : 0u;
    const uint32_t peer_full = NSPLIT ? ptx::mapa_shared(bar_full, cr ^ 1u) : 0u;
    struct Prefetch {
      Vec v[kRowsPerThr][4];
      int ebase;  // geometry index of the prefetched stage's first row
    };
    // (tap, channel chunk) of a stage index, advanced one stage at a time
    struct StageCoord {
      int t, cc;
    };
    auto next_coord = [&](StageCoord c) {
#pragma unroll
      for (int g = 0; g < kGroups; ++g)
        if (++c.t == p.T) {
          c.t = 0;
          ++c.cc;
        }
      return c;
    };
    auto issue = [&](StageCoord sc, Prefetch &P) {
      const int c = sc.cc * kBK + j * (VB / 2);
      const int cvalid = c < p.Cin ? 0xF : 0;
      const int ebase = sc.t * kGRows + row0;
      P.ebase = ebase;
#pragma unroll
      for (int i = 0; i < kRowsPerThr; ++i) {
        const int pk = s_gb[ebase + i * kRowStride];
        const int mk = pk & cvalid;
        const T *p0 = x + (((pk >> 1) & ~7) + c);
        if constexpr (VB == 16) {
          // 16-byte vectors: predicated loads (zeros when off)
          P.v[i][0] = ptx::ld_global_nc_words4_pred(p0, mk & 1);
          P.v[i][1] = ptx::ld_global_nc_words4_pred(p0 + xs3, mk & 2);
          P.v[i][2] = ptx::ld_global_nc_words4_pred(p0 + xs2, mk & 4);
          P.v[i][3] = ptx::ld_global_nc_words4_pred(p0 + (xs2 + xs3), mk & 8);
        } else {
          P.v[i][0] = ptx::ld_global_nc_words<kWords>((mk & 1) ? p0 : zline);
          P.v[i][1] = ptx::ld_global_nc_words<kWords>((mk & 2) ? p0 + xs3 : zline);
          P.v[i][2] = ptx::ld_global_nc_words<kWords>((mk & 4) ? p0 + xs2 : zline);
          P.v[i][3] = ptx::ld_global_nc_words<kWords>((mk & 8) ? p0 + (xs2 + xs3) : zline);
        }
      }
    };
    int cs = grp;        // stage slot of the stage being consumed (grp < STAGES)
    uint32_t cph = 0;    // its phase
    auto consume = [&](Prefetch &P) -> bool {
      // keep this stage's arithmetic behind the next stage's corner loads
#pragma unroll
      for (int i = 0; i < kRowsPerThr; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) ptx::reg_fence(P.v[i][q]);
      if (!wait(bar_empty + 8 * cs, cph ^ 1, kSiteGatherEmpty)) return false;
      const uint32_t a_stage = sA + cs * L::kABytes;
#pragma unroll
      for (int i = 0; i < kRowsPerThr; ++i) {
        const int r = g_row0 + row0 + i * kRowStride;  // row of the A tile
        const uint4 wq = GM::prep(s_gw[P.ebase + i * kRowStride]);
        uint32_t res[kWords];
#pragma unroll
        for (int w = 0; w < kWords; ++w)
          res[w] = GM::lerp2(wq, P.v[i][0].w[w], P.v[i][1].w[w], P.v[i][2].w[w], P.v[i][3].w[w]);
        // 16-byte chunks j*VB/16 .. of row r, at their 128-byte-swizzle slots
#pragma unroll
        for (int h = 0; h < VB / 16; ++h) {
          const int chunk = j * (VB / 16) + h;
          ptx::st_shared_v4(a_stage + r * 128 + ((chunk ^ (r & 7)) << 4),
                            make_uint4(res[4 * h], res[4 * h + 1], res[4 * h + 2], res[4 * h + 3]));
        }
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if constexpr (NSPLIT) {
          // This warp's rows (contiguous in the stage) also go to the other
          // CTA's A stage, which is free: the empty barrier counts its MMA.
#pragma unroll
          for (int i = 0; i < kRowsPerThr; ++i) {
            const uint32_t off_a = static_cast<uint32_t>(
                (g_row0 + gi * kRowsPerInstr + i * kRowStride) * 128);
            ptx::bulk_copy_smem_to_cluster(peer_sA + cs * L::kABytes + off_a,
                                           a_stage + off_a, kRowsPerInstr * 128,
                                           peer_full + 8 * cs);
          }
        }
        if constexpr (PAIR) ptx::mbar_arrive_cluster(full_dst + 8 * cs);
        else ptx::mbar_arrive(bar_full + 8 * cs);
      }
      cs += kGroups;
      if (cs >= STAGES) { cs -= STAGES; cph ^= 1; }
      return true;
    };
    {
      Prefetch A, B;
      StageCoord sc{0, 0};
      if constexpr (N2) sc = StageCoord{k_begin % p.T, k_begin / p.T};
      for (int g = 0; g < grp; ++g)
        if (++sc.t == p.T) { sc.t = 0; ++sc.cc; }
      if (grp < n_loc) issue(sc, A);
      for (int kit = grp; kit < n_loc; kit += 2 * kGroups) {
        sc = next_coord(sc);
        if (kit + kGroups < n_loc) issue(sc, B);
        ok = consume(A);
        if (!ok || kit + kGroups >= n_loc) break;
        sc = next_coord(sc);
        if (kit + 2 * kGroups < n_loc) issue(sc, A);
        ok = consume(B);
        if (!ok) break;
      }
    }
  } else if (warp == R::kTma) {
    if (lane == 0) {
      int issued = 0;
      for (int kit = 0; kit < n_loc; ++kit) {
        const int s = kit % STAGES;
        const uint32_t ph = (kit / STAGES) & 1;
        if (!wait(bar_empty + 8 * s, ph ^ 1, kSiteTmaEmpty)) break;
        const int t = (N2 ? k_begin + kit : kit) % p.T;
        const int cc = (N2 ? k_begin + kit : kit) / p.T;
        if constexpr (PAIR) {
          // the leader expects both CTAs' halves on its own barrier
          if (leader) ptx::mbar_arrive_expect_tx(bar_full + 8 * s, 2 * L::kBBytes);
#pragma unroll
          for (int h = 0; h < NH; ++h)
            ptx::tma_load_2d_pair(sB + s * L::kBBytes + h * (BN / 2) * 128, &tmap_w,
                                  full_dst + 8 * s, t * p.Cin_pad + cc * kBK,
                                  n0 + h * BN + static_cast<int>(cr) * (BN / 2));
        } else {
          // NSPLIT: the other CTA's A rows land on the same barrier
          ptx::mbar_arrive_expect_tx(bar_full + 8 * s, L::kBBytes + (NSPLIT ? kGBytes : 0u));
          ptx::tma_load_2d(sB + s * L::kBBytes, &tmap_w, bar_full + 8 * s,
                           t * p.Cin_pad + cc * kBK, n0);
        }
        issued = kit + 1;
      }
      if (*s_abort && (issued > 0 || CLUSTER)) {
        // The copies issued here (and, clustered, the ones reporting to the
        // other CTA, and the gather warps' copies of A rows to the other CTA)
        // share their barriers with arrivals that an abort may have skipped,
        // so no barrier phase is left to wait on: give them time to land
        // before shared memory can be released.
        for (int i = 0; i < 64; ++i) __nanosleep(2000);
      }
    }
  } else if (warp == R::kMma) {  // (the leader's, when paired)
    if (lane == 0 && (leader || !PAIR)) {
      constexpr uint32_t idesc = ptx::umma_idesc_f16(GM::kFmt, PAIR ? 2 * kBM : kBM, BN);
      for (int kit = 0; kit < n_loc; ++kit) {
        const int s = kit % STAGES;
        if (!wait(bar_full + 8 * s, (kit / STAGES) & 1, kSiteMmaFull)) break;
        ptx::tc_fence_after();
        const uint32_t a_stage = sA + s * L::kABytes;
        const uint32_t b_stage = sB + s * L::kBBytes;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t ad = ptx::umma_desc_sw128(a_stage + k * 32);
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            // accumulator h: TMEM columns [h*BN, h*BN + BN), B half-tile h
            const uint64_t bd = ptx::umma_desc_sw128(b_stage + h * (BN / 2) * 128 + k * 32);
            if constexpr (PAIR)
              ptx::umma_f16_ss_pair(tmem_base + h * BN, ad, bd, idesc, (kit | k) != 0 ? 1u : 0u);
            else ptx::umma_f16_ss(tmem_base, ad, bd, idesc, (kit | k) != 0 ? 1u : 0u);
          }
        }
        if constexpr (PAIR) ptx::umma_commit_pair_both(bar_empty + 8 * s, 0x3);
        else if constexpr (NSPLIT) ptx::umma_commit_multicast(bar_empty + 8 * s, 0x3);
        else ptx::umma_commit(bar_empty + 8 * s);
      }
      // Tracks completion of every MMA issued above (also on abort, so the
      // accumulator is quiescent before TMEM is released).
      if constexpr (PAIR) ptx::umma_commit_pair_both(bar_tmem, 0x3);
      else ptx::umma_commit(bar_tmem);
      if (*s_abort) {
        volatile int dummy = 0;
        ptx::mbar_wait_bounded(bar_tmem, 0, &dummy, &g_bevk_watchdog, kSiteEpilogue);
      }
    }
    __syncwarp();
  }

  // ------------------------------------------------------------ epilogue
  // Warps 0-15 (gather, TMA, MMA and idle warps alike) drain TMEM: warp w
  // reads lane quadrant w % 4, in windows of kColsPerWarp columns: window
  // w / 4 of the tile's columns, or under kModePairN2 window w / 4 of each
  // 256-column half (of the half this cluster finishes, when K is split).
  __syncwarp();
  if (warp < kEpilogueWarps) {
    if (ok) ok = wait(bar_tmem, 0, kSiteEpilogue);
    constexpr int kColsPerWarp = N2 ? kSplitCols / 4 : NCOLS / 4;
    constexpr int kChunk = kColsPerWarp < 32 ? kColsPerWarp : 32;
    const int q = warp & 3;                        // TMEM lane quadrant of this warp
    const int cgrp = warp >> 2;                    // its window in each column block
    const int row = q * 32 + lane;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    int n_win = 1;
    int win0 = cgrp * kColsPerWarp;
    const float4 *partner = nullptr;               // K split: the other half's columns
    if constexpr (N2) {
      n_win = NCOLS / kSplitCols;
      if (p.k_split > 1) {
        // The cluster running K part k finishes columns [k*256, k*256+256) of
        // the tile and hands the other 256 columns of its accumulator to the
        // partner cluster: write them (fp32, [column/4][row][4], so a warp
        // store covers 512 contiguous bytes), then meet the partner CTA on
        // the (tile, rank) ticket.  Both clusters of a tile are resident at
        // once (the host splits K only when all clusters fit on the GPU
        // together), so the wait ends; it is bounded all the same.
        const size_t slot = static_cast<size_t>(tile * 2 + static_cast<int>(cr)) * 2;
        volatile int *s_met = reinterpret_cast<volatile int *>(smem + L::kMisc + 8);
        if (ok) {
          ptx::tc_fence_after();
          const int give = (1 - k_part) * kSplitCols;
          float4 *mine = reinterpret_cast<float4 *>(p.part) +
                         (slot + k_part) * (kSplitCols / 4) * kBM + row;
#pragma unroll 1
          for (int cb = 0; cb < kColsPerWarp; cb += 32) {
            const int c = cgrp * kColsPerWarp + cb;  // column within the handed-over half
            uint32_t r[32];
            ptx::tmem_ld_32x32b<32>(t_row + give + c, r);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int g = 0; g < 8; ++g)
              __stcg(mine + ((c >> 2) + g) * kBM,
                     make_float4(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]),
                                 __uint_as_float(r[4 * g + 2]), __uint_as_float(r[4 * g + 3])));
          }
          __threadfence();
        }
        ptx::named_barrier_sync(2, kEpilogueWarps * 32);
        if (threadIdx.x == 0) {
          // Rendezvous without a reset pass: both CTAs swap this launch's tag
          // into the arrival word.  The one that gets the tag back arrives
          // second (the other's partial sums are written) and releases the
          // other through the second word; the first clears both words once
          // released.  Words left by another launch or by unrelated data
          // hold other values, so the workspace needs no initialisation; a
          // replayed graph node keeps its grid id, and finds the words
          // cleared by its previous run (a wait that gives up clears its
          // arrival too).
          int met = 0;
          if (!*s_abort) {
            unsigned long long *arrive = p.tickets + slot;        // (tile, rank): 2 words
            unsigned long long *release = arrive + 1;
            unsigned long long tag = (ptx::grid_id() + 1) * 0x9E3779B97F4A7C15ull;
            tag = tag ? tag : 1ull;
            if (ptx::atom_exch_acq_rel_gpu(arrive, tag) == tag) {
              ptx::st_release_gpu(release, tag);
              met = 1;
            } else {
              const uint64_t t0 = ptx::globaltimer_ns();
              for (uint32_t it = 0;; ++it) {
                if (ptx::ld_acquire_gpu(release) == tag) {
                  *release = 0ull;
                  *arrive = 0ull;
                  met = 1;
                  break;
                }
                __nanosleep(64);
                if ((it & 7u) == 7u && ptx::globaltimer_ns() - t0 > p.wait_limit_ns) {
                  ptx::atom_exch_acq_rel_gpu(arrive, 0ull);
                  atomicCAS(&g_bevk_watchdog, 0u, static_cast<unsigned int>(kSiteSplitK));
                  *s_abort = 1;
                  break;
                }
              }
            }
          }
          *s_met = met;
        }
        ptx::named_barrier_sync(2, kEpilogueWarps * 32);
        if (!*s_met) ok = false;
        __threadfence();
        partner = reinterpret_cast<const float4 *>(p.part) +
                  (slot + 1 - k_part) * (kSplitCols / 4) * kBM + row;
        n_win = 1;
        win0 = k_part * kSplitCols + cgrp * kColsPerWarp;
        if (ok) {
          // all of this lane's partner sums in flight at once, into L1
          const float4 *pp = partner + (cgrp * kColsPerWarp >> 2) * kBM;
#pragma unroll
          for (int g = 0; g < kColsPerWarp / 4; ++g) ptx::prefetch_l1(pp + g * kBM);
        }
      }
    }
    if (ok) {
      ptx::tc_fence_after();
      const int m = m0 + row;
      const int HoWo = p.Ho * p.Wo;
      const int b = m / HoWo, rem = m - (m / HoWo) * HoWo;
      const int oh = rem / p.Wo, ow = rem - (rem / p.Wo) * p.Wo;
      T *yrow = y + b * p.ys[0] + oh * p.ys[2] + ow * p.ys[3];
      const bool vec_out = p.ys[1] == 1 && (p.Cout & 7) == 0 &&
                           (reinterpret_cast<uintptr_t>(y) & 15) == 0 && (p.ys[0] & 7) == 0 &&
                           (p.ys[2] & 7) == 0 && (p.ys[3] & 7) == 0;
      // accumulator columns [col, col + kChunk) of this lane's row (plus the
      // partner half's partial sums under a K split)
      auto add_partner = [&](int col, uint32_t(&r)[kChunk]) {
        if (N2 && partner != nullptr) {
          const float4 *pp = partner + ((col - k_part * kSplitCols) >> 2) * kBM;
          // four loads (16 registers) in flight at a time: the accumulator
          // chunks already hold 64
#pragma unroll
          for (int g0 = 0; g0 < kChunk / 4; g0 += 4) {
            float4 v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = __ldca(pp + (g0 + i) * kBM);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int g = g0 + i;
              r[4 * g] = __float_as_uint(__uint_as_float(r[4 * g]) + v[i].x);
              r[4 * g + 1] = __float_as_uint(__uint_as_float(r[4 * g + 1]) + v[i].y);
              r[4 * g + 2] = __float_as_uint(__uint_as_float(r[4 * g + 2]) + v[i].z);
              r[4 * g + 3] = __float_as_uint(__uint_as_float(r[4 * g + 3]) + v[i].w);
            }
            asm volatile("" ::: "memory");
          }
        }
      };
      auto acc = [&](int col, uint32_t(&r)[kChunk]) {
        ptx::tmem_ld_32x32b<kChunk>(t_row + col, r);
        ptx::tmem_wait_ld();
        add_partner(col, r);
      };
#pragma unroll 1
      for (int wi = 0; wi < (N2 ? n_win : 1); ++wi) {
        const int c0 = win0 + wi * kSplitCols;   // first tile column of the window
        // A lane holds its own pixel's channels, so direct 16-byte stores put
        // 32 pixels (32 lines) in every warp store.  When the window is in
        // bounds and the output is channel-contiguous, the warp's 32 x
        // kColsPerWarp block is staged in shared memory and written back row
        // by row, kColsPerWarp * 2 contiguous bytes per row.
        if (vec_out && n0 + c0 + kColsPerWarp <= p.Cout) {
          constexpr int kCh = kColsPerWarp / 8;          // 16-byte chunks a row
          // Staged in the weight ring: only this CTA's TMA writes it and the
          // MMAs (also the partner's, in a pair) have finished reading it.  The
          // A ring is not free yet under N-split: bulk copies to the other CTA
          // may still be reading it.
          static_assert(kEpilogueWarps * 32 * kCh * 16 <= STAGES * L::kBBytes, "staging space");
          const uint32_t blk = sB + static_cast<uint32_t>(warp * 32 * kCh * 16);
          // Every chunk's TMEM load in flight before the first wait; under
          // the K split one chunk at a time (the partner's sums need the
          // registers).
          constexpr int kNChunks = kColsPerWarp / kChunk;
          constexpr int kBatch = N2 ? 1 : kNChunks;
          uint32_t r[kNChunks][kChunk];
#pragma unroll
          for (int cc = 0; cc < kNChunks; ++cc) {
            if (cc % kBatch == 0) {
#pragma unroll
              for (int c2 = cc; c2 < cc + kBatch; ++c2)
                ptx::tmem_ld_32x32b<kChunk>(t_row + c0 + c2 * kChunk, r[c2]);
              ptx::tmem_wait_ld();
            }
            add_partner(c0 + cc * kChunk, r[cc]);
            const int co0 = n0 + c0 + cc * kChunk;
#pragma unroll
            for (int g = 0; g < kChunk / 8; ++g) {
              uint4 pk;
              uint32_t *pw = reinterpret_cast<uint32_t *>(&pk);
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                float v0 = __uint_as_float(r[cc][g * 8 + 2 * h]);
                float v1 = __uint_as_float(r[cc][g * 8 + 2 * h + 1]);
                if (p.has_bias) {
                  v0 += ld_float(bias + co0 + g * 8 + 2 * h);
                  v1 += ld_float(bias + co0 + g * 8 + 2 * h + 1);
                }
                if (p.act_relu) {
                  v0 = fmaxf(v0, 0.f);
                  v1 = fmaxf(v1, 0.f);
                }
                pw[h] = GM::pack2(v0, v1);
              }
              const int c = cc * (kChunk / 8) + g;
              ptx::st_shared_v4(blk + lane * (kCh * 16) + ((c ^ (lane % kCh)) << 4), pk);
            }
          }
          __syncwarp();
          constexpr int kRowsPerStore = 32 / kCh;
          const int c = lane % kCh;
          const uint64_t yrow_bits = reinterpret_cast<uint64_t>(yrow);
#pragma unroll
          for (int i = 0; i < 32 / kRowsPerStore; ++i) {
            const int rl = i * kRowsPerStore + lane / kCh;   // row of the warp's block
            const uint4 v = ptx::ld_shared_v4(blk + rl * (kCh * 16) + ((c ^ (rl % kCh)) << 4));
            T *yr = reinterpret_cast<T *>(__shfl_sync(0xffffffffu, yrow_bits, rl));
            if (m0 + q * 32 + rl < p.M)
              *reinterpret_cast<uint4 *>(yr + n0 + c0 + c * 8) = v;
          }
          __syncwarp();   // the block is rewritten by the next window
        } else {
#pragma unroll 1
          for (int cb = 0; cb < kColsPerWarp; cb += kChunk) {
            const int col = c0 + cb;
            if (n0 + col >= p.Cout) break;
            uint32_t r[kChunk];
            acc(col, r);
            if (m < p.M) {
              const int co0 = n0 + col;
              float v[kChunk];
#pragma unroll
              for (int jj = 0; jj < kChunk; ++jj) {
                v[jj] = __uint_as_float(r[jj]);
                if (p.has_bias && co0 + jj < p.Cout) v[jj] += ld_float(bias + co0 + jj);
                if (p.act_relu) v[jj] = fmaxf(v[jj], 0.f);
              }
              if (vec_out && co0 + kChunk <= p.Cout) {
#pragma unroll
                for (int g = 0; g < kChunk / 8; ++g) {
                  uint4 pk;
                  uint32_t *pw = reinterpret_cast<uint32_t *>(&pk);
#pragma unroll
                  for (int h = 0; h < 4; ++h) pw[h] = GM::pack2(v[g * 8 + 2 * h], v[g * 8 + 2 * h + 1]);
                  *reinterpret_cast<uint4 *>(yrow + co0 + g * 8) = pk;
                }
              } else {
#pragma unroll
                for (int jj = 0; jj < kChunk; ++jj) {
                  if (co0 + jj < p.Cout) {
                    const uint16_t bits = GM::store_bits(v[jj]);
                    *reinterpret_cast<uint16_t *>(yrow + (co0 + jj) * p.ys[1]) = bits;
                  }
                }
              }
            }
          }
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  // Clustered CTAs: neither leaves (or frees TMEM) while the other may still
  // be reading its accumulator, arriving on its barriers or copying into it.
  if constexpr (CLUSTER) ptx::cluster_sync();
  if (warp == R::kMma) {
    ptx::tc_fence_after();
    if constexpr (PAIR) ptx::tmem_dealloc_pair(tmem_base, NCOLS);
    else ptx::tmem_dealloc(tmem_base, BN);
  }
}

// VB = bytes of input channels one gather lane loads per corner (16 or 32).
template <typename T, int BN, int STAGES, int VB>
__global__ void __launch_bounds__(tc_threads<kModeSingle>(), 1)
dcn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const TcParams p,
                  const T *__restrict__ x, const T *__restrict__ off, const T *__restrict__ msk,
                  const T *__restrict__ bias, T *__restrict__ y) {
  dcn_fwd_tc_body<T, BN, STAGES, kModeSingle, VB>(tmap_w, p, x, off, msk, bias, y);
}

template <typename T, int BN, int STAGES, int VB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(tc_threads<kModePair>(), 1)
dcn_fwd_tc_pair_kernel(const __grid_constant__ CUtensorMap tmap_w, const TcParams p,
                       const T *__restrict__ x, const T *__restrict__ off,
                       const T *__restrict__ msk, const T *__restrict__ bias,
                       T *__restrict__ y) {
  dcn_fwd_tc_body<T, BN, STAGES, kModePair, VB>(tmap_w, p, x, off, msk, bias, y);
}

template <typename T, int BN, int STAGES, int VB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(tc_threads<kModePairN2>(), 1)
dcn_fwd_tc_pairn2_kernel(const __grid_constant__ CUtensorMap tmap_w, const TcParams p,
                         const T *__restrict__ x, const T *__restrict__ off,
                         const T *__restrict__ msk, const T *__restrict__ bias,
                         T *__restrict__ y) {
  dcn_fwd_tc_body<T, BN, STAGES, kModePairN2, VB>(tmap_w, p, x, off, msk, bias, y);
}

template <typename T, int BN, int STAGES, int VB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(tc_threads<kModeNSplit>(), 1)
dcn_fwd_tc_nsplit_kernel(const __grid_constant__ CUtensorMap tmap_w, const TcParams p,
                         const T *__restrict__ x, const T *__restrict__ off,
                         const T *__restrict__ msk, const T *__restrict__ bias,
                         T *__restrict__ y) {
  dcn_fwd_tc_body<T, BN, STAGES, kModeNSplit, VB>(tmap_w, p, x, off, msk, bias, y);
}

// ---------------------------------------------------------------- host
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

template <typename T>
struct TypeTag {
  using type = T;
};

template <typename T, int BN, int STAGES, int MODE, int VB>
int launch_tc(const TcParams &p, const CUtensorMap &tmap, const void *x, const void *off,
              const void *msk, const void *bias, void *y, int ctas, cudaStream_t stream) {
  using L = Smem<BN, STAGES, MODE == kModePair || MODE == kModePairN2,
                 MODE == kModePairN2 ? 2 : 1>;
  static_assert(L::kAlloc <= 232448, "shared memory budget");
  auto kern = [] {
    if constexpr (MODE == kModePair) return dcn_fwd_tc_pair_kernel<T, BN, STAGES, VB>;
    else if constexpr (MODE == kModePairN2) return dcn_fwd_tc_pairn2_kernel<T, BN, STAGES, VB>;
    else if constexpr (MODE == kModeNSplit) return dcn_fwd_tc_nsplit_kernel<T, BN, STAGES, VB>;
    else return dcn_fwd_tc_kernel<T, BN, STAGES, VB>;
  }();
  // the shared-memory opt-in is a per-device function attribute
  constexpr int kMaxDevices = 64;
  static std::once_flag once[kMaxDevices];
  static cudaError_t attr_err[kMaxDevices];
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(BEVK_ERR_CUDA, "dcn tc: bad device %d", dev);
  std::call_once(once[dev], [&] {
    attr_err[dev] =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  });
  if (attr_err[dev] != cudaSuccess)
    return fail(BEVK_ERR_CUDA, "dcn tc: cudaFuncSetAttribute: %s",
                cudaGetErrorString(attr_err[dev]));
  if constexpr (MODE == kModePairN2) {
    if (p.k_split > 1) {
      // The two K parts of a tile wait for each other: every cluster must be
      // resident at once, or the caller takes a schedule without the split.
      static std::once_flag occ_once[kMaxDevices];
      static int max_clusters[kMaxDevices];
      std::call_once(occ_once[dev], [&] {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2);
        cfg.blockDim = dim3(tc_threads<MODE>());
        cfg.dynamicSmemBytes = L::kAlloc;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
          (void)cudaGetLastError();
          n = 0;
        }
        max_clusters[dev] = n;
      });
      if (ctas / 2 > max_clusters[dev]) return BEVK_ERR_UNSUPPORTED;
    }
  }
  // Programmatic dependent launch: the kernel's prologue overlaps the tail of
  // the stream's previous kernel; it waits for that kernel (griddepcontrol)
  // before touching global memory.
  return launched(launch_dependent(kern, dim3(static_cast<unsigned>(ctas)),
                                   dim3(tc_threads<MODE>()), L::kAlloc, stream, tmap, p,
                                   static_cast<const T *>(x), static_cast<const T *>(off),
                                   static_cast<const T *>(msk), static_cast<const T *>(bias),
                                   static_cast<T *>(y)),
                  "dcn_fwd_tc_kernel");
}

}  // namespace

bool dcn_tc_supported(const bevk_dcn_problem *pr, const DcnDims &d) {
  if (pr->dtype != BEVK_DTYPE_F16 && pr->dtype != BEVK_DTYPE_BF16) return false;
  if (d.groups != 1 || d.dg != 1) return false;
  if (d.Cin % 8 != 0 || d.T > kMaxTaps) return false;
  if (d.M >= (int64_t(1) << 31) - kBM) return false;
  const int dev = current_device();
  if (dev < 0 || device_info(dev).cc_major != 10) return false;
  return true;
}

namespace {
constexpr int kMinSplitStages = 8;   // K stages of each part, at least

// Tiles of the two-accumulator schedule with its K split in two, or 0 when
// the problem does not take it: more than 256 output channels, and all four
// CTAs of every 256-pixel x 512-channel tile fit on the SMs at once (the
// problems whose N-split grid fills at most one wave; per tile and stage the
// paired M=256 MMAs into two accumulators do the work of two N-split stages
// in about 1.5 times the time).
int64_t n2_split_tiles(const DcnDims &d) {
  if (d.Cout <= 256) return 0;
  const int n_k = d.T * (d.Cin_g_pad / kBK);
  if (n_k < 2 * kMinSplitStages) return 0;
  const int64_t tiles = ((d.M + 2 * kBM - 1) / (2 * kBM)) * ((d.Cout + 511) / 512);
  const int sms = device_info(current_device()).sm_count;
  if (sms <= 0 || 4 * tiles > sms) return 0;
  return tiles;
}

size_t align256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

// K-split scratch: tickets [tile][rank][2] (uint64), then the handed-over
// accumulator halves [tile][rank][K part][kSplitCols / 4][kBM][4] (fp32).
size_t split_tickets_bytes(int64_t tiles) {
  return align256(static_cast<size_t>(tiles) * 2 * 2 * sizeof(unsigned long long));
}
size_t split_ws_bytes(int64_t tiles) {
  return split_tickets_bytes(tiles) +
         static_cast<size_t>(tiles) * 4 * kSplitCols * kBM * sizeof(float);
}

// Schedule-dependent fields of p; returns the number of CTAs.
int64_t set_schedule(TcParams &p, const DcnDims &d, int mode, int BN, int k_split) {
  const int tile_n = mode == kModeNSplit || mode == kModePairN2 ? 2 * BN : BN;
  p.n_tiles_n = (d.Cout + tile_n - 1) / tile_n;
  p.k_split = k_split;
  p.k_len = (p.n_k + k_split - 1) / k_split;
  const bool pair = mode == kModePair || mode == kModePairN2;
  const int64_t m_tiles = pair ? (d.M + 2 * kBM - 1) / (2 * kBM) : (d.M + kBM - 1) / kBM;
  return (mode == kModeSingle ? 1 : 2) * m_tiles * p.n_tiles_n * k_split;
}
}  // namespace

size_t dcn_tc_workspace_bytes(const bevk_dcn_problem *p, const DcnDims &d) {
  if (!dcn_tc_supported(p, d)) return 0;
  const int64_t tiles = n2_split_tiles(d);
  return tiles ? split_ws_bytes(tiles) : 0;
}

int launch_dcn_forward_tc(const bevk_dcn_problem *pr, const DcnDims &d, const void *x,
                          const int64_t xs[4], const void *off, const void *msk,
                          const void *wpk, const void *bias, void *y, void *ws, size_t ws_bytes,
                          cudaStream_t stream) {
  if (xs[1] != 1 || xs[0] % 8 || xs[2] % 8 || xs[3] % 8 || !aligned(x, 16) || !aligned(wpk, 16))
    return fail(BEVK_ERR_MISALIGNED, "dcn tc: input must be channel-contiguous with 16-byte rows");
  const int64_t extent = (d.B - 1) * xs[0] + (d.H - 1) * xs[2] + (d.W - 1) * xs[3] + d.Cin;
  // int32 element offsets inside the kernel; corner offsets are stored doubled
  if (extent >= (int64_t(1) << 30) || xs[0] >= (int64_t(1) << 30))
    return fail(BEVK_ERR_INDEX_OVERFLOW, "dcn tc: input extent exceeds 30-bit indexing");
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(BEVK_ERR_CUDA, "dcn tc: cuTensorMapEncodeTiled unavailable");

  const int BN = d.Cout <= 64 ? 64 : (d.Cout <= 128 ? 128 : 256);
  TcParams p;
  p.Cin = d.Cin; p.H = d.H; p.W = d.W; p.Ho = d.Ho; p.Wo = d.Wo; p.Cout = d.Cout;
  p.kW = d.kW; p.T = d.T;
  p.sh = d.sh; p.sw = d.sw; p.ph = d.ph; p.pw = d.pw; p.dh = d.dh; p.dw = d.dw;
  for (int t = 0; t < kMaxTaps; ++t) {
    p.tap_dy[t] = t < d.T ? (t / d.kW) * d.dh - d.ph : 0;
    p.tap_dx[t] = t < d.T ? (t % d.kW) * d.dw - d.pw : 0;
  }
  p.M = static_cast<int>(d.M);
  p.Cin_pad = d.Cin_g_pad;
  p.n_cc = p.Cin_pad / kBK;
  p.n_k = p.T * p.n_cc;
  p.part = nullptr;
  p.tickets = nullptr;
  // Tile schedule: more than 256 output channels -> paired M=256 CTAs with
  // two accumulators and K split in two when the problem fills at most one
  // wave and scratch is given, else N-split CTA pairs (one gather per pixel
  // for 512 channels); 129..256 -> M-paired CTAs (M=256 MMA, half the weight
  // tile per CTA); up to 128 -> single CTAs.
  int mode = d.Cout > 256 ? kModeNSplit : (BN == 256 ? kModePair : kModeSingle);
  const int64_t split_tiles = n2_split_tiles(d);
  if (split_tiles && ws && aligned(ws, 256) && ws_bytes >= split_ws_bytes(split_tiles)) {
    mode = kModePairN2;
    p.tickets = static_cast<unsigned long long *>(ws);
    p.part = reinterpret_cast<float *>(static_cast<char *>(ws) + split_tickets_bytes(split_tiles));
  }
  p.mask_is_logit = pr->mask_is_logit;
  p.has_bias = pr->has_bias;
  p.act_relu = pr->act_relu;
  p.wait_limit_ns = wait_limit(current_device());
  p.xs0 = static_cast<int>(xs[0]); p.xs2 = static_cast<int>(xs[2]); p.xs3 = static_cast<int>(xs[3]);
  for (int i = 0; i < 4; ++i) {
    p.os[i] = pr->offset_strides[i];
    p.ms[i] = pr->mask_strides[i];
    p.ys[i] = pr->output_strides[i];
  }
  const int64_t ctas = set_schedule(p, d, mode, BN, mode == kModePairN2 ? 2 : 1);
  if (ctas > 0x7FFFFFFF) return fail(BEVK_ERR_INDEX_OVERFLOW, "dcn tc: too many tiles");

  // A paired CTA loads its half of each BN-channel weight tile per stage.
  auto make_map = [&](bool pair, CUtensorMap *tmap) -> int {
    const cuuint64_t gdim[2] = {static_cast<cuuint64_t>(d.T) * p.Cin_pad,
                                static_cast<cuuint64_t>(d.Cout)};
    const cuuint64_t gstride[1] = {static_cast<cuuint64_t>(d.T) * p.Cin_pad * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK),
                               static_cast<cuuint32_t>(pair ? BN / 2 : BN)};
    const cuuint32_t estride[2] = {1, 1};
    const CUtensorMapDataType dt = pr->dtype == BEVK_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const CUresult cr = enc(tmap, dt, 2, const_cast<void *>(wpk), gdim, gstride, box, estride,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(BEVK_ERR_CUDA, "dcn tc: tensor map encode failed (%d)", int(cr));
    return BEVK_OK;
  };
  CUtensorMap tmap;
  int st = make_map(mode == kModePair || mode == kModePairN2, &tmap);
  if (st != BEVK_OK) return st;

  // 32-byte corner loads when every pixel row starts on a 32-byte boundary
  // and a lane's 16 channels are all inside or all outside Cin (N-split CTAs
  // gather 64 rows: one 16-byte vector per lane covers them).
  const bool v32 = d.Cin % 16 == 0 && xs[0] % 16 == 0 &&
                   xs[2] % 16 == 0 && xs[3] % 16 == 0 && aligned(x, 32);
  auto go = [&](auto tag) -> int {
    using T = typename decltype(tag)::type;
    int nc = static_cast<int>(ctas);
    if (mode == kModePairN2) {
      // BEVK_ERR_UNSUPPORTED: the clusters would not all be resident at once
      const int rc = v32 ? launch_tc<T, 256, 3, kModePairN2, 32>(p, tmap, x, off, msk, bias, y, nc, stream)
                         : launch_tc<T, 256, 3, kModePairN2, 16>(p, tmap, x, off, msk, bias, y, nc, stream);
      if (rc != BEVK_ERR_UNSUPPORTED) return rc;
      mode = kModeNSplit;
      nc = static_cast<int>(set_schedule(p, d, mode, BN, 1));
      const int mst = make_map(false, &tmap);
      if (mst != BEVK_OK) return mst;
    }
    // N-split CTAs hold the whole 256-channel weight tile per stage: three
    // stages keep shared memory at 159 KB, leaving ~92 KB of L1 for the
    // corner reads (four stages would leave ~28 KB and halve the hit rate).
    if (mode == kModeNSplit)
      return v32 ? launch_tc<T, 256, 3, kModeNSplit, 32>(p, tmap, x, off, msk, bias, y, nc, stream)
                 : launch_tc<T, 256, 3, kModeNSplit, 16>(p, tmap, x, off, msk, bias, y, nc, stream);
    if (v32) {
      if (BN == 256) return launch_tc<T, 256, 4, kModePair, 32>(p, tmap, x, off, msk, bias, y, nc, stream);
      if (BN == 128) return launch_tc<T, 128, 4, kModeSingle, 32>(p, tmap, x, off, msk, bias, y, nc, stream);
      return launch_tc<T, 64, 4, kModeSingle, 32>(p, tmap, x, off, msk, bias, y, nc, stream);
    }
    if (BN == 256) return launch_tc<T, 256, 4, kModePair, 16>(p, tmap, x, off, msk, bias, y, nc, stream);
    if (BN == 128) return launch_tc<T, 128, 4, kModeSingle, 16>(p, tmap, x, off, msk, bias, y, nc, stream);
    return launch_tc<T, 64, 4, kModeSingle, 16>(p, tmap, x, off, msk, bias, y, nc, stream);
  };
  if (pr->dtype == BEVK_DTYPE_F16) return go(TypeTag<__half>{});
  return go(TypeTag<__nv_bfloat16>{});
}

namespace {
// Per-device limit of the fused kernel's pipeline barrier waits, passed to
// every launch (0 = the default).
constexpr int kMaxWaitDevices = 64;
std::atomic<unsigned long long> g_wait_limit_ns[kMaxWaitDevices];
}  // namespace

unsigned long long wait_limit(int device) {
  const unsigned long long v =
      device >= 0 && device < kMaxWaitDevices ? g_wait_limit_ns[device].load() : 0ull;
  return v ? v : ptx::kWaitLimitNs;
}

int set_wait_limit(int device, unsigned long long ns) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(BEVK_ERR_CUDA, "wait limit: no CUDA device");
  }
  if (device < 0 || device >= n || device >= kMaxWaitDevices)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "wait limit: bad device %d", device);
  g_wait_limit_ns[device].store(ns);
  return BEVK_OK;
}

int read_and_clear_watchdog(int device, unsigned int *code) {
  int prev = -1;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) {
    (void)cudaGetLastError();  // leave no error pending for later launch checks
    return fail(BEVK_ERR_INVALID_ARGUMENT, "watchdog: bad device %d", device);
  }
  unsigned int v = 0, zero = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_bevk_watchdog, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_bevk_watchdog, &zero, sizeof(zero));
  if (prev >= 0) cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(BEVK_ERR_CUDA, "watchdog: %s", cudaGetErrorString(e));
  if (code) *code = v;
  return v ? fail(BEVK_ERR_DEVICE_TIMEOUT, "device watchdog fired at site 0x%x", v) : BEVK_OK;
}

}  // namespace bevk
