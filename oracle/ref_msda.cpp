// ref_msda.cpp -- the reference's own generic MSDA forward kernel
// (csrc_musa/msda/ms_deform_attn_kernels.cuh:559-623, with its bilinear helper
// :7-49), included from the reference tree and run on the host through
// ref_shim/.  Pins the C oracle's MSDA restatement.  TEST INFRASTRUCTURE ONLY:
// built into oracle/_ref/ by `make -C oracle ref` when the reference tree is
// present; nothing in the product loads it.
#include "device_shim.h"
#include "ms_deform_attn_kernels.cuh"

extern "C" int ref_msda_forward_f32(const float *value, const int64_t *spatial_shapes,
                                    const int64_t *level_start_index, const float *sampling_loc,
                                    const float *attn_weight, int batch, int spatial_size,
                                    int num_heads, int channels, int num_levels, int num_query,
                                    int num_point, float *out) {
  const int64_t n = static_cast<int64_t>(batch) * num_query * num_heads * channels;
  if (n >= (int64_t(1) << 31)) return -1;
  ms_deformable_im2col_generic_kernel<float>(
      static_cast<int>(n), value, spatial_shapes, level_start_index, sampling_loc, attn_weight,
      batch, spatial_size, num_heads, channels, num_levels, num_query, num_point, out,
      at::musa::FastDivmod(channels), at::musa::FastDivmod(num_heads),
      at::musa::FastDivmod(num_query));
  return 0;
}
