// ref_msda.cpp -- the reference's own generic MSDA kernels, included from the
// reference tree and run on the host through ref_shim/: the forward
// (csrc_musa/msda/ms_deform_attn_kernels.cuh:559-623, bilinear helper :7-49)
// and the backward (ms_deformable_col2im_shm_stride_v1_kernel :1168-1271,
// bilinear gradient helper :426-491, launched as binding_musa.mu:266-282 does:
// one block of `channels` threads per (batch, query, head)).  Pins the C
// oracle's MSDA restatement.  TEST INFRASTRUCTURE ONLY: built into
// oracle/_ref/ by `make -C oracle ref` when the reference tree is present;
// nothing in the product loads it.
#include <thread>
#include <vector>

#include "device_shim.h"
#include "ms_deform_attn_kernels.cuh"

// The backward kernel's dynamic shared memory (3 floats per thread of the
// emulated block); one block runs at a time.
int msda_shm[3 * 1024];

extern "C" int ref_msda_forward_f32(const float *value, const int64_t *spatial_shapes,
                                    const int64_t *level_start_index, const float *sampling_loc,
                                    const float *attn_weight, int batch, int spatial_size,
                                    int num_heads, int channels, int num_levels, int num_query,
                                    int num_point, float *out) {
  const int64_t n = static_cast<int64_t>(batch) * num_query * num_heads * channels;
  if (n >= (int64_t(1) << 31)) return -1;
  blockDim.x = 1;
  ms_deformable_im2col_generic_kernel<float>(
      static_cast<int>(n), value, spatial_shapes, level_start_index, sampling_loc, attn_weight,
      batch, spatial_size, num_heads, channels, num_levels, num_query, num_point, out,
      at::musa::FastDivmod(channels), at::musa::FastDivmod(num_heads),
      at::musa::FastDivmod(num_query));
  return 0;
}

// grad_value is accumulated into (the reference's callers pass zeros);
// grad_sampling_loc and grad_attn_weight are written.  grad_output is
// contiguous [batch, num_query, num_heads * channels].
extern "C" int ref_msda_backward_f32(const float *value, const int64_t *spatial_shapes,
                                     const int64_t *level_start_index,
                                     const float *sampling_loc, const float *attn_weight,
                                     const float *grad_output, int batch, int spatial_size,
                                     int num_heads, int channels, int num_levels,
                                     int num_query, int num_point, float *grad_value,
                                     float *grad_sampling_loc, float *grad_attn_weight) {
  const int64_t n = static_cast<int64_t>(batch) * num_query * num_heads * channels;
  if (n >= (int64_t(1) << 31) || channels < 1 || channels > 1024) return -1;
  blockDim.x = static_cast<unsigned>(channels);
  bevk_ref_block_barrier.parties = static_cast<unsigned>(channels);
  const int64_t sb = static_cast<int64_t>(num_query) * num_heads * channels;
  const int64_t sq = static_cast<int64_t>(num_heads) * channels;
  std::vector<std::thread> block;
  for (int t = 0; t < channels; ++t)
    block.emplace_back([=] {
      threadIdx.x = static_cast<unsigned>(t);
      ms_deformable_col2im_shm_stride_v1_kernel<float>(
          static_cast<int>(n), grad_output, sb, sq, channels, 1, true, value, spatial_shapes,
          level_start_index, sampling_loc, attn_weight, batch, spatial_size, num_heads,
          channels, num_levels, num_query, num_point, grad_value, grad_sampling_loc,
          grad_attn_weight, at::musa::FastDivmod(channels), at::musa::FastDivmod(num_heads),
          at::musa::FastDivmod(num_query));
    });
  for (auto &th : block) th.join();
  blockDim.x = 1;
  bevk_ref_block_barrier.parties = 1;
  return 0;
}
