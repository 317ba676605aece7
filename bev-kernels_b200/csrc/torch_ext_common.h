// torch_ext_common.h -- helpers shared by the torch extensions: dtype mapping,
// device checks and status -> RuntimeError translation.  The extensions hold no
// CUDA code; every kernel runs behind the C ABI of include/bevk.h.
#pragma once

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include "bevk.h"

namespace bevk_ext {

inline int dtype_of(const at::Tensor &t) {
  switch (t.scalar_type()) {
    case at::kFloat: return BEVK_DTYPE_F32;
    case at::kHalf: return BEVK_DTYPE_F16;
    case at::kBFloat16: return BEVK_DTYPE_BF16;
    case at::kDouble: return BEVK_DTYPE_F64;
    default:
      TORCH_CHECK(false, "bevk: unsupported dtype ", t.scalar_type(),
                  " (float32, float16, bfloat16, float64)");
  }
  return -1;
}

inline void check_cuda(const at::Tensor &t, const char *name) {
  TORCH_CHECK(t.is_cuda(), "bevk: ", name, " must be a CUDA tensor (no CPU fallback)");
}

inline void check_same_device(const at::Tensor &a, const at::Tensor &b, const char *name) {
  TORCH_CHECK(a.device() == b.device(), "bevk: ", name, " is on ", b.device(), ", expected ",
              a.device());
}

inline void check_status(int st, const char *what) {
  TORCH_CHECK(st == BEVK_OK, "bevk: ", what, " failed: ", bevk_status_string(st), ": ",
              bevk_last_error_message());
}

inline bevk_stream_t current_stream(const at::Tensor &t) {
  return reinterpret_cast<bevk_stream_t>(
      c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

}  // namespace bevk_ext
