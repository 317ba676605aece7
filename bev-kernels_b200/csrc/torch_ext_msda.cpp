// torch_ext_msda.cpp -- module _ms_deform_attn_ext: the reference MSDA
// extension's forward and backward (csrc_musa/msda/binding_musa.mu:286-412,
// :414-543, :546-556) over the C ABI.  Same argument order, keyword defaults,
// contiguity checks and im2col_step contract; output dtype = value dtype.
#include "torch_ext_common.h"

using at::Tensor;
using namespace bevk_ext;

namespace {

Tensor forward(const Tensor &value, const Tensor &spatial_shapes, const Tensor &level_start_index,
               const Tensor &sampling_loc, const Tensor &attn_weight, int64_t im2col_step,
               bool force_generic) {
  (void)force_generic;  // one kernel family; kept for signature compatibility
  check_cuda(value, "value");
  for (const Tensor *t : {&spatial_shapes, &level_start_index, &sampling_loc, &attn_weight})
    check_same_device(value, *t, "msda tensor");
  TORCH_CHECK(value.is_contiguous(), "value must be contiguous");
  TORCH_CHECK(spatial_shapes.is_contiguous(), "spatial_shapes must be contiguous");
  TORCH_CHECK(level_start_index.is_contiguous(), "level_start_index must be contiguous");
  TORCH_CHECK(sampling_loc.is_contiguous(), "sampling_loc must be contiguous");
  TORCH_CHECK(attn_weight.is_contiguous(), "attn_weight must be contiguous");
  TORCH_CHECK(value.dim() == 4, "value must be [B, S, heads, C]");
  TORCH_CHECK(sampling_loc.dim() == 6, "sampling_loc must be [B, Q, heads, L, P, 2]");
  TORCH_CHECK(attn_weight.dim() == 5, "attn_weight must be [B, Q, heads, L, P]");
  TORCH_CHECK(spatial_shapes.scalar_type() == at::kLong &&
                  level_start_index.scalar_type() == at::kLong,
              "spatial_shapes / level_start_index must be int64");
  TORCH_CHECK(sampling_loc.scalar_type() == value.scalar_type() &&
                  attn_weight.scalar_type() == value.scalar_type(),
              "sampling_loc / attn_weight must share value's dtype");
  const int batch = static_cast<int>(value.size(0));
  const int spatial_size = static_cast<int>(value.size(1));
  const int num_heads = static_cast<int>(value.size(2));
  const int channels = static_cast<int>(value.size(3));
  const int num_levels = static_cast<int>(spatial_shapes.size(0));
  const int num_query = static_cast<int>(sampling_loc.size(1));
  const int num_point = static_cast<int>(sampling_loc.size(4));
  TORCH_CHECK(sampling_loc.size(0) == batch && sampling_loc.size(2) == num_heads &&
                  sampling_loc.size(3) == num_levels && sampling_loc.size(5) == 2,
              "sampling_loc shape mismatch");
  TORCH_CHECK(attn_weight.size(0) == batch && attn_weight.size(1) == num_query &&
                  attn_weight.size(2) == num_heads && attn_weight.size(3) == num_levels &&
                  attn_weight.size(4) == num_point,
              "attn_weight shape mismatch");
  TORCH_CHECK(level_start_index.numel() == num_levels, "level_start_index must have L entries");
  const int step = static_cast<int>(std::min<int64_t>(batch, im2col_step));
  TORCH_CHECK(step > 0 && batch % step == 0, "batch must divide im2col_step");
  const int dt = dtype_of(value);
  Tensor output = at::empty({batch, num_query, num_heads * channels}, value.options());
  if (output.numel() == 0) return output;
  const c10::cuda::CUDAGuard guard(value.device());
  check_status(bevk_ms_deform_attn_forward(
                   value.data_ptr(), spatial_shapes.data_ptr<int64_t>(),
                   level_start_index.data_ptr<int64_t>(), sampling_loc.data_ptr(),
                   attn_weight.data_ptr(), batch, spatial_size, num_heads, channels, num_levels,
                   num_query, num_point, static_cast<int>(im2col_step), output.data_ptr(), dt,
                   current_stream(value)),
               "ms_deform_attn_forward");
  return output;
}

// Writes into caller-zeroed grads like the reference (fp32: grad_value is
// accumulated into; fp16/bf16: accumulated in an fp32 workspace, then written).
void backward(const Tensor &value, const Tensor &spatial_shapes, const Tensor &level_start_index,
              const Tensor &sampling_loc, const Tensor &attn_weight, const Tensor &grad_output,
              Tensor &grad_value, Tensor &grad_sampling_loc, Tensor &grad_attn_weight,
              int64_t im2col_step, bool force_generic_col2im) {
  (void)force_generic_col2im;  // one kernel family; kept for signature compatibility
  check_cuda(value, "value");
  for (const Tensor *t : std::initializer_list<const Tensor *>{
           &spatial_shapes, &level_start_index, &sampling_loc, &attn_weight, &grad_output,
           &grad_value, &grad_sampling_loc, &grad_attn_weight})
    check_same_device(value, *t, "msda tensor");
  TORCH_CHECK(value.is_contiguous(), "value must be contiguous");
  TORCH_CHECK(spatial_shapes.is_contiguous(), "spatial_shapes must be contiguous");
  TORCH_CHECK(level_start_index.is_contiguous(), "level_start_index must be contiguous");
  TORCH_CHECK(sampling_loc.is_contiguous(), "sampling_loc must be contiguous");
  TORCH_CHECK(attn_weight.is_contiguous(), "attn_weight must be contiguous");
  TORCH_CHECK(grad_value.is_contiguous() && grad_sampling_loc.is_contiguous() &&
                  grad_attn_weight.is_contiguous(),
              "gradient outputs must be contiguous");
  TORCH_CHECK(value.dim() == 4 && sampling_loc.dim() == 6 && attn_weight.dim() == 5,
              "value [B,S,heads,C], sampling_loc [B,Q,heads,L,P,2], attn_weight [B,Q,heads,L,P]");
  TORCH_CHECK(grad_value.sizes() == value.sizes() &&
                  grad_sampling_loc.sizes() == sampling_loc.sizes() &&
                  grad_attn_weight.sizes() == attn_weight.sizes(),
              "gradient shapes must match their inputs");
  for (const Tensor *t : std::initializer_list<const Tensor *>{
           &sampling_loc, &attn_weight, &grad_output, &grad_value, &grad_sampling_loc,
           &grad_attn_weight})
    TORCH_CHECK(t->scalar_type() == value.scalar_type(), "msda tensors must share value's dtype");
  const int batch = static_cast<int>(value.size(0));
  const int spatial_size = static_cast<int>(value.size(1));
  const int num_heads = static_cast<int>(value.size(2));
  const int channels = static_cast<int>(value.size(3));
  const int num_levels = static_cast<int>(spatial_shapes.size(0));
  const int num_query = static_cast<int>(sampling_loc.size(1));
  const int num_point = static_cast<int>(sampling_loc.size(4));
  TORCH_CHECK(grad_output.numel() ==
                  static_cast<int64_t>(batch) * num_query * num_heads * channels,
              "grad_output must be [B, Q, heads*C]");
  const int step = static_cast<int>(std::min<int64_t>(batch, im2col_step));
  TORCH_CHECK(step > 0 && batch % step == 0, "batch must divide im2col_step");
  // the reference takes strided grad_output; the kernel reads it contiguous
  const Tensor g = grad_output.contiguous();
  const int dt = dtype_of(value);
  const c10::cuda::CUDAGuard guard(value.device());
  const size_t ws = bevk_ms_deform_attn_backward_workspace_bytes(batch, spatial_size, num_heads,
                                                                 channels, dt);
  Tensor workspace;
  if (ws > 0) workspace = at::empty({static_cast<int64_t>(ws)}, value.options().dtype(at::kByte));
  check_status(bevk_ms_deform_attn_backward(
                   value.data_ptr(), spatial_shapes.data_ptr<int64_t>(),
                   level_start_index.data_ptr<int64_t>(), sampling_loc.data_ptr(),
                   attn_weight.data_ptr(), g.data_ptr(), batch, spatial_size, num_heads, channels,
                   num_levels, num_query, num_point, static_cast<int>(im2col_step),
                   grad_value.data_ptr(), grad_sampling_loc.data_ptr(),
                   grad_attn_weight.data_ptr(), ws > 0 ? workspace.data_ptr() : nullptr, ws, dt,
                   current_stream(value)),
               "ms_deform_attn_backward");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("forward", &forward, "Multi-scale deformable attention forward", py::arg("value"),
        py::arg("spatial_shapes"), py::arg("level_start_index"), py::arg("sampling_loc"),
        py::arg("attn_weight"), py::arg("im2col_step") = 64, py::arg("force_generic") = false);
  m.def("backward", &backward, "Multi-scale deformable attention backward", py::arg("value"),
        py::arg("spatial_shapes"), py::arg("level_start_index"), py::arg("sampling_loc"),
        py::arg("attn_weight"), py::arg("grad_output"), py::arg("grad_value"),
        py::arg("grad_sampling_loc"), py::arg("grad_attn_weight"), py::arg("im2col_step") = 64,
        py::arg("force_generic_col2im") = false);
}
