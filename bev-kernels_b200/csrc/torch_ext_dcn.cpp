// torch_ext_dcn.cpp -- module _modulated_deform_conv_ext: the reference
// extension's forward op names (csrc/binding.cpp:142-191) over the C ABI, plus
// the fused forward and weight packing used by modulated_deform_conv.
#include <cstring>

#include "torch_ext_common.h"

using at::Tensor;
using namespace bevk_ext;

namespace {

void col_common(const Tensor &data_im, const Tensor &data_offset, const Tensor &data_mask,
                int batch_size, int channels, int height_im, int width_im, int height_col,
                int width_col, int kernel_h, int kernel_w, int pad_h, int pad_w, int stride_h,
                int stride_w, int dilation_h, int dilation_w, int deformable_group,
                Tensor data_col, int layout) {
  check_cuda(data_im, "data_im");
  check_same_device(data_im, data_offset, "data_offset");
  check_same_device(data_im, data_mask, "data_mask");
  check_same_device(data_im, data_col, "data_col");
  TORCH_CHECK(data_im.is_contiguous() && data_offset.is_contiguous() &&
                  data_mask.is_contiguous() && data_col.is_contiguous(),
              "bevk: im2col tensors must be contiguous");
  const int dt = dtype_of(data_im);
  TORCH_CHECK(data_offset.scalar_type() == data_im.scalar_type() &&
                  data_mask.scalar_type() == data_im.scalar_type() &&
                  data_col.scalar_type() == data_im.scalar_type(),
              "bevk: im2col tensors must share data_im's dtype");
  const int64_t T = int64_t(kernel_h) * kernel_w;
  const int64_t need = int64_t(channels) * T * batch_size * height_col * width_col;
  TORCH_CHECK(data_col.numel() == need, "bevk: data_col has ", data_col.numel(),
              " elements, expected ", need);
  const c10::cuda::CUDAGuard guard(data_im.device());
  int st;
  if (layout == 0) {
    st = bevk_modulated_deformable_im2col_opt(
        data_im.data_ptr(), data_offset.data_ptr(), data_mask.data_ptr(), batch_size, channels,
        height_im, width_im, height_col, width_col, kernel_h, kernel_w, pad_h, pad_w, stride_h,
        stride_w, dilation_h, dilation_w, deformable_group, data_col.data_ptr(), dt,
        current_stream(data_im));
  } else {
    st = bevk_modulated_deformable_im2col_nhwc(
        data_im.data_ptr(), data_offset.data_ptr(), data_mask.data_ptr(), batch_size, channels,
        height_im, width_im, height_col, width_col, kernel_h, kernel_w, pad_h, pad_w, stride_h,
        stride_w, dilation_h, dilation_w, deformable_group,
        static_cast<int>(data_offset.size(-1)), data_col.data_ptr(), dt, current_stream(data_im));
  }
  check_status(st, layout == 0 ? "modulated_deformable_im2col" : "modulated_deformable_im2col_nhwc");
}

// csrc/binding.cpp:5-11 / :143-145
void modulated_deformable_im2col_cuda(const Tensor data_im, const Tensor data_offset,
                                      const Tensor data_mask, int batch_size, int channels,
                                      int height_im, int width_im, int height_col, int width_col,
                                      int kernel_h, int kernel_w, int pad_h, int pad_w,
                                      int stride_h, int stride_w, int dilation_h, int dilation_w,
                                      int deformable_group, Tensor data_col) {
  col_common(data_im, data_offset, data_mask, batch_size, channels, height_im, width_im,
             height_col, width_col, kernel_h, kernel_w, pad_h, pad_w, stride_h, stride_w,
             dilation_h, dilation_w, deformable_group, data_col, 0);
}

// csrc/binding.cpp:21-27 / :149-151
void modulated_deformable_im2col_opt_cuda(const Tensor data_im, const Tensor data_offset,
                                          const Tensor data_mask, int batch_size, int channels,
                                          int height_im, int width_im, int height_col,
                                          int width_col, int kernel_h, int kernel_w, int pad_h,
                                          int pad_w, int stride_h, int stride_w, int dilation_h,
                                          int dilation_w, int deformable_group, Tensor data_col) {
  col_common(data_im, data_offset, data_mask, batch_size, channels, height_im, width_im,
             height_col, width_col, kernel_h, kernel_w, pad_h, pad_w, stride_h, stride_w,
             dilation_h, dilation_w, deformable_group, data_col, 0);
}

// csrc/binding.cpp:61-67 / :163-165
void modulated_deformable_im2col_nhwc_cuda(const Tensor data_im, const Tensor data_offset,
                                           const Tensor data_mask, int batch_size, int channels,
                                           int height_im, int width_im, int height_col,
                                           int width_col, int kernel_h, int kernel_w, int pad_h,
                                           int pad_w, int stride_h, int stride_w,
                                           int dilation_h, int dilation_w, int deformable_group,
                                           Tensor data_col) {
  col_common(data_im, data_offset, data_mask, batch_size, channels, height_im, width_im,
             height_col, width_col, kernel_h, kernel_w, pad_h, pad_w, stride_h, stride_w,
             dilation_h, dilation_w, deformable_group, data_col, 1);
}

bevk_dcn_problem make_problem(const Tensor &input, const Tensor &offset, const Tensor &mask,
                              const Tensor &output, int64_t out_channels, int kernel_h,
                              int kernel_w, int stride_h, int stride_w, int pad_h, int pad_w,
                              int dil_h, int dil_w, int groups, int deform_groups,
                              bool mask_is_logit, bool has_bias) {
  bevk_dcn_problem p;
  std::memset(&p, 0, sizeof(p));
  p.dtype = dtype_of(input);
  p.batch = static_cast<int>(input.size(0));
  p.in_channels = static_cast<int>(input.size(1));
  p.height = static_cast<int>(input.size(2));
  p.width = static_cast<int>(input.size(3));
  p.out_channels = static_cast<int>(out_channels);
  p.kernel_h = kernel_h; p.kernel_w = kernel_w;
  p.stride_h = stride_h; p.stride_w = stride_w; p.pad_h = pad_h; p.pad_w = pad_w;
  p.dilation_h = dil_h; p.dilation_w = dil_w;
  p.groups = groups; p.deformable_groups = deform_groups;
  for (int i = 0; i < 4; ++i) {
    p.input_strides[i] = input.stride(i);
    p.offset_strides[i] = offset.stride(i);
    p.mask_strides[i] = mask.stride(i);
    p.output_strides[i] = output.defined() ? output.stride(i) : 0;
  }
  p.mask_is_logit = mask_is_logit ? 1 : 0;
  p.has_bias = has_bias ? 1 : 0;
  return p;
}

// Packs weight [Cout, Cin/groups, kH, kW] into the [Cout][kH*kW][Cin_g_pad]
// layout of bevk_dcn_forward.
Tensor dcn_pack_weight(const Tensor &weight, int64_t groups) {
  check_cuda(weight, "weight");
  TORCH_CHECK(weight.dim() == 4, "bevk: weight must be 4-D [Cout, Cin/groups, kH, kW]");
  const Tensor w = weight.contiguous();
  bevk_dcn_problem p;
  std::memset(&p, 0, sizeof(p));
  p.dtype = dtype_of(w);
  p.batch = 1; p.height = 1; p.width = 1;
  p.in_channels = static_cast<int>(w.size(1) * groups);
  p.out_channels = static_cast<int>(w.size(0));
  p.kernel_h = static_cast<int>(w.size(2)); p.kernel_w = static_cast<int>(w.size(3));
  p.stride_h = p.stride_w = p.dilation_h = p.dilation_w = 1;
  p.pad_h = p.kernel_h; p.pad_w = p.kernel_w;
  p.groups = static_cast<int>(groups); p.deformable_groups = 1;
  const size_t bytes = bevk_dcn_packed_weight_bytes(&p);
  TORCH_CHECK(bytes > 0, "bevk: invalid weight geometry: ", bevk_last_error_message());
  const int64_t cin_pad = static_cast<int64_t>(bytes / (w.element_size() * p.out_channels *
                                                        p.kernel_h * p.kernel_w));
  Tensor packed = at::empty({w.size(0), w.size(2) * w.size(3), cin_pad}, w.options());
  const c10::cuda::CUDAGuard guard(w.device());
  check_status(bevk_dcn_pack_weight(&p, w.data_ptr(), packed.data_ptr(), current_stream(w)),
               "dcn_pack_weight");
  return packed;
}

// Fused forward into a caller-provided output (any memory format).
void dcn_forward(const Tensor &input, const Tensor &offset, const Tensor &mask,
                 const Tensor &packed_weight, const c10::optional<Tensor> &bias, Tensor output,
                 int64_t kernel_h, int64_t kernel_w, int64_t stride_h, int64_t stride_w,
                 int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w, int64_t groups,
                 int64_t deform_groups, bool mask_is_logit) {
  check_cuda(input, "input");
  for (const Tensor *t : std::initializer_list<const Tensor *>{&offset, &mask, &packed_weight, &output})
    check_same_device(input, *t, "dcn tensor");
  TORCH_CHECK(input.dim() == 4 && offset.dim() == 4 && mask.dim() == 4 && output.dim() == 4,
              "bevk: dcn_forward expects 4-D input/offset/mask/output");
  const auto st = input.scalar_type();
  TORCH_CHECK(offset.scalar_type() == st && mask.scalar_type() == st &&
                  packed_weight.scalar_type() == st && output.scalar_type() == st,
              "bevk: dcn_forward tensors must share the input dtype");
  TORCH_CHECK(packed_weight.is_contiguous(), "bevk: packed weight must be contiguous");
  const bool has_bias = bias.has_value() && bias->defined();
  Tensor b;
  if (has_bias) {
    b = bias->contiguous();
    check_same_device(input, b, "bias");
    TORCH_CHECK(b.scalar_type() == st && b.numel() == output.size(1), "bevk: bad bias");
  }
  bevk_dcn_problem p = make_problem(input, offset, mask, output, output.size(1),
                                    static_cast<int>(kernel_h), static_cast<int>(kernel_w),
                                    static_cast<int>(stride_h), static_cast<int>(stride_w),
                                    static_cast<int>(pad_h), static_cast<int>(pad_w),
                                    static_cast<int>(dil_h), static_cast<int>(dil_w),
                                    static_cast<int>(groups), static_cast<int>(deform_groups),
                                    mask_is_logit, has_bias);
  int ho = 0, wo = 0;
  check_status(bevk_dcn_output_size(&p, &ho, &wo), "dcn_forward");
  TORCH_CHECK(output.size(0) == p.batch && output.size(2) == ho && output.size(3) == wo,
              "bevk: output must be [", p.batch, ", Cout, ", ho, ", ", wo, "]");
  TORCH_CHECK(offset.size(0) == p.batch && offset.size(1) == 2 * deform_groups * kernel_h * kernel_w &&
                  offset.size(2) == ho && offset.size(3) == wo,
              "bevk: offset must be [B, 2*dg*kH*kW, Ho, Wo]");
  TORCH_CHECK(mask.size(0) == p.batch && mask.size(1) == deform_groups * kernel_h * kernel_w &&
                  mask.size(2) == ho && mask.size(3) == wo,
              "bevk: mask must be [B, dg*kH*kW, Ho, Wo]");
  TORCH_CHECK(static_cast<size_t>(packed_weight.numel()) * packed_weight.element_size() ==
                  bevk_dcn_packed_weight_bytes(&p),
              "bevk: packed weight does not match the problem (pack with dcn_pack_weight)");
  const c10::cuda::CUDAGuard guard(input.device());
  const size_t ws_bytes = bevk_dcn_forward_workspace_bytes(&p);
  Tensor ws;
  if (ws_bytes) ws = at::empty({static_cast<int64_t>(ws_bytes)}, input.options().dtype(at::kByte));
  check_status(bevk_dcn_forward(&p, input.data_ptr(), offset.data_ptr(), mask.data_ptr(),
                                packed_weight.data_ptr(), has_bias ? b.data_ptr() : nullptr,
                                output.data_ptr(), ws_bytes ? ws.data_ptr() : nullptr, ws_bytes,
                                current_stream(input)),
               "dcn_forward");
}

int64_t watchdog(int64_t device) {
  unsigned int code = 0;
  bevk_device_watchdog(static_cast<int>(device), &code);
  return static_cast<int64_t>(code);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("modulated_deformable_im2col_cuda", &modulated_deformable_im2col_cuda,
        "Modulated deformable im2col, NCHW column matrix [C*kH*kW, B*Ho*Wo]");
  m.def("modulated_deformable_im2col_opt_cuda", &modulated_deformable_im2col_opt_cuda,
        "Modulated deformable im2col, NCHW column matrix [C*kH*kW, B*Ho*Wo]");
  m.def("modulated_deformable_im2col_nhwc_cuda", &modulated_deformable_im2col_nhwc_cuda,
        "Modulated deformable gather, NHWC column matrix [B*Ho*Wo, kH*kW*C]");
  m.def("dcn_pack_weight", &dcn_pack_weight, "Pack [Cout, Cin/g, kH, kW] weights",
        py::arg("weight"), py::arg("groups") = 1);
  m.def("dcn_forward", &dcn_forward, "Fused DCNv2 forward (tcgen05 / exact SIMT)",
        py::arg("input"), py::arg("offset"), py::arg("mask"), py::arg("packed_weight"),
        py::arg("bias"), py::arg("output"), py::arg("kernel_h"), py::arg("kernel_w"),
        py::arg("stride_h"), py::arg("stride_w"), py::arg("pad_h"), py::arg("pad_w"),
        py::arg("dil_h"), py::arg("dil_w"), py::arg("groups"), py::arg("deform_groups"),
        py::arg("mask_is_logit") = false);
  m.def("watchdog", &watchdog, "Read and clear the device watchdog word (0 = clean)",
        py::arg("device"));
  m.def("version", []() { return bevk_version(); });
}
