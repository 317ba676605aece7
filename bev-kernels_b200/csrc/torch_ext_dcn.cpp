// torch_ext_dcn.cpp -- module _modulated_deform_conv_ext: the reference
// extension's op names (csrc/binding.cpp:142-191: im2col forward ops and the
// col2im backward family) over the C ABI, plus the fused forward and weight
// packing used by modulated_deform_conv.
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

void dcn_offset_conv_sum(const Tensor &partials, const c10::optional<Tensor> &offset_bias,
                         Tensor offset_out, int64_t batch, int64_t height, int64_t width,
                         int64_t kernel_h, int64_t kernel_w, int64_t stride_h, int64_t stride_w,
                         int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w);

// csrc/binding.cpp:72-78 / :167-169 (csrc/dcn_fused_nhwc_cuda.cu:92-126): the
// Pack module's offset convolution and the deformable gather in one call.
// data_im [B, H, W, Cin] contiguous, w_off [3T, T, Cin] (the offset conv's
// weight [3T, Cin, kH, kW] permuted (0, 2, 3, 1)), b_off [3T] (fp32),
// data_col [B*Ho*Wo, T*Cin] (k = t*Cin + ci), deformable_group 1.  The offset
// conv's channel reduction runs as one GEMM with fp32 output, the tap sum and
// bias in bevk_dcn_offset_conv_sum (rounded once to the input dtype, as the
// unfused offset conv returns it), then the NHWC gather reads offsets and
// mask logits from that output (sigmoid applied on load).
void modulated_deformable_fused_im2col_nhwc_cuda(const Tensor data_im, const Tensor w_off,
                                                 const Tensor b_off, int batch_size, int channels,
                                                 int height_im, int width_im, int height_col,
                                                 int width_col, int kernel_h, int kernel_w,
                                                 int pad_h, int pad_w, int stride_h, int stride_w,
                                                 int dilation_h, int dilation_w,
                                                 int deformable_group, Tensor data_col) {
  TORCH_CHECK(deformable_group == 1, "bevk: the NHWC fused path supports deformable_group == 1");
  TORCH_CHECK(int64_t(kernel_h) * kernel_w <= 9,
              "bevk: the fused offset-conv gather supports kernels of at most 9 taps");
  check_cuda(data_im, "data_im");
  check_same_device(data_im, w_off, "w_off");
  check_same_device(data_im, b_off, "b_off");
  check_same_device(data_im, data_col, "data_col");
  const int64_t T = int64_t(kernel_h) * kernel_w;
  const int64_t C3 = 3 * T;
  TORCH_CHECK(data_im.dim() == 4 && data_im.is_contiguous() && data_im.size(0) == batch_size &&
                  data_im.size(1) == height_im && data_im.size(2) == width_im &&
                  data_im.size(3) == channels,
              "bevk: data_im must be contiguous NHWC [B, H, W, Cin]");
  TORCH_CHECK(w_off.scalar_type() == data_im.scalar_type() && w_off.numel() == C3 * T * channels,
              "bevk: w_off must be [3*kH*kW, kH*kW, Cin] in data_im's dtype");
  TORCH_CHECK(b_off.numel() == C3, "bevk: b_off must have 3*kH*kW elements");
  const c10::cuda::CUDAGuard guard(data_im.device());
  // GEMM operand [ld, Cin]: row t*3T + c = w_off[c, t, :], zero rows up to ld
  const int64_t n = T * C3, ld = (n + 31) / 32 * 32;
  Tensor wz = at::zeros({ld, channels}, data_im.options());
  wz.narrow(0, 0, n).copy_(w_off.reshape({C3, T, channels}).permute({1, 0, 2}).reshape({n, channels}));
  const Tensor x2 = data_im.reshape({int64_t(batch_size) * height_im * width_im, channels});
  const Tensor partials = data_im.scalar_type() == at::kFloat
                              ? at::mm(x2, wz.t())
                              : at::mm(x2, wz.t(), at::kFloat);
  Tensor y = at::empty({batch_size, height_col, width_col, C3}, data_im.options());
  dcn_offset_conv_sum(partials, b_off, y, batch_size, height_im, width_im, kernel_h, kernel_w,
                      stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w);
  col_common(data_im, y, y, batch_size, channels, height_im, width_im, height_col, width_col,
             kernel_h, kernel_w, pad_h, pad_w, stride_h, stride_w, dilation_h, dilation_w, 1,
             data_col, 1);
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

// Offset convolution from its per-tap partial products
// (bevk_dcn_offset_conv_sum): partials [B*H*W, ld >= T*3T] fp32 with unit
// column stride; offset_out [B, Ho, Wo, 3T] contiguous in the output dtype.
void dcn_offset_conv_sum(const Tensor &partials, const c10::optional<Tensor> &offset_bias,
                         Tensor offset_out, int64_t batch, int64_t height, int64_t width,
                         int64_t kernel_h, int64_t kernel_w, int64_t stride_h, int64_t stride_w,
                         int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w) {
  check_cuda(partials, "partials");
  check_same_device(partials, offset_out, "offset_out");
  const int64_t T = kernel_h * kernel_w;
  TORCH_CHECK(partials.scalar_type() == at::kFloat && partials.dim() == 2 &&
                  partials.size(0) == batch * height * width && partials.size(1) >= T * 3 * T &&
                  partials.stride(1) == 1 && partials.stride(0) >= T * 3 * T,
              "bevk: partials must be fp32 [B*H*W, >= 3*T*T] with unit column stride");
  Tensor ob;
  if (offset_bias.has_value() && offset_bias->defined()) {
    ob = offset_bias->to(at::kFloat).contiguous();
    check_same_device(partials, ob, "offset_bias");
    TORCH_CHECK(ob.numel() == 3 * T, "bevk: offset_bias must have 3*kH*kW elements");
  }
  bevk_dcn_problem p;
  std::memset(&p, 0, sizeof(p));
  p.dtype = dtype_of(offset_out);
  p.batch = static_cast<int>(batch);
  p.height = static_cast<int>(height);
  p.width = static_cast<int>(width);
  p.in_channels = 8;
  p.out_channels = 1;
  p.kernel_h = static_cast<int>(kernel_h); p.kernel_w = static_cast<int>(kernel_w);
  p.stride_h = static_cast<int>(stride_h); p.stride_w = static_cast<int>(stride_w);
  p.pad_h = static_cast<int>(pad_h); p.pad_w = static_cast<int>(pad_w);
  p.dilation_h = static_cast<int>(dil_h); p.dilation_w = static_cast<int>(dil_w);
  p.groups = 1; p.deformable_groups = 1;
  int ho = 0, wo = 0;
  check_status(bevk_dcn_output_size(&p, &ho, &wo), "dcn_offset_conv_sum");
  TORCH_CHECK(offset_out.is_contiguous() && offset_out.dim() == 4 && offset_out.size(0) == batch &&
                  offset_out.size(1) == ho && offset_out.size(2) == wo &&
                  offset_out.size(3) == 3 * T,
              "bevk: offset_out must be contiguous [B, Ho, Wo, 3*kH*kW]");
  const c10::cuda::CUDAGuard guard(partials.device());
  bevk_dcn_zoff_args z{partials.data_ptr<float>(), partials.stride(0),
                       ob.defined() ? ob.data_ptr<float>() : nullptr, offset_out.data_ptr()};
  check_status(bevk_dcn_offset_conv_sum(&p, &z, current_stream(partials)), "dcn_offset_conv_sum");
}

// Fused forward into a caller-provided output (any memory format).
void dcn_forward(const Tensor &input, const Tensor &offset, const Tensor &mask,
                 const Tensor &packed_weight, const c10::optional<Tensor> &bias, Tensor output,
                 int64_t kernel_h, int64_t kernel_w, int64_t stride_h, int64_t stride_w,
                 int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w, int64_t groups,
                 int64_t deform_groups, bool mask_is_logit, bool act_relu) {
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
  p.act_relu = act_relu ? 1 : 0;
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

// ------------------------------------------------------------------ backward
// Logical (b, c, h, w) strides of a tensor stored NCHW or NHWC ([B, H, W, C]).
void logical_strides(const Tensor &t, bool nhwc, int64_t out[4]) {
  if (nhwc) {
    out[0] = t.stride(0); out[1] = t.stride(3); out[2] = t.stride(1); out[3] = t.stride(2);
  } else {
    for (int i = 0; i < 4; ++i) out[i] = t.stride(i);
  }
}

// One gradient output of the scatter: written in place when it already is the
// accumulation type and the op accumulates, else through an fp32 (fp64)
// scratch that is added to it (accumulate) or copied over it (overwrite).
struct GradOut {
  Tensor *dst = nullptr;
  Tensor buf;
  bool overwrite = false;
  void *prepare(at::ScalarType acc) {
    if (dst == nullptr || !dst->defined()) return nullptr;
    if (!overwrite && dst->scalar_type() == acc) return dst->data_ptr();
    buf = at::zeros(dst->sizes(), dst->options().dtype(acc).memory_format(
                                       dst->suggest_memory_format()));
    return buf.data_ptr();
  }
  const Tensor &target() const { return buf.defined() ? buf : *dst; }
  void finish() {
    if (!buf.defined()) return;
    if (overwrite) dst->copy_(buf);
    else dst->add_(buf);
  }
};

// col_nhwc: dcol is [M, kH*kW*C] (k = t*C + c) instead of [C*kH*kW, M];
// img_nhwc: data_im [B, H, W, C], offset [B, Ho, Wo, 2T] or the fused
// offset-conv output [B, Ho, Wo, 3T] (mask then read from it, pre-sigmoid),
// mask [B, Ho, Wo, T], gradients in the same layouts.
void col2im_common(const Tensor &dcol, const Tensor *data_im, const Tensor &offset,
                   const Tensor &mask, int batch, int channels, int height, int width,
                   int height_col, int width_col, int kernel_h, int kernel_w, int pad_h,
                   int pad_w, int stride_h, int stride_w, int dil_h, int dil_w, int dg,
                   bool col_nhwc, bool img_nhwc, Tensor *grad_im, Tensor *grad_offset,
                   Tensor *grad_mask, bool overwrite_coord, const char *what) {
  check_cuda(dcol, "dcol");
  check_same_device(dcol, offset, "offset");
  check_same_device(dcol, mask, "mask");
  if (data_im) check_same_device(dcol, *data_im, "data_im");
  TORCH_CHECK(dcol.is_contiguous(), "bevk: ", what, ": the column gradient must be contiguous");
  const int T = kernel_h * kernel_w;
  const int64_t M = static_cast<int64_t>(batch) * height_col * width_col;
  TORCH_CHECK(dcol.numel() == static_cast<int64_t>(channels) * T * M, "bevk: ", what,
              ": the column gradient has ", dcol.numel(), " elements, expected ",
              static_cast<int64_t>(channels) * T * M);
  const at::ScalarType xt = offset.scalar_type();
  TORCH_CHECK(mask.scalar_type() == xt && (!data_im || data_im->scalar_type() == xt),
              "bevk: ", what, ": data_im / offset / mask must share a dtype");
  TORCH_CHECK(dcol.scalar_type() == xt || dcol.scalar_type() == at::kFloat, "bevk: ", what,
              ": the column gradient must be float32 or the input dtype");
  const bool fused_y = img_nhwc && offset.dim() == 4 && offset.size(-1) == 3 * T && dg == 1;
  bevk_dcn_col2im_args a;
  std::memset(&a, 0, sizeof(a));
  bevk_dcn_problem &p = a.problem;
  p.dtype = dtype_of(offset);
  p.batch = batch; p.in_channels = channels; p.height = height; p.width = width;
  p.out_channels = 1; p.kernel_h = kernel_h; p.kernel_w = kernel_w;
  p.stride_h = stride_h; p.stride_w = stride_w; p.pad_h = pad_h; p.pad_w = pad_w;
  p.dilation_h = dil_h; p.dilation_w = dil_w; p.groups = 1; p.deformable_groups = dg;
  if (data_im) logical_strides(*data_im, img_nhwc, p.input_strides);
  logical_strides(offset, img_nhwc, p.offset_strides);
  const void *mask_ptr = mask.data_ptr();
  if (fused_y) {
    for (int i = 0; i < 4; ++i) p.mask_strides[i] = p.offset_strides[i];
    mask_ptr = static_cast<const char *>(offset.data_ptr()) +
               static_cast<int64_t>(2 * T) * offset.stride(3) * offset.element_size();
    p.mask_is_logit = 1;
  } else {
    logical_strides(mask, img_nhwc, p.mask_strides);
  }
  a.col_dtype = dtype_of(dcol);
  if (col_nhwc) {
    a.col_strides[0] = static_cast<int64_t>(T) * channels; a.col_strides[1] = 1;
    a.col_strides[2] = channels;
  } else {
    a.col_strides[0] = 1; a.col_strides[1] = static_cast<int64_t>(T) * M; a.col_strides[2] = M;
  }
  const at::ScalarType acc = xt == at::kDouble ? at::kDouble : at::kFloat;
  GradOut gx, go, gm;
  gx.dst = grad_im;
  go.dst = grad_offset; go.overwrite = overwrite_coord;
  gm.dst = grad_mask; gm.overwrite = overwrite_coord;
  for (Tensor *t : {grad_im, grad_offset, grad_mask})
    if (t && t->defined()) check_same_device(dcol, *t, "gradient");
  const c10::cuda::CUDAGuard guard(dcol.device());
  void *gx_ptr = gx.prepare(acc), *go_ptr = go.prepare(acc), *gm_ptr = gm.prepare(acc);
  if (gx_ptr) logical_strides(gx.target(), img_nhwc, a.grad_input_strides);
  if (go_ptr) logical_strides(go.target(), img_nhwc, a.grad_offset_strides);
  if (gm_ptr) logical_strides(gm.target(), img_nhwc, a.grad_mask_strides);
  check_status(bevk_dcn_col2im(&a, data_im ? data_im->data_ptr() : nullptr, offset.data_ptr(),
                               mask_ptr, dcol.data_ptr(), gx_ptr, go_ptr, gm_ptr,
                               current_stream(dcol)),
               what);
  gx.finish();
  go.finish();
  gm.finish();
}

#define BEVK_COL2IM_GEOM_ARGS                                                              \
  int batch_size, int channels, int height_im, int width_im, int height_col, int width_col, \
      int kernel_h, int kernel_w, int pad_h, int pad_w, int stride_h, int stride_w,          \
      int dilation_h, int dilation_w, int deformable_group
#define BEVK_COL2IM_GEOM                                                                   \
  batch_size, channels, height_im, width_im, height_col, width_col, kernel_h, kernel_w,     \
      pad_h, pad_w, stride_h, stride_w, dilation_h, dilation_w, deformable_group

// csrc/binding.cpp:13-43: NCHW column matrix -> grad_im (accumulated)
void col2im_nchw(const Tensor data_col, const Tensor data_offset, const Tensor data_mask,
                 BEVK_COL2IM_GEOM_ARGS, Tensor grad_im) {
  col2im_common(data_col, nullptr, data_offset, data_mask, BEVK_COL2IM_GEOM, false, false,
                &grad_im, nullptr, nullptr, false, "modulated_deformable_col2im");
}

// csrc/binding.cpp:45-59: NCHW column matrix -> grad_offset, grad_mask (written)
void col2im_coord_nchw(const Tensor data_col, const Tensor data_im, const Tensor data_offset,
                       const Tensor data_mask, BEVK_COL2IM_GEOM_ARGS, Tensor grad_offset,
                       Tensor grad_mask) {
  col2im_common(data_col, &data_im, data_offset, data_mask, BEVK_COL2IM_GEOM, false, false,
                nullptr, &grad_offset, &grad_mask, true, "modulated_deformable_col2im_coord");
}

// csrc/binding.cpp:80-87, :115-140: NHWC dcol -> grad_im, grad_offset, grad_mask
// (accumulated into the caller's zeroed fp32 tensors)
void col2im_nhwc(const Tensor dcol, const Tensor data_im, const Tensor data_offset,
                 const Tensor data_mask, BEVK_COL2IM_GEOM_ARGS, Tensor grad_im,
                 Tensor grad_offset, Tensor grad_mask) {
  col2im_common(dcol, &data_im, data_offset, data_mask, BEVK_COL2IM_GEOM, true, true, &grad_im,
                &grad_offset, &grad_mask, false, "modulated_deformable_col2im_nhwc");
}

// csrc/binding.cpp:89-95
void col2im_coord_nhwc(const Tensor dcol, const Tensor data_im, const Tensor data_offset,
                       const Tensor data_mask, BEVK_COL2IM_GEOM_ARGS, Tensor grad_offset,
                       Tensor grad_mask) {
  col2im_common(dcol, &data_im, data_offset, data_mask, BEVK_COL2IM_GEOM, true, true, nullptr,
                &grad_offset, &grad_mask, false, "modulated_deformable_col2im_coord_nhwc");
}

// csrc/binding.cpp:97-113: NHWC dcol -> grad_im only
void gradx_nhwc(const Tensor dcol, const Tensor data_offset, const Tensor data_mask,
                BEVK_COL2IM_GEOM_ARGS, Tensor grad_im) {
  col2im_common(dcol, nullptr, data_offset, data_mask, BEVK_COL2IM_GEOM, true, true, &grad_im,
                nullptr, nullptr, false, "modulated_deformable_gradx_nhwc");
}
void gradx_gather_nhwc(const Tensor dcol, const Tensor data_offset, const Tensor data_mask,
                       BEVK_COL2IM_GEOM_ARGS, int win, Tensor grad_im) {
  (void)win;  // the reference's gather window; the scatter needs none
  gradx_nhwc(dcol, data_offset, data_mask, BEVK_COL2IM_GEOM, grad_im);
}

// Generic scatter used by the autograd Functions: NCHW-shaped input / offset /
// mask / gradients in any memory format, the column gradient [M, kH*kW*C]
// (k = t*C + c); undefined gradient tensors are skipped.
void dcn_col2im(const Tensor &dcol, const c10::optional<Tensor> &input, const Tensor &offset,
                const Tensor &mask, int64_t in_channels, int64_t height, int64_t width,
                int64_t kernel_h, int64_t kernel_w, int64_t stride_h, int64_t stride_w,
                int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w,
                int64_t deform_groups, c10::optional<Tensor> grad_input,
                c10::optional<Tensor> grad_offset, c10::optional<Tensor> grad_mask) {
  TORCH_CHECK(offset.dim() == 4 && mask.dim() == 4, "bevk: dcn_col2im: offset / mask must be 4-D");
  Tensor gi = grad_input.has_value() ? *grad_input : Tensor();
  Tensor go = grad_offset.has_value() ? *grad_offset : Tensor();
  Tensor gm = grad_mask.has_value() ? *grad_mask : Tensor();
  const Tensor *in = input.has_value() && input->defined() ? &*input : nullptr;
  col2im_common(dcol, in, offset, mask, static_cast<int>(offset.size(0)),
                static_cast<int>(in_channels), static_cast<int>(height), static_cast<int>(width),
                static_cast<int>(offset.size(2)), static_cast<int>(offset.size(3)),
                static_cast<int>(kernel_h), static_cast<int>(kernel_w), static_cast<int>(pad_h),
                static_cast<int>(pad_w), static_cast<int>(stride_h), static_cast<int>(stride_w),
                static_cast<int>(dil_h), static_cast<int>(dil_w), static_cast<int>(deform_groups),
                true, false, gi.defined() ? &gi : nullptr, go.defined() ? &go : nullptr,
                gm.defined() ? &gm : nullptr, false, "dcn_col2im");
}

// Data side of the backward in one call (bevk_dcn_backward_data): NCHW-shaped
// input / offset / mask / gradients in any memory format (an NHWC tensor is
// passed as its permuted view), NHWC column matrices [M, kH*kW*C] with unit
// column stride.  Returns false, having written nothing, when the layouts are
// not the channel-contiguous 16-byte-vector ones the kernels need or the
// problem exceeds their 32-bit indices.
bool dcn_backward_data(const c10::optional<Tensor> &dcol, const c10::optional<Tensor> &input,
                       const Tensor &offset, const Tensor &mask, bool mask_is_logit,
                       int64_t in_channels, int64_t height, int64_t width, int64_t kernel_h,
                       int64_t kernel_w, int64_t stride_h, int64_t stride_w, int64_t pad_h,
                       int64_t pad_w, int64_t dil_h, int64_t dil_w, int64_t deform_groups,
                       c10::optional<Tensor> grad_input, c10::optional<Tensor> grad_offset,
                       c10::optional<Tensor> grad_mask, c10::optional<Tensor> col) {
  auto get = [](const c10::optional<Tensor> &t) {
    return t.has_value() && t->defined() ? *t : Tensor();
  };
  const Tensor dc = get(dcol), in = get(input), gi = get(grad_input), go = get(grad_offset),
               gm = get(grad_mask), cl = get(col);
  check_cuda(offset, "offset");
  check_same_device(offset, mask, "mask");
  TORCH_CHECK(offset.dim() == 4 && mask.dim() == 4,
              "bevk: dcn_backward_data: offset / mask must be 4-D");
  TORCH_CHECK(mask.scalar_type() == offset.scalar_type(),
              "bevk: dcn_backward_data: offset / mask must share a dtype");
  for (const Tensor *t : {&dc, &in, &gi, &go, &gm, &cl})
    if (t->defined()) check_same_device(offset, *t, "tensor");
  for (const Tensor *t : {&dc, &in, &cl})
    if (t->defined())
      TORCH_CHECK(t->scalar_type() == offset.scalar_type(),
                  "bevk: dcn_backward_data: input / dcol / col must have the offset dtype");
  at::ScalarType gt = offset.scalar_type();
  bool first = true;
  for (const Tensor *t : {&gi, &go, &gm})
    if (t->defined()) {
      TORCH_CHECK(first || t->scalar_type() == gt,
                  "bevk: dcn_backward_data: the gradients must share a dtype");
      gt = t->scalar_type();
      first = false;
    }
  const int64_t T = kernel_h * kernel_w;
  const int64_t M = offset.size(0) * offset.size(2) * offset.size(3);
  for (const Tensor *t : {&dc, &cl})
    if (t->defined())
      TORCH_CHECK(t->dim() == 2 && t->size(0) == M && t->size(1) == T * in_channels &&
                      t->stride(1) == 1,
                  "bevk: dcn_backward_data: column matrices must be [M, kH*kW*C] with unit "
                  "column stride");
  bevk_dcn_backward_data_args a;
  std::memset(&a, 0, sizeof(a));
  bevk_dcn_problem &p = a.problem;
  p.dtype = dtype_of(offset);
  p.batch = static_cast<int>(offset.size(0));
  p.in_channels = static_cast<int>(in_channels);
  p.height = static_cast<int>(height);
  p.width = static_cast<int>(width);
  p.out_channels = 1;
  p.kernel_h = static_cast<int>(kernel_h); p.kernel_w = static_cast<int>(kernel_w);
  p.stride_h = static_cast<int>(stride_h); p.stride_w = static_cast<int>(stride_w);
  p.pad_h = static_cast<int>(pad_h); p.pad_w = static_cast<int>(pad_w);
  p.dilation_h = static_cast<int>(dil_h); p.dilation_w = static_cast<int>(dil_w);
  p.groups = 1;
  p.deformable_groups = static_cast<int>(deform_groups);
  p.mask_is_logit = mask_is_logit ? 1 : 0;
  for (int i = 0; i < 4; ++i) {
    p.input_strides[i] = in.defined() ? in.stride(i) : 0;
    p.offset_strides[i] = offset.stride(i);
    p.mask_strides[i] = mask.stride(i);
    a.grad_input_strides[i] = gi.defined() ? gi.stride(i) : 0;
    a.grad_offset_strides[i] = go.defined() ? go.stride(i) : 0;
    a.grad_mask_strides[i] = gm.defined() ? gm.stride(i) : 0;
  }
  a.grad_dtype = first ? p.dtype : (gt == at::kFloat ? BEVK_DTYPE_F32 : p.dtype);
  if (!first && gt != at::kFloat)
    TORCH_CHECK(gt == offset.scalar_type(),
                "bevk: dcn_backward_data: gradients must be float32 or the input dtype");
  a.dcol_ld = dc.defined() ? dc.stride(0) : 0;
  a.col_ld = cl.defined() ? cl.stride(0) : 0;
  const c10::cuda::CUDAGuard guard(offset.device());
  Tensor ws;
  if (gi.defined()) {
    const size_t bytes = bevk_dcn_backward_data_workspace_bytes(&p);
    ws = at::empty({static_cast<int64_t>(bytes)}, offset.options().dtype(at::kByte));
  }
  auto ptr = [](const Tensor &t) { return t.defined() ? t.data_ptr() : nullptr; };
  const int st = bevk_dcn_backward_data(&a, ptr(in), offset.data_ptr(), mask.data_ptr(), ptr(dc),
                                        ptr(gi), ptr(go), ptr(gm), ptr(cl), ptr(ws),
                                        ws.defined() ? static_cast<size_t>(ws.numel()) : 0,
                                        current_stream(offset));
  // layouts or sizes this entry point does not cover: the caller takes the
  // general scatter path (any strides, 64-bit indices)
  if (st == BEVK_ERR_UNSUPPORTED || st == BEVK_ERR_INDEX_OVERFLOW) return false;
  check_status(st, "dcn_backward_data");
  return true;
}

// Deformable columns of NCHW-shaped tensors in any memory format: layout 0
// [C*kH*kW, M], layout 1 [M, kH*kW*C].
Tensor dcn_columns(const Tensor &input, const Tensor &offset, const Tensor &mask,
                   int64_t kernel_h, int64_t kernel_w, int64_t stride_h, int64_t stride_w,
                   int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w,
                   int64_t deform_groups, int64_t layout) {
  check_cuda(input, "input");
  check_same_device(input, offset, "offset");
  check_same_device(input, mask, "mask");
  TORCH_CHECK(offset.scalar_type() == input.scalar_type() &&
                  mask.scalar_type() == input.scalar_type(),
              "bevk: dcn_columns: input / offset / mask must share a dtype");
  const int64_t T = kernel_h * kernel_w;
  const int64_t M = offset.size(0) * offset.size(2) * offset.size(3);
  Tensor col = layout == 0 ? at::empty({input.size(1) * T, M}, input.options())
                           : at::empty({M, T * input.size(1)}, input.options());
  bevk_dcn_problem p = make_problem(input, offset, mask, Tensor(), 1, static_cast<int>(kernel_h),
                                    static_cast<int>(kernel_w), static_cast<int>(stride_h),
                                    static_cast<int>(stride_w), static_cast<int>(pad_h),
                                    static_cast<int>(pad_w), static_cast<int>(dil_h),
                                    static_cast<int>(dil_w), 1, static_cast<int>(deform_groups),
                                    false, false);
  const c10::cuda::CUDAGuard guard(input.device());
  check_status(bevk_dcn_columns(&p, input.data_ptr(), offset.data_ptr(), mask.data_ptr(),
                                col.data_ptr(), static_cast<int>(layout), current_stream(input)),
               "dcn_columns");
  return col;
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
  m.def("modulated_deformable_fused_im2col_nhwc_cuda",
        &modulated_deformable_fused_im2col_nhwc_cuda,
        "Offset conv + deformable gather + sigmoid modulation -> Col [M, T*Cin], NHWC dg=1");
  m.def("dcn_pack_weight", &dcn_pack_weight, "Pack [Cout, Cin/g, kH, kW] weights",
        py::arg("weight"), py::arg("groups") = 1);
  m.def("dcn_offset_conv_sum", &dcn_offset_conv_sum,
        "Offset convolution of the Pack module from its per-tap partial products",
        py::arg("partials"), py::arg("offset_bias"), py::arg("offset_out"), py::arg("batch"),
        py::arg("height"), py::arg("width"), py::arg("kernel_h"), py::arg("kernel_w"),
        py::arg("stride_h"), py::arg("stride_w"), py::arg("pad_h"), py::arg("pad_w"),
        py::arg("dil_h"), py::arg("dil_w"));
  m.def("dcn_forward", &dcn_forward, "Fused DCNv2 forward (tcgen05 / exact SIMT)",
        py::arg("input"), py::arg("offset"), py::arg("mask"), py::arg("packed_weight"),
        py::arg("bias"), py::arg("output"), py::arg("kernel_h"), py::arg("kernel_w"),
        py::arg("stride_h"), py::arg("stride_w"), py::arg("pad_h"), py::arg("pad_w"),
        py::arg("dil_h"), py::arg("dil_w"), py::arg("groups"), py::arg("deform_groups"),
        py::arg("mask_is_logit") = false, py::arg("act_relu") = false);
  // backward column scatter under the reference's op names (csrc/binding.cpp:146-191)
  for (const char *name : {"modulated_deformable_col2im_cuda", "modulated_deformable_col2im_opt_cuda",
                           "modulated_deformable_col2im_smem_cuda"})
    m.def(name, &col2im_nchw, "Column gradient [C*kH*kW, B*Ho*Wo] -> grad_im (accumulated)");
  for (const char *name : {"modulated_deformable_col2im_coord_cuda",
                           "modulated_deformable_col2im_coord_opt_cuda"})
    m.def(name, &col2im_coord_nchw,
          "Column gradient [C*kH*kW, B*Ho*Wo] -> grad_offset, grad_mask (written)");
  for (const char *name : {"modulated_deformable_col2im_nhwc_cuda",
                           "modulated_deformable_col2im_fused_smem_nhwc_cuda",
                           "modulated_deformable_col2im_perelem_nhwc_cuda",
                           "modulated_deformable_col2im_perelem_smem_nhwc_cuda"})
    m.def(name, &col2im_nhwc,
          "NHWC column gradient [M, kH*kW*C] -> grad_im, grad_offset, grad_mask (accumulated)");
  m.def("modulated_deformable_col2im_coord_nhwc_cuda", &col2im_coord_nhwc,
        "NHWC column gradient -> grad_offset, grad_mask (accumulated)");
  m.def("modulated_deformable_gradx_smem_nhwc_cuda", &gradx_nhwc,
        "NHWC column gradient -> grad_im (accumulated)");
  m.def("modulated_deformable_gradx_gather_nhwc_cuda", &gradx_gather_nhwc,
        "NHWC column gradient -> grad_im (accumulated)");
  m.def("dcn_col2im", &dcn_col2im,
        "DCN backward scatter: NHWC column gradient -> grad_input / grad_offset / grad_mask "
        "(NCHW-shaped, any memory format, accumulated)",
        py::arg("dcol"), py::arg("input"), py::arg("offset"), py::arg("mask"),
        py::arg("in_channels"), py::arg("height"), py::arg("width"), py::arg("kernel_h"),
        py::arg("kernel_w"), py::arg("stride_h"), py::arg("stride_w"), py::arg("pad_h"),
        py::arg("pad_w"), py::arg("dil_h"), py::arg("dil_w"), py::arg("deform_groups"),
        py::arg("grad_input"), py::arg("grad_offset"), py::arg("grad_mask"));
  m.def("dcn_backward_data", &dcn_backward_data,
        "DCN backward data side without floating-point atomics: grad_input / grad_offset / "
        "grad_mask (written) and the NHWC column matrix; False when the layout is not covered",
        py::arg("dcol"), py::arg("input"), py::arg("offset"), py::arg("mask"),
        py::arg("mask_is_logit"), py::arg("in_channels"), py::arg("height"), py::arg("width"),
        py::arg("kernel_h"), py::arg("kernel_w"), py::arg("stride_h"), py::arg("stride_w"),
        py::arg("pad_h"), py::arg("pad_w"), py::arg("dil_h"), py::arg("dil_w"),
        py::arg("deform_groups"), py::arg("grad_input"), py::arg("grad_offset"),
        py::arg("grad_mask"), py::arg("col"));
  m.def("dcn_columns", &dcn_columns,
        "Deformable column matrix (layout 0: [C*kH*kW, M], 1: [M, kH*kW*C])",
        py::arg("input"), py::arg("offset"), py::arg("mask"), py::arg("kernel_h"),
        py::arg("kernel_w"), py::arg("stride_h"), py::arg("stride_w"), py::arg("pad_h"),
        py::arg("pad_w"), py::arg("dil_h"), py::arg("dil_w"), py::arg("deform_groups"),
        py::arg("layout"));
  m.def("watchdog", &watchdog, "Read and clear the device watchdog word (0 = clean)",
        py::arg("device"));
  m.def("version", []() { return bevk_version(); });
}
