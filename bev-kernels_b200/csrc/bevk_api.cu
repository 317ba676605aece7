// bevk_api.cu -- the extern "C" entry points declared in include/bevk.h:
// argument validation, kernel selection and error reporting.  No entry point
// allocates device memory; scratch comes from the caller's workspace.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <string>

#include "bevk.h"
#include "bevk_internal.h"

#define BEVK_VERSION_NUMBER 10000  // 1.0.0

namespace bevk {

namespace {
thread_local char g_last_error[512] = {0};
}

int fail(int status, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

void clear_error() { g_last_error[0] = 0; }

const char *last_error() { return g_last_error; }

int check_launch(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(BEVK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return BEVK_OK;
}

int launched(cudaError_t launch_result, const char *what) {
  if (launch_result != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(BEVK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(launch_result));
  }
  return check_launch(what);
}

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

bool programmatic_launch_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("BEVK_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

const DeviceInfo &device_info(int device) {
  constexpr int kMaxDevices = 64;
  static DeviceInfo infos[kMaxDevices];
  static std::once_flag flags[kMaxDevices];
  static DeviceInfo invalid;
  if (device < 0 || device >= kMaxDevices) return invalid;
  std::call_once(flags[device], [device] {
    DeviceInfo &d = infos[device];
    d.device = device;
    cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, device);
    cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, device);
    cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    cudaDeviceGetAttribute(&d.l2_bytes, cudaDevAttrL2CacheSize, device);
  });
  return infos[device];
}

static int out_size(int in, int pad, int dil, int k, int stride) {
  return (in + 2 * pad - (dil * (k - 1) + 1)) / stride + 1;
}

int dcn_dims(const bevk_dcn_problem *p, DcnDims *d) {
  if (!p || !d) return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn: null problem");
  if (dtype_size(p->dtype) == 0) return fail(BEVK_ERR_UNSUPPORTED, "dcn: unknown dtype %d", p->dtype);
  if (p->batch <= 0 || p->in_channels <= 0 || p->height <= 0 || p->width <= 0 ||
      p->out_channels <= 0 || p->kernel_h <= 0 || p->kernel_w <= 0)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn: sizes must be positive");
  if (p->stride_h <= 0 || p->stride_w <= 0 || p->dilation_h <= 0 || p->dilation_w <= 0 ||
      p->pad_h < 0 || p->pad_w < 0)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn: stride/dilation must be > 0 and padding >= 0");
  if (p->groups <= 0 || p->in_channels % p->groups || p->out_channels % p->groups)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn: groups=%d must divide in (%d) and out (%d) channels",
                p->groups, p->in_channels, p->out_channels);
  if (p->deformable_groups <= 0 || p->in_channels % p->deformable_groups)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn: deformable_groups=%d must divide in_channels=%d",
                p->deformable_groups, p->in_channels);
  d->B = p->batch; d->Cin = p->in_channels; d->H = p->height; d->W = p->width;
  d->Cout = p->out_channels; d->kH = p->kernel_h; d->kW = p->kernel_w; d->T = d->kH * d->kW;
  d->sh = p->stride_h; d->sw = p->stride_w; d->ph = p->pad_h; d->pw = p->pad_w;
  d->dh = p->dilation_h; d->dw = p->dilation_w; d->groups = p->groups; d->dg = p->deformable_groups;
  d->Ho = out_size(d->H, d->ph, d->dh, d->kH, d->sh);
  d->Wo = out_size(d->W, d->pw, d->dw, d->kW, d->sw);
  if (d->Ho <= 0 || d->Wo <= 0)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn: empty output (%d x %d)", d->Ho, d->Wo);
  d->Cin_g = d->Cin / d->groups;
  d->Cout_g = d->Cout / d->groups;
  d->Cin_g_pad = (d->Cin_g + 63) / 64 * 64;
  d->cpdg = d->Cin / d->dg;
  d->M = static_cast<int64_t>(d->B) * d->Ho * d->Wo;
  return BEVK_OK;
}

}  // namespace bevk

using namespace bevk;

namespace {

// Largest element offset addressed by a 4-D tensor of the given sizes/strides.
int64_t max_offset(const int64_t sizes[4], const int64_t strides[4]) {
  int64_t o = 0;
  for (int i = 0; i < 4; ++i) {
    if (strides[i] < 0) return -1;
    o += (sizes[i] - 1) * strides[i];
  }
  return o;
}

}  // namespace

namespace bevk {

int validate_dcn_tensors(const bevk_dcn_problem *p, const DcnDims &d) {
  const int T = d.T;
  const int64_t xsz[4] = {d.B, d.Cin, d.H, d.W};
  const int64_t osz[4] = {d.B, 2LL * d.dg * T, d.Ho, d.Wo};
  const int64_t msz[4] = {d.B, static_cast<int64_t>(d.dg) * T, d.Ho, d.Wo};
  const int64_t ysz[4] = {d.B, d.Cout, d.Ho, d.Wo};
  if (max_offset(xsz, p->input_strides) < 0 || max_offset(osz, p->offset_strides) < 0 ||
      max_offset(msz, p->mask_strides) < 0 || max_offset(ysz, p->output_strides) < 0)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn: negative strides are not supported");
  return BEVK_OK;
}

bool input_needs_transpose(const bevk_dcn_problem *p) {
  const int64_t *s = p->input_strides;
  return !(s[1] == 1 && s[0] % 8 == 0 && s[2] % 8 == 0 && s[3] % 8 == 0);
}

}  // namespace bevk

extern "C" {

BEVK_API int bevk_version(void) { return BEVK_VERSION_NUMBER; }

BEVK_API const char *bevk_status_string(int status) {
  switch (status) {
    case BEVK_OK: return "ok";
    case BEVK_ERR_INVALID_ARGUMENT: return "invalid argument";
    case BEVK_ERR_UNSUPPORTED: return "unsupported";
    case BEVK_ERR_INDEX_OVERFLOW: return "index overflow";
    case BEVK_ERR_MISALIGNED: return "misaligned";
    case BEVK_ERR_CUDA: return "cuda error";
    case BEVK_ERR_WORKSPACE: return "workspace too small";
    case BEVK_ERR_DEVICE_TIMEOUT: return "device watchdog timeout";
    default: return "unknown status";
  }
}

BEVK_API const char *bevk_last_error_message(void) { return last_error(); }

BEVK_API int bevk_device_watchdog(int device, unsigned int *code) {
  clear_error();
  return read_and_clear_watchdog(device, code);
}

BEVK_API int bevk_set_wait_limit_ns(int device, unsigned long long ns) {
  clear_error();
  return set_wait_limit(device, ns);
}

// ------------------------------------------------------------------ DCN
BEVK_API int bevk_dcn_output_size(const bevk_dcn_problem *p, int *height_out, int *width_out) {
  clear_error();
  DcnDims d;
  const int st = dcn_dims(p, &d);
  if (st != BEVK_OK) return st;
  if (height_out) *height_out = d.Ho;
  if (width_out) *width_out = d.Wo;
  return BEVK_OK;
}

BEVK_API size_t bevk_dcn_packed_weight_bytes(const bevk_dcn_problem *p) {
  DcnDims d;
  if (dcn_dims(p, &d) != BEVK_OK) return 0;
  return static_cast<size_t>(d.Cout) * d.T * d.Cin_g_pad * dtype_size(p->dtype);
}

BEVK_API int bevk_dcn_pack_weight(const bevk_dcn_problem *p, const void *weight,
                                  void *packed_weight, bevk_stream_t stream) {
  clear_error();
  DcnDims d;
  int st = dcn_dims(p, &d);
  if (st != BEVK_OK) return st;
  if (!weight || !packed_weight) return fail(BEVK_ERR_INVALID_ARGUMENT, "pack_weight: null pointer");
  return launch_dcn_pack_weight(d, weight, packed_weight, p->dtype,
                                reinterpret_cast<cudaStream_t>(stream));
}

// Forward scratch: [NHWC copy of an input that is not channel-contiguous,
// rounded up to 256 bytes][the tensor-core kernel's K-split scratch].
static size_t transpose_bytes(const bevk_dcn_problem *p, const DcnDims &d) {
  if (!input_needs_transpose(p)) return 0;
  return (static_cast<size_t>(d.B) * d.H * d.W * d.Cin * dtype_size(p->dtype) + 255) &
         ~static_cast<size_t>(255);
}

BEVK_API size_t bevk_dcn_forward_workspace_bytes(const bevk_dcn_problem *p) {
  DcnDims d;
  if (dcn_dims(p, &d) != BEVK_OK) return 0;
  if (!dcn_tc_supported(p, d)) return 0;
  return transpose_bytes(p, d) + dcn_tc_workspace_bytes(p, d);
}

BEVK_API int bevk_dcn_offset_conv_sum(const bevk_dcn_problem *p, const bevk_dcn_zoff_args *z,
                                      bevk_stream_t stream) {
  clear_error();
  DcnDims d;
  int st = dcn_dims(p, &d);
  if (st != BEVK_OK) return st;
  if (!z || !z->partials || !z->offset_out)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn_offset_conv_sum: null pointer");
  if (z->partials_ld < 3 * d.T * d.T)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn_offset_conv_sum: partials_ld %lld < 3*T*T",
                static_cast<long long>(z->partials_ld));
  return launch_dcn_offset_sum(p, d, z->partials, z->partials_ld, z->offset_bias, z->offset_out,
                               reinterpret_cast<cudaStream_t>(stream));
}

BEVK_API int bevk_dcn_forward_zoff(const bevk_dcn_problem *p, const bevk_dcn_zoff_args *z,
                                   const void *input, const void *packed_weight,
                                   const void *bias, void *output, bevk_stream_t stream) {
  int st = bevk_dcn_offset_conv_sum(p, z, stream);
  if (st != BEVK_OK) return st;
  DcnDims d;
  dcn_dims(p, &d);
  // offset / mask views of the [B, Ho, Wo, 3T] offset-conv output
  bevk_dcn_problem q = *p;
  const int64_t c3 = 3 * d.T;
  const int64_t ys[4] = {static_cast<int64_t>(d.Ho) * d.Wo * c3, 1,
                         static_cast<int64_t>(d.Wo) * c3, c3};
  for (int i = 0; i < 4; ++i) q.offset_strides[i] = q.mask_strides[i] = ys[i];
  q.mask_is_logit = 1;
  const char *yb = static_cast<const char *>(z->offset_out);
  return bevk_dcn_forward(&q, input, yb, yb + 2 * d.T * dtype_size(p->dtype), packed_weight, bias,
                          output, nullptr, 0, stream);
}

BEVK_API int bevk_dcn_forward(const bevk_dcn_problem *p, const void *input, const void *offset,
                              const void *mask, const void *packed_weight, const void *bias,
                              void *output, void *workspace, size_t workspace_bytes,
                              bevk_stream_t stream) {
  clear_error();
  DcnDims d;
  int st = dcn_dims(p, &d);
  if (st != BEVK_OK) return st;
  if (!input || !offset || !mask || !packed_weight || !output || (p->has_bias && !bias))
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn_forward: null pointer");
  st = validate_dcn_tensors(p, d);
  if (st != BEVK_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool tc = dcn_tc_supported(p, d) && (input_needs_transpose(p) || aligned(input, 16));
  if (tc) {
    const void *x = input;
    int64_t xs[4] = {p->input_strides[0], p->input_strides[1], p->input_strides[2],
                     p->input_strides[3]};
    // the K-split scratch follows the transposed input (optional: without it
    // the kernel takes a schedule that needs none)
    void *tail = workspace;
    size_t tail_bytes = workspace ? workspace_bytes : 0;
    if (input_needs_transpose(p)) {
      const size_t need = static_cast<size_t>(d.B) * d.H * d.W * d.Cin * dtype_size(p->dtype);
      if (!workspace || workspace_bytes < need || !aligned(workspace, 16))
        return fail(BEVK_ERR_WORKSPACE, "dcn_forward: needs a 16-byte aligned workspace of %zu bytes",
                    need);
      const size_t used = transpose_bytes(p, d);
      tail = workspace_bytes > used ? static_cast<char *>(workspace) + used : nullptr;
      tail_bytes = workspace_bytes > used ? workspace_bytes - used : 0;
      st = launch_nchw_to_nhwc(input, workspace, d.B, d.Cin, d.H, d.W, p->input_strides, p->dtype, s);
      if (st != BEVK_OK) return st;
      x = workspace;
      xs[0] = static_cast<int64_t>(d.H) * d.W * d.Cin;
      xs[1] = 1;
      xs[2] = static_cast<int64_t>(d.W) * d.Cin;
      xs[3] = d.Cin;
    }
    st = launch_dcn_forward_tc(p, d, x, xs, offset, mask, packed_weight, bias, output, tail,
                               tail_bytes, s);
    if (st != BEVK_ERR_INDEX_OVERFLOW && st != BEVK_ERR_MISALIGNED) return st;
    clear_error();  // geometry the tensor-core kernel cannot index: exact path below
  }
  return launch_dcn_forward_simt(p, d, input, offset, mask, packed_weight, bias, output, s);
}

static int im2col_common(const void *data_im, const void *data_offset, const void *data_mask,
                         int batch_size, int channels, int height_im, int width_im,
                         int height_col, int width_col, int kernel_h, int kernel_w, int pad_h,
                         int pad_w, int stride_h, int stride_w, int dilation_h, int dilation_w,
                         int deformable_group, int offset_last_dim, void *data_col, int dtype,
                         int layout, bevk_stream_t stream) {
  clear_error();
  bevk_dcn_problem p;
  std::memset(&p, 0, sizeof(p));
  p.dtype = dtype;
  p.batch = batch_size; p.in_channels = channels; p.height = height_im; p.width = width_im;
  p.out_channels = 1; p.kernel_h = kernel_h; p.kernel_w = kernel_w;
  p.stride_h = stride_h; p.stride_w = stride_w; p.pad_h = pad_h; p.pad_w = pad_w;
  p.dilation_h = dilation_h; p.dilation_w = dilation_w;
  p.groups = 1; p.deformable_groups = deformable_group;
  DcnDims d;
  int st = dcn_dims(&p, &d);
  if (st != BEVK_OK) return st;
  if (d.Ho != height_col || d.Wo != width_col)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "im2col: height_col/width_col (%d x %d) do not match "
                "the convolution geometry (%d x %d)", height_col, width_col, d.Ho, d.Wo);
  if (!data_im || !data_offset || !data_col || (!data_mask && offset_last_dim != 3 * d.T))
    return fail(BEVK_ERR_INVALID_ARGUMENT, "im2col: null pointer");
  const int64_t HW = static_cast<int64_t>(d.H) * d.W, HoWo = static_cast<int64_t>(d.Ho) * d.Wo;
  const void *mask_ptr = data_mask;
  if (layout == 0) {  // NCHW tensors
    const int64_t xs[4] = {d.Cin * HW, HW, d.W, 1};
    const int64_t os[4] = {2LL * d.dg * d.T * HoWo, HoWo, d.Wo, 1};
    const int64_t ms[4] = {static_cast<int64_t>(d.dg) * d.T * HoWo, HoWo, d.Wo, 1};
    std::memcpy(p.input_strides, xs, sizeof(xs));
    std::memcpy(p.offset_strides, os, sizeof(os));
    std::memcpy(p.mask_strides, ms, sizeof(ms));
  } else {  // NHWC tensors
    if (deformable_group != 1)
      return fail(BEVK_ERR_UNSUPPORTED, "NHWC im2col supports deformable_group == 1 only");
    if (offset_last_dim != 2 * d.T && offset_last_dim != 3 * d.T)
      return fail(BEVK_ERR_INVALID_ARGUMENT, "NHWC im2col: offset last dim %d must be 2T or 3T (T=%d)",
                  offset_last_dim, d.T);
    const int64_t xs[4] = {HW * d.Cin, 1, static_cast<int64_t>(d.W) * d.Cin, d.Cin};
    const int64_t os[4] = {HoWo * offset_last_dim, 1, static_cast<int64_t>(d.Wo) * offset_last_dim,
                           offset_last_dim};
    std::memcpy(p.input_strides, xs, sizeof(xs));
    std::memcpy(p.offset_strides, os, sizeof(os));
    if (offset_last_dim == 3 * d.T) {  // raw offset-conv output: pre-sigmoid mask in [2T, 3T)
      std::memcpy(p.mask_strides, os, sizeof(os));
      mask_ptr = static_cast<const char *>(data_offset) + 2LL * d.T * dtype_size(dtype);
      p.mask_is_logit = 1;
    } else {
      const int64_t ms[4] = {HoWo * d.T, 1, static_cast<int64_t>(d.Wo) * d.T, d.T};
      std::memcpy(p.mask_strides, ms, sizeof(ms));
    }
  }
  return launch_dcn_im2col(&p, d, data_im, data_offset, mask_ptr, data_col, layout,
                           reinterpret_cast<cudaStream_t>(stream));
}

BEVK_API int bevk_modulated_deformable_im2col(
    const void *data_im, const void *data_offset, const void *data_mask, int batch_size,
    int channels, int height_im, int width_im, int height_col, int width_col, int kernel_h,
    int kernel_w, int pad_h, int pad_w, int stride_h, int stride_w, int dilation_h,
    int dilation_w, int deformable_group, void *data_col, int dtype, bevk_stream_t stream) {
  return im2col_common(data_im, data_offset, data_mask, batch_size, channels, height_im,
                       width_im, height_col, width_col, kernel_h, kernel_w, pad_h, pad_w,
                       stride_h, stride_w, dilation_h, dilation_w, deformable_group, 0, data_col,
                       dtype, 0, stream);
}

BEVK_API int bevk_modulated_deformable_im2col_opt(
    const void *data_im, const void *data_offset, const void *data_mask, int batch_size,
    int channels, int height_im, int width_im, int height_col, int width_col, int kernel_h,
    int kernel_w, int pad_h, int pad_w, int stride_h, int stride_w, int dilation_h,
    int dilation_w, int deformable_group, void *data_col, int dtype, bevk_stream_t stream) {
  return im2col_common(data_im, data_offset, data_mask, batch_size, channels, height_im,
                       width_im, height_col, width_col, kernel_h, kernel_w, pad_h, pad_w,
                       stride_h, stride_w, dilation_h, dilation_w, deformable_group, 0, data_col,
                       dtype, 0, stream);
}

BEVK_API int bevk_modulated_deformable_im2col_nhwc(
    const void *data_im, const void *data_offset, const void *data_mask, int batch_size,
    int channels, int height_im, int width_im, int height_col, int width_col, int kernel_h,
    int kernel_w, int pad_h, int pad_w, int stride_h, int stride_w, int dilation_h,
    int dilation_w, int deformable_group, int offset_last_dim, void *data_col, int dtype,
    bevk_stream_t stream) {
  return im2col_common(data_im, data_offset, data_mask, batch_size, channels, height_im,
                       width_im, height_col, width_col, kernel_h, kernel_w, pad_h, pad_w,
                       stride_h, stride_w, dilation_h, dilation_w, deformable_group,
                       offset_last_dim, data_col, dtype, 1, stream);
}

// ------------------------------------------------------------------ MSDA
BEVK_API int bevk_ms_deform_attn_forward(const void *value, const int64_t *spatial_shapes,
                                         const int64_t *level_start_index,
                                         const void *sampling_loc, const void *attention_weights,
                                         int batch, int spatial_size, int num_heads,
                                         int channels, int num_levels, int num_query,
                                         int num_point, int im2col_step, void *output, int dtype,
                                         bevk_stream_t stream) {
  clear_error();
  // the per-query arrays are empty (and may be NULL) when num_query == 0
  if (!value || !spatial_shapes || !level_start_index ||
      (num_query != 0 && (!sampling_loc || !attention_weights || !output)))
    return fail(BEVK_ERR_INVALID_ARGUMENT, "ms_deform_attn_forward: null pointer");
  if (batch <= 0 || spatial_size <= 0 || num_heads <= 0 || channels <= 0 || num_levels <= 0 ||
      num_query < 0 || num_point <= 0)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "ms_deform_attn_forward: sizes must be positive");
  if (im2col_step <= 0) return fail(BEVK_ERR_INVALID_ARGUMENT, "im2col_step must be positive");
  const int step = batch < im2col_step ? batch : im2col_step;
  if (batch % step != 0)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "batch must divide im2col_step (batch=%d, step=%d)",
                batch, step);
  if (static_cast<int64_t>(spatial_size) * num_heads >= (int64_t(1) << 31) / 2)
    return fail(BEVK_ERR_INDEX_OVERFLOW, "ms_deform_attn_forward: spatial_size*heads too large");
  return launch_msda_forward(value, spatial_shapes, level_start_index, sampling_loc,
                             attention_weights, batch, spatial_size, num_heads, channels,
                             num_levels, num_query, num_point, output, dtype,
                             reinterpret_cast<cudaStream_t>(stream));
}

BEVK_API int bevk_dcn_columns(const bevk_dcn_problem *p, const void *input,
                              const void *offset, const void *mask, void *col, int layout,
                              bevk_stream_t stream) {
  clear_error();
  if (!p || !input || !offset || !mask || !col)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn_columns: null pointer");
  if (layout != 0 && layout != 1)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn_columns: layout must be 0 or 1");
  bevk_dcn_problem pr = *p;
  pr.out_channels = 1;
  pr.groups = 1;
  DcnDims d;
  const int st = dcn_dims(&pr, &d);
  if (st != BEVK_OK) return st;
  if (d.M == 0) return BEVK_OK;
  return launch_dcn_im2col(&pr, d, input, offset, mask, col, layout,
                           reinterpret_cast<cudaStream_t>(stream));
}

BEVK_API int bevk_dcn_col2im(const bevk_dcn_col2im_args *args, const void *input,
                             const void *offset, const void *mask, const void *dcol,
                             void *grad_input, void *grad_offset, void *grad_mask,
                             bevk_stream_t stream) {
  clear_error();
  if (!args || !offset || !mask || !dcol)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn_col2im: null pointer");
  if (!input && (grad_offset || grad_mask))
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn_col2im: grad_offset / grad_mask need the input");
  // out_channels and groups play no part in the scatter
  bevk_dcn_problem pr = args->problem;
  pr.out_channels = 1;
  pr.groups = 1;
  DcnDims d;
  const int st = dcn_dims(&pr, &d);
  if (st != BEVK_OK) return st;
  if (args->col_dtype != args->problem.dtype && args->col_dtype != BEVK_DTYPE_F32)
    return fail(BEVK_ERR_UNSUPPORTED, "dcn_col2im: column dtype must be the input dtype or f32");
  if (!grad_input && !grad_offset && !grad_mask) return BEVK_OK;
  return launch_dcn_col2im(args, d, input, offset, mask, dcol, grad_input, grad_offset,
                           grad_mask, reinterpret_cast<cudaStream_t>(stream));
}

BEVK_API size_t bevk_dcn_backward_data_workspace_bytes(const bevk_dcn_problem *p) {
  if (!p) return 0;
  bevk_dcn_problem pr = *p;
  pr.out_channels = 1;
  pr.groups = 1;
  DcnDims d;
  if (dcn_dims(&pr, &d) != BEVK_OK) return 0;
  return dcn_backward_data_workspace_bytes(d);
}

BEVK_API int bevk_dcn_backward_data(const bevk_dcn_backward_data_args *args,
                                    const void *input, const void *offset, const void *mask,
                                    const void *dcol, void *grad_input, void *grad_offset,
                                    void *grad_mask, void *col, void *workspace,
                                    size_t workspace_bytes, bevk_stream_t stream) {
  clear_error();
  if (!args || !offset || !mask)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn_backward_data: null pointer");
  if (!input && (grad_offset || grad_mask || col))
    return fail(BEVK_ERR_INVALID_ARGUMENT,
                "dcn_backward_data: grad_offset / grad_mask / col need the input");
  if (!dcol && (grad_input || grad_offset || grad_mask))
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn_backward_data: the gradients need dcol");
  // out_channels and groups play no part in the data side
  bevk_dcn_problem pr = args->problem;
  pr.out_channels = 1;
  pr.groups = 1;
  DcnDims d;
  const int st = dcn_dims(&pr, &d);
  if (st != BEVK_OK) return st;
  if (!grad_input && !grad_offset && !grad_mask && !col) return BEVK_OK;
  return launch_dcn_backward_data(args, d, input, offset, mask, dcol, grad_input, grad_offset,
                                  grad_mask, col, workspace, workspace_bytes,
                                  reinterpret_cast<cudaStream_t>(stream));
}

BEVK_API size_t bevk_ms_deform_attn_backward_workspace_bytes(int batch, int spatial_size,
                                                             int num_heads, int channels,
                                                             int dtype) {
  return msda_backward_workspace_bytes(batch, spatial_size, num_heads, channels, dtype);
}

BEVK_API int bevk_ms_deform_attn_backward(const void *value, const int64_t *spatial_shapes,
                                          const int64_t *level_start_index,
                                          const void *sampling_loc,
                                          const void *attention_weights, const void *grad_output,
                                          int batch, int spatial_size, int num_heads,
                                          int channels, int num_levels, int num_query,
                                          int num_point, int im2col_step, void *grad_value,
                                          void *grad_sampling_loc, void *grad_attention_weights,
                                          void *workspace, size_t workspace_bytes, int dtype,
                                          bevk_stream_t stream) {
  clear_error();
  // the per-query arrays are empty (and may be NULL) when num_query == 0
  const bool per_query_ok = num_query == 0 || (sampling_loc && attention_weights && grad_output &&
                                               grad_sampling_loc && grad_attention_weights);
  if (!value || !spatial_shapes || !level_start_index || !grad_value || !per_query_ok)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "ms_deform_attn_backward: null pointer");
  if (batch <= 0 || spatial_size <= 0 || num_heads <= 0 || channels <= 0 || num_levels <= 0 ||
      num_query < 0 || num_point <= 0)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "ms_deform_attn_backward: sizes must be positive");
  if (im2col_step <= 0) return fail(BEVK_ERR_INVALID_ARGUMENT, "im2col_step must be positive");
  const int step = batch < im2col_step ? batch : im2col_step;
  if (batch % step != 0)
    return fail(BEVK_ERR_INVALID_ARGUMENT, "batch must divide im2col_step (batch=%d, step=%d)",
                batch, step);
  if (static_cast<int64_t>(spatial_size) * num_heads >= (int64_t(1) << 31) / 2)
    return fail(BEVK_ERR_INDEX_OVERFLOW, "ms_deform_attn_backward: spatial_size*heads too large");
  return launch_msda_backward(value, spatial_shapes, level_start_index, sampling_loc,
                              attention_weights, grad_output, grad_value, grad_sampling_loc,
                              grad_attention_weights, batch, spatial_size, num_heads, channels,
                              num_levels, num_query, num_point, workspace, workspace_bytes, dtype,
                              reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
