/*
 * bevk.h -- C ABI of the B200 (sm_100a) deformable-sampling kernels.
 *
 * Plain pointers, sizes and strides; no torch types.  Every entry point
 *   - takes device pointers that it borrows for the duration of the call,
 *   - never allocates or frees device memory (scratch comes from the caller
 *     through an explicit workspace argument),
 *   - enqueues its kernels asynchronously on the given stream (NULL = the
 *     legacy default stream) of the current CUDA device,
 *   - returns BEVK_OK or a negative status; bevk_last_error_message() then
 *     holds a human-readable reason for the calling thread.
 *
 * Shapes follow the reference operator surface (naotic/bev-kernels):
 *   DCNv2:  input [B, Cin, H, W], offset [B, 2*dg*kH*kW, Ho, Wo] with channel
 *           2t = dh and 2t+1 = dw of tap t = ki*kW + kj, mask [B, dg*kH*kW, Ho, Wo],
 *           weight [Cout, Cin/groups, kH, kW], output [B, Cout, Ho, Wo].
 *           Any of them may be channels-last; strides describe the layout.
 *   MSDA:   value [B, S, heads, C], spatial_shapes [L, 2] int64 (H, W),
 *           level_start_index [L] int64, sampling_loc [B, Q, heads, L, P, 2]
 *           (x then y, normalised to [0, 1]), attention_weights [B, Q, heads, L, P],
 *           output [B, Q, heads*C].
 */
#ifndef BEVK_H_
#define BEVK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define BEVK_API
#else
#define BEVK_API __attribute__((visibility("default")))
#endif

/* Same underlying type as cudaStream_t / CUstream. */
typedef struct CUstream_st *bevk_stream_t;

/* Element types. */
enum bevk_dtype {
  BEVK_DTYPE_F32 = 0,
  BEVK_DTYPE_F16 = 1,
  BEVK_DTYPE_BF16 = 2,
  BEVK_DTYPE_F64 = 3
};

/* Status codes (0 = success). */
enum bevk_status {
  BEVK_OK = 0,
  BEVK_ERR_INVALID_ARGUMENT = -1, /* null pointer, bad shape, bad stride     */
  BEVK_ERR_UNSUPPORTED = -2,      /* dtype / geometry this build cannot run */
  BEVK_ERR_INDEX_OVERFLOW = -3,   /* tensor too large for 32-bit indexing   */
  BEVK_ERR_MISALIGNED = -4,       /* pointer/stride alignment requirement   */
  BEVK_ERR_CUDA = -5,             /* CUDA runtime / launch failure          */
  BEVK_ERR_WORKSPACE = -6,        /* workspace missing or too small         */
  BEVK_ERR_DEVICE_TIMEOUT = -7    /* a kernel's bounded wait gave up        */
};

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
BEVK_API int bevk_version(void);
/* Static description of a status code. */
BEVK_API const char *bevk_status_string(int status);
/* Detail of the most recent failure on the calling thread ("" if none). */
BEVK_API const char *bevk_last_error_message(void);

/*
 * Device-side watchdog.  Kernels that wait on barriers bound every wait; a
 * wait that gives up records a nonzero code in a per-device word instead of
 * hanging.  This call synchronises the given device, returns the word in
 * *code (0 = clean) and clears it.  Returns BEVK_ERR_DEVICE_TIMEOUT when the
 * word was set, BEVK_OK otherwise.
 */
BEVK_API int bevk_device_watchdog(int device, unsigned int *code);

/*
 * Diagnostics, no counterpart in the reference: sets the time limit of the
 * fused DCN forward kernel's pipeline barrier waits on `device` to `ns`
 * nanoseconds (0 restores the default, 2 s).  The teardown waits that drain
 * tensor-core work and copies before a CTA releases its memory keep the
 * default.  With a short limit, launches give up mid-pipeline: the kernel
 * unwinds, writes no output and records the site in the watchdog word above.
 * For tests of that path.  Applies to launches made after the call.
 */
BEVK_API int bevk_set_wait_limit_ns(int device, unsigned long long ns);

/*
 * Launch order.  The library's kernels are launched as programmatic
 * dependents of the stream's previous kernel: their set-up (barriers, tensor
 * memory, descriptor prefetch) may overlap that kernel's last CTAs, and each
 * waits for it to complete before reading or writing global memory, so stream
 * order holds as with ordinary launches.  Setting the environment variable
 * BEVK_PDL=0 (read once per process) launches them the ordinary way.
 */

/* ------------------------------------------------------------------------ */
/* DCNv2 (modulated deformable convolution), forward                        */
/* ------------------------------------------------------------------------ */

/*
 * Problem description shared by the DCN entry points.  Strides are element
 * strides in (b, c, h, w) order for each 4-D tensor; output spatial size is
 * derived as (in + 2*pad - (dil*(k-1)+1)) / stride + 1.
 */
typedef struct bevk_dcn_problem {
  int dtype;                 /* enum bevk_dtype; all tensors share it        */
  int batch, in_channels, height, width;
  int out_channels, kernel_h, kernel_w;
  int stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w;
  int groups, deformable_groups;
  int64_t input_strides[4];
  int64_t offset_strides[4];
  int64_t mask_strides[4];
  int64_t output_strides[4];
  int mask_is_logit;         /* 1: mask holds pre-sigmoid values; sigmoid is
                                applied on load (the fused offset-conv output
                                path of dcn_split_nhwc.py:159-174)             */
  int has_bias;
  int act_relu;              /* 1: output = max(0, conv + bias), the ReLU of a
                                FrozenBN+ReLU epilogue whose affine is folded
                                into weight and bias (dcn_split_nhwc.py:185-199) */
} bevk_dcn_problem;

/* Output height/width of a problem (BEVK_ERR_INVALID_ARGUMENT if <= 0). */
BEVK_API int bevk_dcn_output_size(const bevk_dcn_problem *p, int *height_out,
                                  int *width_out);

/*
 * Packed weight layout used by bevk_dcn_forward: [Cout][kH*kW][Cin_g_pad] in
 * the problem dtype, Cin_g = Cin/groups rounded up to a multiple of 64 with
 * zeros, so every output channel's reduction row is tap-major and contiguous.
 * Packing is a one-off per weight update (the reference re-packs on every
 * call: dcn_split_nhwc.py:176).
 */
BEVK_API size_t bevk_dcn_packed_weight_bytes(const bevk_dcn_problem *p);
/* weight: [Cout, Cin/groups, kH, kW] contiguous. */
BEVK_API int bevk_dcn_pack_weight(const bevk_dcn_problem *p, const void *weight,
                                  void *packed_weight, bevk_stream_t stream);

/*
 * Scratch bytes for bevk_dcn_forward on this problem (0 when none): an NHWC
 * copy of an input that is not channel-contiguous (required), followed by the
 * tensor-core kernel's K-split scratch (optional: problems with more than 256
 * output channels that fill at most one wave of the GPU split their K loop in
 * two when it is given; with less workspace they run unsplit).  256-byte
 * aligned workspace; its contents need no initialisation.
 */
BEVK_API size_t bevk_dcn_forward_workspace_bytes(const bevk_dcn_problem *p);

/*
 * Fused DCNv2 forward: output = conv(weight, deformable-bilinear(input,
 * offset) * mask) + bias, without materialising the column matrix.
 *
 * Replaces ModulatedDeformConv2dFunction.forward
 * (modulated_deform_conv/modulated_deform_conv.py:331-403: im2col_opt + torch.mm
 * + permute + bias) and the gather + GEMM of DCNSplitNHWCFunction.forward
 * (modulated_deform_conv/dcn_split_nhwc.py:159-203).
 *
 * fp16/bf16 with groups == 1, deformable_groups == 1, Cin % 8 == 0 and
 * kH*kW <= 9 run the tcgen05 tensor-core kernel (fp32 accumulation in TMEM);
 * every other case (fp32, fp64, grouped, ...) runs the exact SIMT kernel.
 * bias may be NULL when has_bias == 0.
 */
BEVK_API int bevk_dcn_forward(const bevk_dcn_problem *p, const void *input,
                              const void *offset, const void *mask,
                              const void *packed_weight, const void *bias,
                              void *output, void *workspace,
                              size_t workspace_bytes, bevk_stream_t stream);

/*
 * The offset convolution of the DCNv2 Pack module from its per-tap partial
 * products.  T = kernel_h * kernel_w, P = batch * height * width (input pixels
 * in NHWC order).
 */
typedef struct bevk_dcn_zoff_args {
  const float *partials;     /* [P][partials_ld] fp32: partials[p*ld + t*3T + c]
                                = sum_ci input[p, ci] * w_off[c, ci, t]        */
  int64_t partials_ld;       /* row stride in elements, >= T * 3T             */
  const float *offset_bias;  /* [3T] fp32 (the offset conv's bias) or NULL    */
  void *offset_out;          /* [batch*Ho*Wo][3T] contiguous, problem dtype:
                                the offset-conv output                        */
} bevk_dcn_zoff_args;

/*
 * Offset convolution of the Pack module (conv_offset of
 * DCNSplitNHWCFunction.forward, modulated_deform_conv/dcn_split_nhwc.py:171-172,
 * and of ModulatedDeformConv2dPack, modulated_deform_conv.py:604-626): the
 * DCN's kernel size, stride, padding and dilation, 3T output channels --
 * channel c < 2T is offset channel c (2t = dh, 2t+1 = dw of tap t), channel
 * 2T + t the mask logit of tap t.  The reference runs it as a cuDNN
 * convolution; its fused offset-conv + gather kernel
 * (csrc/dcn_fused_nhwc_kernel.cuh:211-303, bound at csrc/binding.cpp:167-169)
 * and the TileLang mega-kernel (modulated_deform_conv/fused_tl.py:565-688)
 * compute it in-kernel.
 *
 * Here its channel reduction is one plain GEMM the caller runs ([P, Cin] x
 * [Cin, T*3T] with fp32 output: partials); this call adds the T shifted taps
 * and offset_bias for every output pixel and rounds the sum to the problem
 * dtype (what the unfused offset-conv output holds), writing offset_out.
 * (Summing the taps in the DCN kernel's prologue instead measured slower on
 * B200: the extra L2 round trips sit on every tile's critical path.)
 * fp16, bf16 and fp32; kH*kW <= 9.  Only the shape, stride, padding,
 * dilation and dtype fields of the problem are used.
 */
BEVK_API int bevk_dcn_offset_conv_sum(const bevk_dcn_problem *p, const bevk_dcn_zoff_args *z,
                                      bevk_stream_t stream);

/*
 * bevk_dcn_offset_conv_sum followed by bevk_dcn_forward on its output (offsets
 * from offset_out channels [0, 2T), the mask sigmoid applied on load to
 * channels [2T, 3T)).  The problem's offset_strides, mask_strides and
 * mask_is_logit are ignored; input must not need the NCHW copy of
 * bevk_dcn_forward (no workspace is taken).
 */
BEVK_API int bevk_dcn_forward_zoff(const bevk_dcn_problem *p, const bevk_dcn_zoff_args *z,
                                   const void *input, const void *packed_weight,
                                   const void *bias, void *output, bevk_stream_t stream);

/*
 * Allocation-free variant of bevk_dcn_forward.  No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc or hand out a
 * workspace at the moment they run the layer -- an inference engine's plugin
 * whose enqueue step may not allocate and was promised no workspace, or a
 * runtime that freezes device memory after start-up for determinism.
 *
 * Takes the unpacked weight [Cout, Cin/groups, kH, kW] (contiguous) and does
 * the weight packing and, for NCHW input on the tensor-core path, the NHWC
 * copy of the input inside a fixed scratch array that the library itself
 * holds in device memory: BEVK_DCN_NOALLOC_SCRATCH_BYTES per GPU on which the
 * library's code is loaded, kept until the process exits.  Problems needing
 * more than that (packed weight, rounded up to 256 bytes, plus the input copy
 * when one is needed) return BEVK_ERR_WORKSPACE without launching anything.
 *
 * The first call on a device looks up the array's device address (once per
 * device, with that device current); make that first call before capturing
 * a stream into a CUDA graph -- a first call made during a capture returns
 * BEVK_ERR_CUDA without touching the stream.  All calls on a device share the one array and
 * its contents persist between calls (nothing in it needs to start at zero):
 * calls whose kernels can overlap on the GPU -- different streams without
 * ordering between them -- race on it, so serialise them.
 */
#define BEVK_DCN_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)
BEVK_API int bevk_dcn_forward_noalloc(const bevk_dcn_problem *p, const void *input,
                                      const void *offset, const void *mask,
                                      const void *weight, const void *bias, void *output,
                                      bevk_stream_t stream);

/*
 * Column-matrix ops of the reference extension (binding names kept).
 *
 * bevk_modulated_deformable_im2col / _opt replace
 *   modulated_deformable_im2col_cuda      (csrc/binding.cpp:5-11, :143-145)
 *   modulated_deformable_im2col_opt_cuda  (csrc/binding.cpp:21-27, :149-151)
 * NCHW contiguous input/offset/mask; data_col is the [C*kH*kW, B*Ho*Wo] matrix
 * (row c*kH*kW + t).  Every element is written.
 */
BEVK_API int bevk_modulated_deformable_im2col(
    const void *data_im, const void *data_offset, const void *data_mask,
    int batch_size, int channels, int height_im, int width_im, int height_col,
    int width_col, int kernel_h, int kernel_w, int pad_h, int pad_w,
    int stride_h, int stride_w, int dilation_h, int dilation_w,
    int deformable_group, void *data_col, int dtype, bevk_stream_t stream);

BEVK_API int bevk_modulated_deformable_im2col_opt(
    const void *data_im, const void *data_offset, const void *data_mask,
    int batch_size, int channels, int height_im, int width_im, int height_col,
    int width_col, int kernel_h, int kernel_w, int pad_h, int pad_w,
    int stride_h, int stride_w, int dilation_h, int dilation_w,
    int deformable_group, void *data_col, int dtype, bevk_stream_t stream);

/*
 * replaces modulated_deformable_im2col_nhwc_cuda (csrc/binding.cpp:61-67,
 * :163-165; launcher csrc/dcn_fused_nhwc_cuda.cu:27-87).
 * data_im [B, H, W, C]; data_offset [B, Ho, Wo, offset_last_dim] where
 * offset_last_dim is 2*kH*kW (offset only; data_mask is [B, Ho, Wo, kH*kW]
 * post-sigmoid) or 3*kH*kW (the raw offset-conv output y: offsets in
 * [0, 2T), pre-sigmoid mask in [2T, 3T); data_mask is ignored).
 * data_col is [B*Ho*Wo, kH*kW*C] with k = t*C + c.  deformable_group must
 * be 1 (as in the reference).
 */
BEVK_API int bevk_modulated_deformable_im2col_nhwc(
    const void *data_im, const void *data_offset, const void *data_mask,
    int batch_size, int channels, int height_im, int width_im, int height_col,
    int width_col, int kernel_h, int kernel_w, int pad_h, int pad_w,
    int stride_h, int stride_w, int dilation_h, int dilation_w,
    int deformable_group, int offset_last_dim, void *data_col, int dtype,
    bevk_stream_t stream);

/*
 * Deformable column matrix of a problem with any input / offset / mask
 * strides (problem fields as for bevk_dcn_forward; out_channels, groups,
 * output_strides and has_bias unused): layout 0 writes the reference's
 * [C*kH*kW, M] matrix (modulated_deform_conv.py:370), layout 1 the NHWC
 * matrix [M, kH*kW*C] with k = t*C + c (dcn_split_nhwc.py:21-45).  Every
 * element is written.  Used for the weight gradient of the backward.
 */
BEVK_API int bevk_dcn_columns(const bevk_dcn_problem *p, const void *input,
                              const void *offset, const void *mask, void *col,
                              int layout, bevk_stream_t stream);

/* ------------------------------------------------------------------------ */
/* DCNv2 backward: column scatter                                           */
/* ------------------------------------------------------------------------ */

/*
 * Arguments of bevk_dcn_col2im.  `problem` gives the geometry, the input /
 * offset / mask dtype and strides and mask_is_logit (out_channels, groups,
 * output_strides and has_bias are not used).  The column gradient dcol holds
 * element (pixel m, input channel c, tap t) at
 *   dcol[m*col_strides[0] + c*col_strides[1] + t*col_strides[2]],
 * m = (b*Ho + oh)*Wo + ow, t = ki*kW + kj; its dtype is the problem dtype or
 * BEVK_DTYPE_F32.  The reference's NCHW column matrix [C*kH*kW, B*Ho*Wo]
 * (modulated_deform_conv.py:444-451) has col_strides {1, kH*kW*M, M}; the NHWC
 * matrix [M, kH*kW*C] of dcn_split_nhwc.py:200 has {kH*kW*C, 1, C}.  Gradient
 * strides are element strides (b, channel, h, w) of the fp32 gradient
 * buffers (fp64 for fp64 problems).
 */
typedef struct bevk_dcn_col2im_args {
  bevk_dcn_problem problem;
  int col_dtype;
  int64_t col_strides[3];
  int64_t grad_input_strides[4];
  int64_t grad_offset_strides[4];
  int64_t grad_mask_strides[4];
} bevk_dcn_col2im_args;

/*
 * replaces modulated_deformable_col2im[_opt|_smem]_cuda,
 * modulated_deformable_col2im_coord[_opt]_cuda and the NHWC col2im family
 * (csrc/binding.cpp:13-62, :80-140; used by ModulatedDeformConv2dFunction.
 * backward, modulated_deform_conv.py:405-499, and col2im_nhwc,
 * dcn_split_nhwc.py:48-120).  ACCUMULATES, as the reference's atomics do:
 *   grad_input  [b, c, h, w]        += dcol * mask * (bilinear corner weight)
 *   grad_offset [b, 2*(gi*T+t)+{0,1}, oh, ow] += mask * sum_c dcol * d(bilinear)/d(h, w)
 *   grad_mask   [b, gi*T+t, oh, ow] += sum_c dcol * bilinear   (* sigmoid'(z)
 *                                       when mask_is_logit)
 * Any of grad_input / grad_offset / grad_mask may be NULL to skip it; input
 * may be NULL when only grad_input is wanted (the corner values feed only the
 * coordinate gradients).
 * Samples outside the bilinear gate contribute nothing.  grad_input uses
 * floating-point atomics (last bits vary between runs, as in the reference).
 */
BEVK_API int bevk_dcn_col2im(const bevk_dcn_col2im_args *args, const void *input,
                             const void *offset, const void *mask, const void *dcol,
                             void *grad_input, void *grad_offset, void *grad_mask,
                             bevk_stream_t stream);

/* ------------------------------------------------------------------------ */
/* DCNv2 backward: data side in one call, without floating-point atomics    */
/* ------------------------------------------------------------------------ */

/*
 * Arguments of bevk_dcn_backward_data.  `problem` as for bevk_dcn_col2im
 * (geometry, dtype f32 / f16 / bf16, input / offset / mask strides,
 * mask_is_logit).  dcol and col are NHWC column matrices [M, kH*kW*C]
 * (element (m, t*C + c) at m*ld + t*C + c, m = (b*Ho + oh)*Wo + ow) in the
 * problem dtype with row strides dcol_ld / col_ld.  The three gradients are
 * stored in grad_dtype (the problem dtype or BEVK_DTYPE_F32) with the given
 * element strides (b, channel, h, w).
 */
typedef struct bevk_dcn_backward_data_args {
  bevk_dcn_problem problem;
  int grad_dtype;
  int64_t dcol_ld;
  int64_t col_ld;
  int64_t grad_input_strides[4];
  int64_t grad_offset_strides[4];
  int64_t grad_mask_strides[4];
} bevk_dcn_backward_data_args;

/* Device workspace bytes bevk_dcn_backward_data needs when grad_input is
 * requested (destination buckets of the samples' corners); 0 otherwise. */
BEVK_API size_t bevk_dcn_backward_data_workspace_bytes(const bevk_dcn_problem *p);

/*
 * replaces the data side of the backward -- col2im_nhwc + col2im_coord_nhwc +
 * im2col_nhwc (csrc/binding.cpp:63-140) as DCNSplitNHWCFunction.backward runs
 * them (dcn_split_nhwc.py:231-291, col2im_nhwc :48-120) and the col2im /
 * col2im_coord / im2col calls of ModulatedDeformConv2dFunction.backward
 * (modulated_deform_conv.py:405-499) -- for channel-contiguous input, column
 * and grad_input layouts.  WRITES (does not accumulate):
 *   grad_input  [b, c, h, w] = sum of dcol * mask * (bilinear corner weight)
 *                over the samples whose in-range corners include (h, w)
 *                (0 where none lands)
 *   grad_offset, grad_mask    the values bevk_dcn_col2im adds
 *   col[m, t*C + c]           = mask * bilinear(input), the columns of the
 *                grad_weight GEMM (f32 / bf16: bit-identical to bevk_dcn_columns
 *                layout 1; f16: built as bevk_dcn_forward builds its tiles,
 *                fp16 corner weights and packed half2 FMAs)
 * Any of grad_input / grad_offset / grad_mask / col may be NULL to skip it;
 * input may be NULL when only grad_input is wanted, dcol when only col is.
 * grad_input is summed in registers per destination after a counting sort of
 * the samples' corners (the workspace), not by atomics; the summation order
 * inside a destination follows the sort's integer atomics, so its last bits
 * may vary between runs.  Layouts: input channel stride 1 (when read),
 * grad_input channel stride 1, C / (C / deformable_groups) / the row strides
 * whole 16-byte vectors, 16-byte-aligned pointers; otherwise
 * BEVK_ERR_UNSUPPORTED.  Sizes: M * dcol_ld below 2^32, one input image
 * below 2^31 elements, 4 * M * deformable_groups * kH * kW below 2^31;
 * otherwise BEVK_ERR_INDEX_OVERFLOW.  (bevk_dcn_col2im + bevk_dcn_columns
 * cover any layout and size.)
 */
BEVK_API int bevk_dcn_backward_data(const bevk_dcn_backward_data_args *args,
                                    const void *input, const void *offset, const void *mask,
                                    const void *dcol, void *grad_input, void *grad_offset,
                                    void *grad_mask, void *col, void *workspace,
                                    size_t workspace_bytes, bevk_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Multi-scale deformable attention, forward                                */
/* ------------------------------------------------------------------------ */

/*
 * replaces _msda_opt2_musa.forward (csrc_musa/msda/binding_musa.mu:286-412,
 * :546-549) / ms_deform_attn_forward
 * (msda_musa_opt2/msda_musa_opt2/dispatch.py:15-35).
 * All tensors contiguous; spatial_shapes / level_start_index are device
 * int64 arrays.  im2col_step keeps the reference's contract
 * (batch % min(batch, im2col_step) == 0, else BEVK_ERR_INVALID_ARGUMENT)
 * but the whole batch runs in one launch.  value, sampling_loc,
 * attention_weights and output share dtype (f32, f16 or bf16; f16/bf16
 * accumulate in fp32).  Every output element is written.  num_query may be 0
 * (sampling_loc, attention_weights and output are then empty and may be
 * NULL).
 */
BEVK_API int bevk_ms_deform_attn_forward(
    const void *value, const int64_t *spatial_shapes,
    const int64_t *level_start_index, const void *sampling_loc,
    const void *attention_weights, int batch, int spatial_size, int num_heads,
    int channels, int num_levels, int num_query, int num_point,
    int im2col_step, void *output, int dtype, bevk_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Multi-scale deformable attention, backward                               */
/* ------------------------------------------------------------------------ */

/*
 * Bytes of device workspace bevk_ms_deform_attn_backward needs: 0 for f32;
 * batch*spatial_size*num_heads*channels*4 for f16/bf16 (the fp32 grad_value
 * accumulator, binding_musa.mu:450-507).
 */
BEVK_API size_t bevk_ms_deform_attn_backward_workspace_bytes(int batch, int spatial_size,
                                                             int num_heads, int channels,
                                                             int dtype);

/*
 * replaces _msda_opt2_musa.backward (csrc_musa/msda/binding_musa.mu:414-543,
 * :550-556) / ms_deform_attn_backward (msda_musa_opt2/msda_musa_opt2/
 * dispatch.py:38-69).  Same inputs as the forward plus grad_output
 * [batch, num_query, num_heads*channels]; all contiguous, one dtype.
 *   f32:      grad_value is ACCUMULATED into (the reference's callers pass
 *             zeros); workspace may be NULL.
 *   f16/bf16: grad_value is accumulated in the fp32 workspace (zeroed here)
 *             and then written (narrowed) to grad_value.
 * grad_sampling_loc [batch, num_query, num_heads, num_levels, num_point, 2]
 * and grad_attention_weights [..., num_point] are written for every sample
 * (zeros for samples outside the bilinear gate).  im2col_step as in the
 * forward.  grad_value accumulation uses floating-point atomics, so its
 * last bits vary from run to run, as in the reference.  num_query may be 0
 * (the per-query arrays are then empty and may be NULL; grad_value is left
 * as it is for f32 and written with zeros for f16/bf16).
 */
BEVK_API int bevk_ms_deform_attn_backward(
    const void *value, const int64_t *spatial_shapes,
    const int64_t *level_start_index, const void *sampling_loc,
    const void *attention_weights, const void *grad_output, int batch,
    int spatial_size, int num_heads, int channels, int num_levels,
    int num_query, int num_point, int im2col_step, void *grad_value,
    void *grad_sampling_loc, void *grad_attention_weights, void *workspace,
    size_t workspace_bytes, int dtype, bevk_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* BEVK_H_ */
