// bevk_internal.h -- host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>

#include "bevk.h"

namespace bevk {

// Records a formatted message for bevk_last_error_message() and returns
// `status` so call sites can `return fail(BEVK_ERR_..., "...")`.
int fail(int status, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();
const char *last_error();

// Maps a CUDA error from the most recent launch into a status.
int check_launch(const char *what);
// Maps the result of a cudaLaunchKernelEx (then any pending launch error)
// into a status.
int launched(cudaError_t launch_result, const char *what);

// Cached per-device properties (filled once per device, thread-safe).
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  int max_smem_optin = 0;
  int l2_bytes = 0;
};
const DeviceInfo &device_info(int device);
int current_device();

// Whether kernels that support it are launched as programmatic dependents of
// the stream's previous kernel (on unless the environment sets BEVK_PDL=0;
// read once).
bool programmatic_launch_enabled();

// Launches `kern` (grid, block, dynamic shared memory, stream) as a
// programmatic dependent of the stream's previous kernel when that is
// enabled.  The kernel calls ptx::grid_wait_prerequisites() before it touches
// global memory, so results are as with an ordinary launch.
template <typename... Params, typename... Args>
cudaError_t launch_dependent(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t stream, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = programmatic_launch_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args &&>(args)...);
}

inline size_t dtype_size(int dtype) {
  switch (dtype) {
    case BEVK_DTYPE_F32: return 4;
    case BEVK_DTYPE_F16: return 2;
    case BEVK_DTYPE_BF16: return 2;
    case BEVK_DTYPE_F64: return 8;
    default: return 0;
  }
}

inline bool aligned(const void *p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// Derived geometry of a DCN problem (validated).
struct DcnDims {
  int B, Cin, H, W, Cout, kH, kW, T;
  int sh, sw, ph, pw, dh, dw, groups, dg;
  int Ho, Wo;
  int Cin_g, Cout_g, Cin_g_pad, cpdg;
  int64_t M;  // B*Ho*Wo
};
int dcn_dims(const bevk_dcn_problem *p, DcnDims *d);
// Checks the problem's tensor strides (no negative strides) -- shared by the
// DCN forward entry points so they accept exactly the same problems.
int validate_dcn_tensors(const bevk_dcn_problem *p, const DcnDims &d);
// The tensor-core path needs channel-contiguous input with pixel rows of a
// multiple of 8 elements; other input is first transposed to NHWC.
bool input_needs_transpose(const bevk_dcn_problem *p);

// Kernel launchers (return BEVK_OK or a status; arguments are pre-validated).
int launch_dcn_col2im(const bevk_dcn_col2im_args *a, const DcnDims &d, const void *input,
                      const void *offset, const void *mask, const void *dcol, void *grad_input,
                      void *grad_offset, void *grad_mask, cudaStream_t stream);
size_t dcn_backward_data_workspace_bytes(const DcnDims &d);
int launch_dcn_backward_data(const bevk_dcn_backward_data_args *a, const DcnDims &d,
                             const void *input, const void *offset, const void *mask,
                             const void *dcol, void *grad_input, void *grad_offset,
                             void *grad_mask, void *col, void *workspace,
                             size_t workspace_bytes, cudaStream_t stream);
size_t msda_backward_workspace_bytes(int B, int S, int heads, int C, int dtype);
int launch_msda_backward(const void *value, const int64_t *shapes, const int64_t *lsi,
                         const void *loc, const void *attn, const void *grad_out,
                         void *grad_value, void *grad_loc, void *grad_attn, int B, int S,
                         int heads, int C, int L, int Q, int P, void *workspace,
                         size_t workspace_bytes, int dtype, cudaStream_t stream);
int launch_msda_forward(const void *value, const int64_t *shapes, const int64_t *lsi,
                        const void *loc, const void *attn, int B, int S, int heads,
                        int C, int L, int Q, int P, void *out, int dtype,
                        cudaStream_t stream);

int launch_dcn_pack_weight(const DcnDims &d, const void *w, void *wpk, int dtype,
                           cudaStream_t stream);
int launch_nchw_to_nhwc(const void *src, void *dst, int B, int C, int H, int W,
                        const int64_t src_strides[4], int dtype, cudaStream_t stream);
int launch_dcn_forward_simt(const bevk_dcn_problem *p, const DcnDims &d,
                            const void *x, const void *off, const void *msk,
                            const void *wpk, const void *bias, void *out,
                            cudaStream_t stream);
// Tensor-core path: x must be channel-contiguous (c stride 1) with 16-byte
// aligned pixel rows; returns BEVK_ERR_UNSUPPORTED when the geometry is not
// covered so the caller can pick the SIMT kernel.
// `ws` (may be null) is scratch for the K-split schedule, used when it holds
// dcn_tc_workspace_bytes(p, d) bytes at a 256-byte boundary; without it the
// kernel takes a schedule that needs none.
bool dcn_tc_supported(const bevk_dcn_problem *p, const DcnDims &d);
size_t dcn_tc_workspace_bytes(const bevk_dcn_problem *p, const DcnDims &d);
int launch_dcn_forward_tc(const bevk_dcn_problem *p, const DcnDims &d,
                          const void *x, const int64_t x_strides[4],
                          const void *off, const void *msk, const void *wpk,
                          const void *bias, void *out, void *ws, size_t ws_bytes,
                          cudaStream_t stream);

// Offset convolution from its per-tap partial products (see
// bevk_dcn_zoff_args): y[m, c] = round(bias[c] + sum_t z[p_t(m) * ld + t*3T + c]),
// y [B*Ho*Wo][3T] in the problem dtype (fp16/bf16/fp32).
int launch_dcn_offset_sum(const bevk_dcn_problem *p, const DcnDims &d, const float *z,
                          int64_t ld, const float *bias, void *y, cudaStream_t stream);

// Column-matrix ops.  col_layout 0: [C*T, B*Ho*Wo] (row c*T + t);
// col_layout 1: [B*Ho*Wo, T*C] (k = t*C + c).
int launch_dcn_im2col(const bevk_dcn_problem *p, const DcnDims &d, const void *x,
                      const void *off, const void *msk, void *col, int col_layout,
                      cudaStream_t stream);

// Device watchdog word (one per device, defined in dcn_tc.cu).
int read_and_clear_watchdog(int device, unsigned int *code);
// Limit of the fused DCN kernel's pipeline barrier waits on `device` (0: the
// default 2 s); launches read it on the host and pass it to the kernel.
int set_wait_limit(int device, unsigned long long ns);
unsigned long long wait_limit(int device);

}  // namespace bevk
