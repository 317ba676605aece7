// dcn_noalloc.cu -- bevk_dcn_forward_noalloc: the DCNv2 forward for callers
// that may not allocate device memory when the layer runs (an engine plugin
// whose enqueue may not allocate, a runtime with memory frozen after start-up).
//
// The scratch the regular entry point takes from the caller's workspace -- the
// packed weight and, for NCHW input on the tensor-core path, the NHWC copy of
// the input -- lives here in one file-scope device array instead.  Host code
// never uses the array's name as an address: the device address is looked up
// with cudaGetSymbolAddress by the first call on each device (with that device
// current; a failed lookup is retried by the next call) and passed to the
// kernels.  Nothing in the array needs to start at zero: the
// packing kernel writes every packed element including the zero padding, and
// the transpose writes every element of the input copy.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "bevk.h"
#include "bevk_internal.h"

// The scratch: one fixed array per device, held for the life of the process.
static __device__ __align__(256) unsigned char g_dcn_noalloc_scratch[BEVK_DCN_NOALLOC_SCRATCH_BYTES];

namespace bevk {
namespace {

constexpr int kMaxDevices = 64;

// Device address of the scratch array per device, filled by the first
// successful lookup (a failed lookup is not remembered: the next call retries).
std::mutex g_scratch_mutex;
void *g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device.
int scratch_address(cudaStream_t stream, void **out) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(BEVK_ERR_CUDA, "dcn noalloc: no current device");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    // The lookup may load the library's device code on this device, which a
    // stream capture does not allow: refuse instead of breaking the capture.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
      (void)cudaGetLastError();
      cap = cudaStreamCaptureStatusNone;
    }
    if (cap != cudaStreamCaptureStatusNone)
      return fail(BEVK_ERR_CUDA,
                  "dcn noalloc: the first call on device %d ran during a stream capture; make "
                  "one call on this device before capturing",
                  dev);
    void *ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_dcn_noalloc_scratch);
    if (err != cudaSuccess || ptr == nullptr) {
      (void)cudaGetLastError();  // leave no error pending for later checks in this thread
      return fail(BEVK_ERR_CUDA, "dcn noalloc: cudaGetSymbolAddress failed on device %d: %s",
                  dev, cudaGetErrorString(err));
    }
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return BEVK_OK;
}

size_t round256(size_t n) { return (n + 255) / 256 * 256; }

}  // namespace
}  // namespace bevk

using namespace bevk;

extern "C" BEVK_API int bevk_dcn_forward_noalloc(const bevk_dcn_problem *p, const void *input,
                                                 const void *offset, const void *mask,
                                                 const void *weight, const void *bias,
                                                 void *output, bevk_stream_t stream) {
  clear_error();
  DcnDims d;
  int st = dcn_dims(p, &d);
  if (st != BEVK_OK) return st;
  if (!input || !offset || !mask || !weight || !output || (p->has_bias && !bias))
    return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn_forward_noalloc: null pointer");
  // the same checks and path choice as bevk_dcn_forward
  st = validate_dcn_tensors(p, d);
  if (st != BEVK_OK) return st;

  const size_t esz = dtype_size(p->dtype);
  const int64_t *xs_in = p->input_strides;
  const bool tc = dcn_tc_supported(p, d) && (input_needs_transpose(p) || aligned(input, 16));
  const bool transpose = tc && input_needs_transpose(p);
  const size_t wbytes = static_cast<size_t>(d.Cout) * d.T * d.Cin_g_pad * esz;
  const size_t xbytes = transpose ? static_cast<size_t>(d.B) * d.H * d.W * d.Cin * esz : 0;
  const size_t need = round256(wbytes) + xbytes;
  if (need > BEVK_DCN_NOALLOC_SCRATCH_BYTES)
    return fail(BEVK_ERR_WORKSPACE,
                "dcn_forward_noalloc: this problem needs %zu bytes of scratch (packed weight "
                "%zu%s); the built-in scratch holds %zu bytes -- use bevk_dcn_forward with a "
                "caller workspace",
                need, wbytes, transpose ? " + NHWC input copy" : "",
                static_cast<size_t>(BEVK_DCN_NOALLOC_SCRATCH_BYTES));

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  void *scratch = nullptr;
  st = scratch_address(s, &scratch);
  if (st != BEVK_OK) return st;
  unsigned char *base = static_cast<unsigned char *>(scratch);
  void *wpk = base;
  st = launch_dcn_pack_weight(d, weight, wpk, p->dtype, s);
  if (st != BEVK_OK) return st;
  if (tc) {
    const void *x = input;
    int64_t xs[4] = {xs_in[0], xs_in[1], xs_in[2], xs_in[3]};
    if (transpose) {
      void *xcopy = base + round256(wbytes);
      st = launch_nchw_to_nhwc(input, xcopy, d.B, d.Cin, d.H, d.W, xs_in, p->dtype, s);
      if (st != BEVK_OK) return st;
      x = xcopy;
      xs[0] = static_cast<int64_t>(d.H) * d.W * d.Cin;
      xs[1] = 1;
      xs[2] = static_cast<int64_t>(d.W) * d.Cin;
      xs[3] = d.Cin;
    }
    st = launch_dcn_forward_tc(p, d, x, xs, offset, mask, wpk, bias, output, nullptr, 0, s);
    if (st != BEVK_ERR_INDEX_OVERFLOW && st != BEVK_ERR_MISALIGNED) return st;
    clear_error();
  }
  return launch_dcn_forward_simt(p, d, input, offset, mask, wpk, bias, output, s);
}
