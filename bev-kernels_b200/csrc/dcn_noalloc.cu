// dcn_noalloc.cu -- bevk_dcn_forward_noalloc: the DCNv2 forward for callers
// that may not allocate device memory when the layer runs (an engine plugin
// whose enqueue may not allocate, a runtime with memory frozen after start-up).
//
// The scratch the regular entry point takes from the caller's workspace -- the
// packed weight and, for NCHW input on the tensor-core path, the NHWC copy of
// the input -- lives here in one file-scope device array instead.  Host code
// never uses the array's name as an address: the device address is looked up
// with cudaGetSymbolAddress once per device (with that device current) and
// passed to the kernels.  Nothing in the array needs to start at zero: the
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

struct ScratchSlot {
  std::once_flag once;
  void *ptr = nullptr;
  cudaError_t err = cudaSuccess;
};
ScratchSlot g_scratch_slots[kMaxDevices];

// Device address of the scratch array on the current device (looked up once).
int scratch_address(void **out) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(BEVK_ERR_CUDA, "dcn noalloc: no current device");
  ScratchSlot &slot = g_scratch_slots[dev];
  std::call_once(slot.once, [&slot] {
    slot.err = cudaGetSymbolAddress(&slot.ptr, g_dcn_noalloc_scratch);
  });
  if (slot.err != cudaSuccess || slot.ptr == nullptr)
    return fail(BEVK_ERR_CUDA, "dcn noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(slot.err));
  *out = slot.ptr;
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
  for (int i = 0; i < 4; ++i)
    if (p->input_strides[i] < 0 || p->offset_strides[i] < 0 || p->mask_strides[i] < 0 ||
        p->output_strides[i] < 0)
      return fail(BEVK_ERR_INVALID_ARGUMENT, "dcn_forward_noalloc: negative strides are not supported");

  const size_t esz = dtype_size(p->dtype);
  const int64_t *xs_in = p->input_strides;
  const bool channel_contig = xs_in[1] == 1 && xs_in[0] % 8 == 0 && xs_in[2] % 8 == 0 &&
                              xs_in[3] % 8 == 0;
  const bool tc = dcn_tc_supported(p, d) && (!channel_contig || aligned(input, 16));
  const bool transpose = tc && !channel_contig;
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

  void *scratch = nullptr;
  st = scratch_address(&scratch);
  if (st != BEVK_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
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
    st = launch_dcn_forward_tc(p, d, x, xs, offset, mask, wpk, bias, output, s);
    if (st != BEVK_ERR_INDEX_OVERFLOW && st != BEVK_ERR_MISALIGNED) return st;
    clear_error();
  }
  return launch_dcn_forward_simt(p, d, input, offset, mask, wpk, bias, output, s);
}
