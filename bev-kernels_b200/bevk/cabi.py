"""ctypes binding of the C ABI in ``include/bevk.h`` (``libbevk.so``).

This is the binding a Python caller without the torch extensions would use,
and the one the GPU parity tests call through.  Pointers are plain integers
(e.g. ``tensor.data_ptr()``); streams are raw ``cudaStream_t`` handles
(e.g. ``torch.cuda.current_stream().cuda_stream``).
"""
from __future__ import annotations

import ctypes
import os

from . import LIB_PATH, _BUILD_HINT

DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_F64 = 0, 1, 2, 3

OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_INDEX_OVERFLOW = -3
ERR_MISALIGNED = -4
ERR_CUDA = -5
ERR_WORKSPACE = -6
ERR_DEVICE_TIMEOUT = -7

# Size of the scratch array behind bevk_dcn_forward_noalloc (BEVK_DCN_NOALLOC_SCRATCH_BYTES).
DCN_NOALLOC_SCRATCH_BYTES = 32 << 20

# Every exported symbol of include/bevk.h.
EXPORTED_SYMBOLS = (
    "bevk_version",
    "bevk_status_string",
    "bevk_last_error_message",
    "bevk_device_watchdog",
    "bevk_set_wait_limit_ns",
    "bevk_dcn_output_size",
    "bevk_dcn_packed_weight_bytes",
    "bevk_dcn_pack_weight",
    "bevk_dcn_forward_workspace_bytes",
    "bevk_dcn_forward",
    "bevk_dcn_offset_conv_sum",
    "bevk_dcn_forward_zoff",
    "bevk_dcn_forward_noalloc",
    "bevk_modulated_deformable_im2col",
    "bevk_modulated_deformable_im2col_opt",
    "bevk_modulated_deformable_im2col_nhwc",
    "bevk_dcn_columns",
    "bevk_dcn_col2im",
    "bevk_dcn_backward_data_workspace_bytes",
    "bevk_dcn_backward_data",
    "bevk_ms_deform_attn_forward",
    "bevk_ms_deform_attn_backward_workspace_bytes",
    "bevk_ms_deform_attn_backward",
)


class DcnZoffArgs(ctypes.Structure):
    """Mirror of ``bevk_dcn_zoff_args``."""

    _fields_ = [("partials", ctypes.c_void_p), ("partials_ld", ctypes.c_int64),
                ("offset_bias", ctypes.c_void_p), ("offset_out", ctypes.c_void_p)]


class DcnProblem(ctypes.Structure):
    """Mirror of ``bevk_dcn_problem``."""

    _fields_ = [
        ("dtype", ctypes.c_int),
        ("batch", ctypes.c_int), ("in_channels", ctypes.c_int),
        ("height", ctypes.c_int), ("width", ctypes.c_int),
        ("out_channels", ctypes.c_int), ("kernel_h", ctypes.c_int), ("kernel_w", ctypes.c_int),
        ("stride_h", ctypes.c_int), ("stride_w", ctypes.c_int),
        ("pad_h", ctypes.c_int), ("pad_w", ctypes.c_int),
        ("dilation_h", ctypes.c_int), ("dilation_w", ctypes.c_int),
        ("groups", ctypes.c_int), ("deformable_groups", ctypes.c_int),
        ("input_strides", ctypes.c_int64 * 4),
        ("offset_strides", ctypes.c_int64 * 4),
        ("mask_strides", ctypes.c_int64 * 4),
        ("output_strides", ctypes.c_int64 * 4),
        ("mask_is_logit", ctypes.c_int),
        ("has_bias", ctypes.c_int),
        ("act_relu", ctypes.c_int),
    ]


class DcnCol2imArgs(ctypes.Structure):
    """Mirror of ``bevk_dcn_col2im_args``."""

    _fields_ = [
        ("problem", DcnProblem),
        ("col_dtype", ctypes.c_int),
        ("col_strides", ctypes.c_int64 * 3),
        ("grad_input_strides", ctypes.c_int64 * 4),
        ("grad_offset_strides", ctypes.c_int64 * 4),
        ("grad_mask_strides", ctypes.c_int64 * 4),
    ]


class DcnBackwardDataArgs(ctypes.Structure):
    """Mirror of ``bevk_dcn_backward_data_args``."""

    _fields_ = [
        ("problem", DcnProblem),
        ("grad_dtype", ctypes.c_int),
        ("dcol_ld", ctypes.c_int64),
        ("col_ld", ctypes.c_int64),
        ("grad_input_strides", ctypes.c_int64 * 4),
        ("grad_offset_strides", ctypes.c_int64 * 4),
        ("grad_mask_strides", ctypes.c_int64 * 4),
    ]


class BevkError(RuntimeError):
    def __init__(self, status: int, what: str, detail: str):
        super().__init__(f"{what}: {status_string(status)} ({status}): {detail}")
        self.status = status


_lib = None


def lib():
    """Load libbevk.so and declare argument types (idempotent)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"{LIB_PATH} not found; {_BUILD_HINT}")
    L = ctypes.CDLL(LIB_PATH)
    i, vp, sz, i64p = ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int64)
    pp = ctypes.POINTER(DcnProblem)
    L.bevk_version.restype = i
    L.bevk_status_string.restype = ctypes.c_char_p
    L.bevk_status_string.argtypes = [i]
    L.bevk_last_error_message.restype = ctypes.c_char_p
    L.bevk_device_watchdog.restype = i
    L.bevk_device_watchdog.argtypes = [i, ctypes.POINTER(ctypes.c_uint)]
    L.bevk_set_wait_limit_ns.restype = i
    L.bevk_set_wait_limit_ns.argtypes = [i, ctypes.c_ulonglong]
    L.bevk_dcn_output_size.restype = i
    L.bevk_dcn_output_size.argtypes = [pp, ctypes.POINTER(i), ctypes.POINTER(i)]
    L.bevk_dcn_packed_weight_bytes.restype = sz
    L.bevk_dcn_packed_weight_bytes.argtypes = [pp]
    L.bevk_dcn_pack_weight.restype = i
    L.bevk_dcn_pack_weight.argtypes = [pp, vp, vp, vp]
    L.bevk_dcn_forward_workspace_bytes.restype = sz
    L.bevk_dcn_forward_workspace_bytes.argtypes = [pp]
    L.bevk_dcn_forward.restype = i
    L.bevk_dcn_forward.argtypes = [pp, vp, vp, vp, vp, vp, vp, vp, sz, vp]
    L.bevk_dcn_forward_noalloc.restype = i
    L.bevk_dcn_forward_noalloc.argtypes = [pp, vp, vp, vp, vp, vp, vp, vp]
    L.bevk_dcn_offset_conv_sum.restype = i
    L.bevk_dcn_offset_conv_sum.argtypes = [pp, ctypes.POINTER(DcnZoffArgs), vp]
    L.bevk_dcn_forward_zoff.restype = i
    L.bevk_dcn_forward_zoff.argtypes = [pp, ctypes.POINTER(DcnZoffArgs), vp, vp, vp, vp, vp]
    L.bevk_dcn_columns.restype = i
    L.bevk_dcn_columns.argtypes = [pp, vp, vp, vp, vp, i, vp]
    L.bevk_dcn_col2im.restype = i
    L.bevk_dcn_col2im.argtypes = [ctypes.POINTER(DcnCol2imArgs), vp, vp, vp, vp, vp, vp, vp, vp]
    L.bevk_dcn_backward_data_workspace_bytes.restype = sz
    L.bevk_dcn_backward_data_workspace_bytes.argtypes = [pp]
    L.bevk_dcn_backward_data.restype = i
    L.bevk_dcn_backward_data.argtypes = ([ctypes.POINTER(DcnBackwardDataArgs)] + [vp] * 9 +
                                         [sz, vp])
    col_args = [vp, vp, vp] + [i] * 15
    L.bevk_modulated_deformable_im2col.restype = i
    L.bevk_modulated_deformable_im2col.argtypes = col_args + [vp, i, vp]
    L.bevk_modulated_deformable_im2col_opt.restype = i
    L.bevk_modulated_deformable_im2col_opt.argtypes = col_args + [vp, i, vp]
    L.bevk_modulated_deformable_im2col_nhwc.restype = i
    L.bevk_modulated_deformable_im2col_nhwc.argtypes = col_args + [i, vp, i, vp]
    L.bevk_ms_deform_attn_forward.restype = i
    L.bevk_ms_deform_attn_forward.argtypes = [vp, i64p, i64p, vp, vp] + [i] * 8 + [vp, i, vp]
    L.bevk_ms_deform_attn_backward_workspace_bytes.restype = ctypes.c_size_t
    L.bevk_ms_deform_attn_backward_workspace_bytes.argtypes = [i] * 5
    L.bevk_ms_deform_attn_backward.restype = i
    L.bevk_ms_deform_attn_backward.argtypes = ([vp, i64p, i64p, vp, vp, vp] + [i] * 8 +
                                               [vp, vp, vp, vp, ctypes.c_size_t, i, vp])
    _lib = L
    return L


def status_string(status: int) -> str:
    return lib().bevk_status_string(int(status)).decode()


def last_error() -> str:
    return lib().bevk_last_error_message().decode()


def check(status: int, what: str) -> None:
    if status != OK:
        raise BevkError(status, what, last_error())


def version() -> int:
    return int(lib().bevk_version())
