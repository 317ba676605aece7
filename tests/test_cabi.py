"""The C-ABI library loads on a CPU-only host, exports every symbol declared in
include/bevk.h and rejects bad arguments before touching a device."""
import ctypes
import os
import re

import pytest

from bevk import cabi

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    with open(os.path.join(REPO, "include", "bevk.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"BEVK_API\s+[^;(]*?\b(bevk_\w+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = _declared_symbols()
    assert set(names) == set(cabi.EXPORTED_SYMBOLS), names


def test_library_exports_every_declared_symbol():
    lib = cabi.lib()
    missing = [n for n in _declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_version_and_status_strings():
    assert cabi.version() >= 10000
    assert cabi.status_string(cabi.OK) == "ok"
    for code in range(-7, 0):
        assert cabi.status_string(code) not in ("ok", "unknown status")
    assert cabi.status_string(-99) == "unknown status"


def _problem(**kw):
    p = cabi.DcnProblem()
    p.dtype = cabi.DTYPE_F16
    p.batch, p.in_channels, p.height, p.width = 6, 512, 29, 50
    p.out_channels, p.kernel_h, p.kernel_w = 512, 3, 3
    p.stride_h = p.stride_w = p.pad_h = p.pad_w = p.dilation_h = p.dilation_w = 1
    p.groups = p.deformable_groups = 1
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def test_output_size_and_packed_bytes():
    lib = cabi.lib()
    ho, wo = ctypes.c_int(), ctypes.c_int()
    p = _problem()
    assert lib.bevk_dcn_output_size(ctypes.byref(p), ctypes.byref(ho), ctypes.byref(wo)) == 0
    assert (ho.value, wo.value) == (29, 50)
    assert lib.bevk_dcn_packed_weight_bytes(ctypes.byref(p)) == 512 * 9 * 512 * 2
    p2 = _problem(in_channels=72, out_channels=40, stride_h=2)
    assert lib.bevk_dcn_packed_weight_bytes(ctypes.byref(p2)) == 40 * 9 * 128 * 2  # 72 -> 128
    lib.bevk_dcn_output_size(ctypes.byref(p2), ctypes.byref(ho), ctypes.byref(wo))
    assert (ho.value, wo.value) == (15, 50)


@pytest.mark.parametrize("kw,status", [
    (dict(groups=3), cabi.ERR_INVALID_ARGUMENT),
    (dict(deformable_groups=5), cabi.ERR_INVALID_ARGUMENT),
    (dict(stride_h=0), cabi.ERR_INVALID_ARGUMENT),
    (dict(pad_h=-1), cabi.ERR_INVALID_ARGUMENT),
    (dict(height=1, pad_h=0), cabi.ERR_INVALID_ARGUMENT),
    (dict(dtype=9), cabi.ERR_UNSUPPORTED),
])
def test_problem_validation(kw, status):
    lib = cabi.lib()
    p = _problem(**kw)
    ho, wo = ctypes.c_int(), ctypes.c_int()
    assert lib.bevk_dcn_output_size(ctypes.byref(p), ctypes.byref(ho), ctypes.byref(wo)) == status
    assert cabi.last_error()


def test_forward_rejects_null_pointers_without_device():
    lib = cabi.lib()
    p = _problem()
    st = lib.bevk_dcn_forward(ctypes.byref(p), None, None, None, None, None, None, None, 0, None)
    assert st == cabi.ERR_INVALID_ARGUMENT and "null" in cabi.last_error()


def test_im2col_geometry_mismatch():
    lib = cabi.lib()
    fake = 16  # never dereferenced: validation fails first
    st = lib.bevk_modulated_deformable_im2col_opt(fake, fake, fake, 1, 8, 10, 10, 9, 10, 3, 3,
                                                  1, 1, 1, 1, 1, 1, 1, fake, cabi.DTYPE_F32, None)
    assert st == cabi.ERR_INVALID_ARGUMENT and "height_col" in cabi.last_error()
    st = lib.bevk_modulated_deformable_im2col_nhwc(fake, fake, fake, 1, 8, 10, 10, 10, 10, 3, 3,
                                                   1, 1, 1, 1, 1, 1, 2, 18, fake, cabi.DTYPE_F32,
                                                   None)
    assert st == cabi.ERR_UNSUPPORTED                      # deformable_group must be 1
    st = lib.bevk_modulated_deformable_im2col_nhwc(fake, fake, fake, 1, 8, 10, 10, 10, 10, 3, 3,
                                                   1, 1, 1, 1, 1, 1, 1, 20, fake, cabi.DTYPE_F32,
                                                   None)
    assert st == cabi.ERR_INVALID_ARGUMENT                 # offset last dim must be 2T or 3T


def test_msda_im2col_step_contract():
    lib = cabi.lib()
    fake = 16
    i64p = ctypes.POINTER(ctypes.c_int64)
    st = lib.bevk_ms_deform_attn_forward(fake, ctypes.cast(fake, i64p), ctypes.cast(fake, i64p),
                                         fake, fake, 3, 100, 8, 32, 1, 10, 4, 2, fake,
                                         cabi.DTYPE_F32, None)
    assert st == cabi.ERR_INVALID_ARGUMENT and "im2col_step" in cabi.last_error()
    st = lib.bevk_ms_deform_attn_forward(None, None, None, None, None, 3, 100, 8, 32, 1, 10, 4,
                                         64, None, cabi.DTYPE_F32, None)
    assert st == cabi.ERR_INVALID_ARGUMENT


def test_backward_data_size_limits_without_device():
    """bevk_dcn_backward_data rejects problems past its 32-bit indices with
    BEVK_ERR_INDEX_OVERFLOW before touching the device, and sizes the
    workspace of any problem."""
    lib = cabi.lib()
    B, C, H, W = 64, 16, 1000, 1000          # 64 M pixels x 9 taps: 2.3 G corner entries
    a = cabi.DcnBackwardDataArgs()
    a.problem = _problem(batch=B, in_channels=C, out_channels=C, height=H, width=W)
    for i, v in enumerate((H * W * C, 1, W * C, C)):           # NHWC input
        a.problem.input_strides[i] = v
        a.grad_input_strides[i] = v
    for i, v in enumerate((18 * H * W, H * W, W, 1)):
        a.problem.offset_strides[i] = v
        a.grad_offset_strides[i] = v
    for i, v in enumerate((9 * H * W, H * W, W, 1)):
        a.problem.mask_strides[i] = v
        a.grad_mask_strides[i] = v
    a.grad_dtype = cabi.DTYPE_F16
    a.dcol_ld = a.col_ld = 9 * C
    nbytes = lib.bevk_dcn_backward_data_workspace_bytes(ctypes.byref(a.problem))
    assert nbytes >= 4 * B * H * W * 9 * 8
    fake = 256  # 16-byte aligned, never dereferenced: the size checks come first
    st = lib.bevk_dcn_backward_data(ctypes.byref(a), fake, fake, fake, fake, fake, fake, fake,
                                    fake, fake, nbytes, None)
    assert st == cabi.ERR_INDEX_OVERFLOW, (st, cabi.last_error())
    assert "32-bit" in cabi.last_error()
