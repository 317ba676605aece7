"""bevk_dcn_forward_noalloc: the DCN forward for callers that cannot allocate
device memory when the layer runs (an inference engine's plugin whose enqueue
may not allocate, a runtime whose device memory is frozen after start-up).

It must give the same result as the regular entry point, which takes the
packed weight and workspace from the caller, and it keeps state in one shared
scratch array -- so two calls in a row, with different data and weights, must
each match.  This file is collected last so a failure here comes after every
other test has run.
"""
import ctypes

import pytest
import torch

from bevk import cabi
from helpers import FP32_ABS, FP32_REL, HALF_REL, cabi_dcn_forward, dcn_inputs, problem, rel_l2

pytestmark = pytest.mark.gpu


def _noalloc(x, off, mask, w, b, out, stride, pad, dil, groups=1, dg=1):
    p = problem(x, off, mask, out, w.shape[0], (w.shape[2], w.shape[3]), stride, pad, dil,
                groups, dg, False, b is not None)
    wc = w.contiguous()
    st = cabi.lib().bevk_dcn_forward_noalloc(
        ctypes.byref(p), x.data_ptr(), off.data_ptr(), mask.data_ptr(), wc.data_ptr(),
        b.data_ptr() if b is not None else None, out.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    cabi.check(st, "bevk_dcn_forward_noalloc")
    return out


CASES = [
    # dtype, NCHW input (needs the NHWC copy in scratch), B, C, H, W, Cout
    (torch.float16, True, 2, 64, 16, 20, 128),
    (torch.bfloat16, False, 3, 96, 11, 13, 160),
    (torch.float32, True, 1, 24, 9, 10, 40),       # exact SIMT path: only the packed weight
]


@pytest.mark.parametrize("case", CASES, ids=["f16_nchw", "bf16_nhwc", "f32"])
def test_noalloc_matches_workspace_entry_point_twice(cuda, case):
    dt, nchw, B, C, H, W, Cout = case
    for call, seed in enumerate((101, 202)):          # two calls in a row, new data each time
        x, off, mask, w, b = dcn_inputs(seed, B, C, H, W, Cout + 16 * call)
        x, off, mask, w, b = (t.to(cuda, dt) for t in (x, off, mask, w, b))
        if not nchw:
            x = x.contiguous(memory_format=torch.channels_last)
        want = torch.empty(B, w.shape[0], H, W, dtype=dt, device=cuda)
        cabi_dcn_forward(x, off, mask, w, b, want, (1, 1), (1, 1), (1, 1))
        got = torch.full_like(want, float("nan"))
        _noalloc(x, off, mask, w, b, got, (1, 1), (1, 1), (1, 1))
        torch.cuda.synchronize()
        assert torch.isfinite(got).all(), f"call {call}"
        r = rel_l2(got, want)
        if dt == torch.float32:
            assert r <= FP32_REL and float((got - want).abs().max()) <= FP32_ABS, (call, r)
        else:
            assert r <= HALF_REL, (call, r)


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    # a 2048 -> 2048 channel 3x3 fp16 layer: its packed weight alone
    # (2048 * 9 * 2048 * 2 bytes = 72 MiB) exceeds the 32 MiB built-in scratch,
    # so the call refuses on every path (tensor-core or SIMT, NCHW or NHWC)
    # before it touches any pointer.
    B, C, H, W = 1, 2048, 8, 8
    p = cabi.DcnProblem()
    p.dtype = cabi.DTYPE_F16
    p.batch, p.in_channels, p.height, p.width = B, C, H, W
    p.out_channels, p.kernel_h, p.kernel_w = C, 3, 3
    p.stride_h = p.stride_w = p.pad_h = p.pad_w = p.dilation_h = p.dilation_w = 1
    p.groups = p.deformable_groups = 1
    hw = H * W
    for i, v in enumerate((C * hw, hw, W, 1)):
        p.input_strides[i] = v
        p.output_strides[i] = v
    for i, v in enumerate((18 * hw, hw, W, 1)):
        p.offset_strides[i] = v
    for i, v in enumerate((9 * hw, hw, W, 1)):
        p.mask_strides[i] = v
    assert cabi.lib().bevk_dcn_packed_weight_bytes(ctypes.byref(p)) > (32 << 20)
    fake = 256  # never dereferenced: the size check comes first
    st = cabi.lib().bevk_dcn_forward_noalloc(ctypes.byref(p), fake, fake, fake, fake, None, fake,
                                             None)
    assert st == cabi.ERR_WORKSPACE
    assert "scratch" in cabi.last_error()
