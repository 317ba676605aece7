"""The Pack module's offset convolution as one GEMM plus this library's tap-sum
kernel (offset_conv / bevk_dcn_offset_conv_sum / bevk_dcn_forward_zoff),
against the unfused composite: the offset conv in fp32 on the up-cast inputs,
rounded to the input dtype (what the reference's cuDNN offset conv returns,
dcn_split_nhwc.py:171-172), then the oracle DCN forward with the sigmoid mask.

Tolerances: the offset-conv output within 2e-3 relative L2 of the rounded fp32
convolution (the two sums differ in order, so a few elements round to the
neighbouring fp16/bf16 value); the DCN output within 5e-3 relative L2 of the
oracle (fp16/bf16 in, fp32 accumulate).
"""
import ctypes

import pytest
import torch
import torch.nn.functional as F

from helpers import HALF_REL, problem, rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu

CASES = [
    # B, Cin, H, W, Cout, k, stride, pad, dil
    (2, 64, 12, 17, 64, (3, 3), (1, 1), (1, 1), (1, 1)),       # single CTAs
    (2, 128, 10, 19, 320, (3, 3), (2, 2), (1, 1), (1, 1)),     # N-split pairs, stride 2
    (1, 72, 11, 13, 160, (3, 3), (1, 1), (2, 2), (2, 2)),      # M-paired CTAs, dilation 2
    (1, 40, 9, 9, 130, (1, 3), (1, 1), (0, 1), (1, 1)),        # 1x3 kernel (3T = 9 channels)
    (3, 256, 8, 12, 256, (3, 3), (1, 1), (1, 1), (1, 1)),
]


def _inputs(seed, B, C, H, W, Cout, k, dt):
    g = torch.Generator().manual_seed(seed)
    T = k[0] * k[1]
    x = torch.randn(B, H, W, C, generator=g)
    # offsets of a few pixels and mask logits around 0
    w_off = torch.randn(3 * T, C, *k, generator=g) * (1.5 / (C * T) ** 0.5)
    b_off = torch.randn(3 * T, generator=g) * 0.5
    w = torch.randn(Cout, C, *k, generator=g) * (1.0 / (C * T) ** 0.5)
    b = torch.randn(Cout, generator=g)
    return [t.to(dt) for t in (x, w_off, b_off, w, b)]


def _composite(x, w_off, b_off, w, b, stride, pad, dil):
    """Unfused CPU composite -> (output NHWC fp32, rounded offset-conv output NHWC)."""
    T = w.shape[2] * w.shape[3]
    y = F.conv2d(x.permute(0, 3, 1, 2).float(), w_off.float(), b_off.float(), stride, pad, dil)
    y = y.to(x.dtype).float()
    off, mask = y[:, :2 * T], torch.sigmoid(y[:, 2 * T:])
    out = oracle.dcn_forward(x.permute(0, 3, 1, 2).float().numpy(), off.numpy(), mask.numpy(),
                             w.float().numpy(), b.float().numpy(), stride, pad, dil)
    return torch.from_numpy(out).permute(0, 2, 3, 1), y.permute(0, 2, 3, 1)


@pytest.mark.parametrize("case", CASES, ids=[f"z{i}" for i in range(len(CASES))])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_offset_conv_and_forward_match_unfused_composite(cuda, case, dt):
    from modulated_deform_conv import dcn_forward_into, offset_conv
    B, C, H, W, Cout, k, stride, pad, dil = case
    x, w_off, b_off, w, b = _inputs(3, B, C, H, W, Cout, k, dt)
    want, y_want = _composite(x, w_off, b_off, w, b, stride, pad, dil)
    T = k[0] * k[1]
    xd, wod, bod, wd, bd = (t.to(cuda) for t in (x, w_off, b_off, w, b))
    y = offset_conv(xd, wod, bod, stride, pad, dil)
    assert y.shape == y_want.shape and y.dtype == dt
    assert rel_l2(y.float(), y_want) <= 2e-3, rel_l2(y.float(), y_want)
    out = torch.empty(want.shape, device=cuda, dtype=dt)
    yv = y.permute(0, 3, 1, 2)
    dcn_forward_into(xd.permute(0, 3, 1, 2), yv[:, :2 * T], yv[:, 2 * T:], wd, bd,
                     out.permute(0, 3, 1, 2), stride, pad, dil, mask_is_logit=True)
    assert rel_l2(out.float(), want) <= HALF_REL, rel_l2(out.float(), want)


def test_offset_conv_partials_layout(cuda):
    """Summing the shifted taps of the partial products on the host gives the
    offset convolution (the layout contract of bevk_dcn_zoff_args)."""
    from modulated_deform_conv import offset_conv_partials
    B, C, H, W, k = 2, 32, 7, 9, (3, 3)
    x, w_off, _, _, _ = _inputs(5, B, C, H, W, 8, k, torch.float16)
    T = 9
    z = offset_conv_partials(x.to(cuda), w_off.to(cuda)).cpu()
    assert z.shape[0] == B * H * W and z.shape[1] >= T * 3 * T
    z = z[:, :T * 3 * T].reshape(B, H, W, T, 3 * T).permute(3, 4, 0, 1, 2)   # [T, 3T, B, H, W]
    zp = F.pad(z, (1, 1, 1, 1))                       # zero taps outside the image
    y = sum(zp[t, :, :, t // 3:t // 3 + H, t % 3:t % 3 + W] for t in range(T))
    want = F.conv2d(x.permute(0, 3, 1, 2).float(), w_off.float(), None, 1, 1, 1)
    assert rel_l2(y.permute(1, 0, 2, 3), want) <= 1e-5


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_split_nhwc_gemm_offset_matches_cudnn_offset(cuda, dt, monkeypatch):
    """dcn_split_nhwc forward and backward over offset_conv against the same
    Function with cuDNN's offset conv made to return offset_conv's own output:
    same y, so the outputs and all five gradients must agree (the bilinear
    weights' gradients jump where an offset crosses an integer, so a 1-ulp
    difference in y would not compare)."""
    import sys
    from modulated_deform_conv import offset_conv
    split = sys.modules["modulated_deform_conv.dcn_split_nhwc"]
    B, C, H, W, Cout, k = 2, 64, 11, 14, 128, (3, 3)
    tens = [t.to(cuda) for t in _inputs(9, B, C, H, W, Cout, k, dt)]
    gout = torch.randn(B, H, W, Cout, generator=torch.Generator().manual_seed(10)).to(dt)
    y_g = offset_conv(tens[0], tens[1], tens[2], 1, 1, 1)
    results = []
    for gemm in (True, False):
        if not gemm:
            monkeypatch.setattr(split, "offset_conv_supported", lambda *a: False)
            monkeypatch.setattr(split.F, "conv2d", lambda *a, **kw: y_g.permute(0, 3, 1, 2))
        ts = [t.clone().requires_grad_() for t in tens]
        out = split.dcn_split_nhwc(*ts, 1, 1, 1)
        out.backward(gout.to(cuda))
        results.append((out.detach().float(), [t.grad.float() for t in ts]))
    (o1, g1), (o2, g2) = results
    assert torch.equal(o1, o2)
    for name, a, b_ in zip(("x", "w_off", "b_off", "weight", "bias"), g1, g2):
        assert rel_l2(a, b_) <= 1e-3, (name, rel_l2(a, b_))


def test_cabi_offset_conv_contract(cuda):
    """bevk_dcn_offset_conv_sum and bevk_dcn_forward_zoff through the C ABI:
    NULL pointers and a short partials_ld are invalid arguments; the composite
    forward equals offset conv + bevk_dcn_forward."""
    from bevk import cabi
    from modulated_deform_conv import dcn_forward_into, offset_conv_partials, packed_weight
    L = cabi.lib()
    B, C, H, W, Cout, k = 1, 64, 6, 7, 64, (3, 3)
    x, w_off, b_off, w, b = (t.to(cuda) for t in _inputs(4, B, C, H, W, Cout, k, torch.float16))
    out = torch.empty(B, H, W, Cout, device=cuda, dtype=torch.float16)
    xv, ov = x.permute(0, 3, 1, 2), out.permute(0, 3, 1, 2)
    p = problem(xv, xv, xv, ov, Cout, k, (1, 1), (1, 1), (1, 1), has_bias=True)
    wpk = packed_weight(w, 1)
    partials = offset_conv_partials(x, w_off)
    bf = b_off.float()
    y = torch.zeros(B, H, W, 27, device=cuda, dtype=torch.float16)
    for args in (cabi.DcnZoffArgs(None, partials.stride(0), bf.data_ptr(), y.data_ptr()),
                 cabi.DcnZoffArgs(partials.data_ptr(), partials.stride(0), bf.data_ptr(), None),
                 cabi.DcnZoffArgs(partials.data_ptr(), 26, bf.data_ptr(), y.data_ptr())):
        assert L.bevk_dcn_offset_conv_sum(ctypes.byref(p), ctypes.byref(args), None) == \
            cabi.ERR_INVALID_ARGUMENT
    args = cabi.DcnZoffArgs(partials.data_ptr(), partials.stride(0), bf.data_ptr(), y.data_ptr())
    st = L.bevk_dcn_forward_zoff(ctypes.byref(p), ctypes.byref(args), xv.data_ptr(),
                                 wpk.data_ptr(), b.data_ptr(), ov.data_ptr(), None)
    assert st == cabi.OK, cabi.last_error()
    torch.cuda.synchronize()
    y_want = F.conv2d(xv.float(), w_off.float(), bf, 1, 1, 1).half().float().permute(0, 2, 3, 1)
    assert rel_l2(y.float(), y_want) <= 2e-3
    want = torch.empty_like(out)
    yv = y.permute(0, 3, 1, 2)
    dcn_forward_into(xv, yv[:, :18], yv[:, 18:], w, b, want.permute(0, 3, 1, 2), 1, 1, 1,
                     mask_is_logit=True)
    assert torch.equal(out, want)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32],
                         ids=["f16", "bf16", "f32"])
@pytest.mark.parametrize("geom", [((3, 3), 1, 1, 1), ((3, 3), 2, 2, 2)], ids=["s1", "s2d2"])
def test_fused_im2col_nhwc_op(cuda, dt, geom):
    """modulated_deformable_fused_im2col_nhwc_cuda (the reference's binding.cpp
    :72-78): offset conv + gather + sigmoid modulation into Col [M, T*Cin],
    against the offset conv in fp32 (rounded to the input dtype) and the
    oracle's NHWC columns."""
    import _modulated_deform_conv_ext as ext
    k, stride, pad, dil = geom
    B, C, H, W = 2, 64, 11, 14
    x, w_off, b_off, _, _ = _inputs(9, B, C, H, W, 8, k, dt)
    T = k[0] * k[1]
    y = F.conv2d(x.permute(0, 3, 1, 2).float(), w_off.float(), b_off.float(), stride, pad, dil)
    y = y.to(dt).float()
    Ho, Wo = y.shape[2], y.shape[3]
    want = torch.from_numpy(oracle.dcn_columns(
        x.permute(0, 3, 1, 2).float().numpy(), y[:, :2 * T].numpy(),
        torch.sigmoid(y[:, 2 * T:]).numpy(), k, stride, pad, dil, 1, layout="nhwc"))
    col = torch.full((B * Ho * Wo, T * C), float("nan"), device=cuda, dtype=dt)
    ext.modulated_deformable_fused_im2col_nhwc_cuda(
        x.to(cuda).contiguous(), w_off.permute(0, 2, 3, 1).contiguous().to(cuda),
        b_off.float().to(cuda), B, C, H, W, Ho, Wo, k[0], k[1], pad, pad, stride, stride, dil,
        dil, 1, col)
    torch.cuda.synchronize()
    assert torch.isfinite(col).all()
    tol = 1e-5 if dt == torch.float32 else HALF_REL
    assert rel_l2(col.float(), want) <= tol, rel_l2(col.float(), want)
