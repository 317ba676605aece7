"""DCNv2 backward parity on the GPU vs the reference's backward goldens and the
CPU oracle: the col2im ops (reference names, NCHW column matrix), the C-ABI
scatter with the NHWC column matrix, ModulatedDeformConv2dFunction.backward and
the NHWC split Function's backward.

Tolerances: fp32 within 1e-5 relative L2; fp16/bf16 within 5e-3 relative L2 of
the fp32 oracle on the up-cast inputs.
"""
import ctypes
import glob
import os

import numpy as np
import pytest
import torch

from bevk import cabi
from helpers import DT, FP32_REL, HALF_REL, dcn_inputs, problem, rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DCN_FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "dcn_*.npz")))


def _meta(z):
    kh, kw, sh, sw, ph, pw, dh, dw, groups, dg = (int(v) for v in z["meta"])
    return (kh, kw), (sh, sw), (ph, pw), (dh, dw), groups, dg


def _nchw_dcol(weight, gout, groups):
    """Reference column gradient [C*T, B*Ho*Wo] = W^T . dO per conv group
    (modulated_deform_conv.py:435-451)."""
    Cout = weight.shape[0]
    B, _, Ho, Wo = gout.shape
    wg = weight.reshape(groups, Cout // groups, -1)
    go = gout.permute(1, 0, 2, 3).reshape(groups, Cout // groups, B * Ho * Wo)
    return torch.cat([wg[g].t() @ go[g] for g in range(groups)], 0).contiguous()


@pytest.mark.parametrize("path", DCN_FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_col2im_ops_match_reference_golden(cuda, path):
    import _modulated_deform_conv_ext as ext
    z = np.load(path)
    (kh, kw), (sh, sw), (ph, pw), (dh, dw), groups, dg = _meta(z)
    x, off, mask, w, gout = (torch.from_numpy(z[n]).to(cuda) for n in (
        "x", "offset", "mask", "weight", "grad_out"))
    B, C, H, W = x.shape
    Ho, Wo = gout.shape[2], gout.shape[3]
    dcol = _nchw_dcol(w, gout, groups)
    geom = (B, C, H, W, Ho, Wo, kh, kw, ph, pw, sh, sw, dh, dw, dg)
    gx = torch.zeros_like(x)
    ext.modulated_deformable_col2im_smem_cuda(dcol, off, mask, *geom, gx)
    goff = torch.full_like(off, 7.0)        # written, not accumulated
    gm = torch.full_like(mask, 7.0)
    ext.modulated_deformable_col2im_coord_opt_cuda(dcol, x, off, mask, *geom, goff, gm)
    for got, name in ((gx, "grad_x"), (goff, "grad_offset"), (gm, "grad_mask")):
        want = torch.from_numpy(z[name])
        assert rel_l2(got, want) <= FP32_REL, (name, rel_l2(got, want))


@pytest.mark.parametrize("path", DCN_FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_function_backward_matches_reference_golden(cuda, path):
    import modulated_deform_conv as mdc
    z = np.load(path)
    k, st, pd, dl, groups, dg = _meta(z)
    tens = {n: torch.from_numpy(z[n]).to(cuda).requires_grad_() for n in (
        "x", "offset", "mask", "weight")}
    bias = (torch.from_numpy(z["bias"]).to(cuda).requires_grad_()
            if "bias" in z.files else None)
    out = mdc.modulated_deform_conv2d(tens["x"], tens["offset"], tens["mask"], tens["weight"],
                                      bias, st, pd, dl, groups, dg)
    out.backward(torch.from_numpy(z["grad_out"]).to(cuda))
    pairs = [(tens["x"].grad, "grad_x"), (tens["offset"].grad, "grad_offset"),
             (tens["mask"].grad, "grad_mask"), (tens["weight"].grad, "grad_weight")]
    if bias is not None:
        pairs.append((bias.grad, "grad_bias"))
    for got, name in pairs:
        want = torch.from_numpy(z[name])
        assert rel_l2(got, want) <= FP32_REL, (name, rel_l2(got, want))


def test_cabi_col2im_nhwc_columns(cuda):
    """bevk_dcn_col2im through ctypes with channels-last tensors and the NHWC
    column matrix [M, T*C] (k = t*C + c)."""
    B, C, H, W, Cout = 2, 32, 9, 11, 16
    x, off, mask, w, _ = dcn_inputs(31, B, C, H, W, Cout, big_frac=0.05, bias=False)
    gout = torch.randn(B, Cout, H, W, generator=torch.Generator().manual_seed(32))
    want = oracle.dcn_backward(x.numpy(), off.numpy(), mask.numpy(), w.numpy(), gout.numpy(),
                               1, 1, 1, with_bias=False)
    xc = x.to(cuda).contiguous(memory_format=torch.channels_last)
    offc, maskc = off.to(cuda), mask.to(cuda)
    M = B * H * W
    go = gout.to(cuda).permute(0, 2, 3, 1).reshape(M, Cout)
    dcol = (go @ w.to(cuda).permute(0, 2, 3, 1).reshape(Cout, 9 * C)).contiguous()
    gx = torch.zeros(B, C, H, W, device=cuda).contiguous(memory_format=torch.channels_last)
    goff = torch.zeros_like(offc)
    gm = torch.zeros_like(maskc)
    a = cabi.DcnCol2imArgs()
    a.problem = problem(xc, offc, maskc, gx, 1, (3, 3), (1, 1), (1, 1), (1, 1))
    a.col_dtype = DT[torch.float32]
    a.col_strides[0], a.col_strides[1], a.col_strides[2] = 9 * C, 1, C
    for i in range(4):
        a.grad_input_strides[i] = gx.stride(i)
        a.grad_offset_strides[i] = goff.stride(i)
        a.grad_mask_strides[i] = gm.stride(i)
    L = cabi.lib()
    cabi.check(L.bevk_dcn_col2im(ctypes.byref(a), xc.data_ptr(), offc.data_ptr(),
                                 maskc.data_ptr(), dcol.data_ptr(), gx.data_ptr(),
                                 goff.data_ptr(), gm.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream), "dcn_col2im")
    for got, ref in zip((gx, goff, gm), want[:3]):
        assert rel_l2(got, torch.from_numpy(ref)) <= FP32_REL


HALF_CASES = [
    # B, C, H, W, Cout, big_frac
    (2, 64, 10, 13, 64, 0.0),
    (1, 128, 8, 9, 320, 0.05),
    (2, 24, 7, 6, 40, 0.0),
]


@pytest.mark.parametrize("case", HALF_CASES, ids=[f"h{i}" for i in range(len(HALF_CASES))])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("layout", ["nchw", "nhwc"])
def test_function_backward_half(cuda, case, dt, layout):
    import modulated_deform_conv as mdc
    B, C, H, W, Cout, big = case
    x, off, mask, w, b = dcn_inputs(41, B, C, H, W, Cout, big_frac=big)
    gout = torch.randn(B, Cout, H, W, generator=torch.Generator().manual_seed(42))
    xs, offs, masks, ws, bs, gouts = (t.to(dt) for t in (x, off, mask, w, b, gout))
    want = oracle.dcn_backward(*(t.float().numpy() for t in (xs, offs, masks, ws, gouts)),
                               1, 1, 1)
    xg = xs.to(cuda)
    if layout == "nhwc":
        xg = xg.contiguous(memory_format=torch.channels_last)
    tens = [xg.requires_grad_(), offs.to(cuda).requires_grad_(),
            masks.to(cuda).requires_grad_(), ws.to(cuda).requires_grad_(),
            bs.to(cuda).requires_grad_()]
    out = mdc.modulated_deform_conv2d(*tens, 1, 1, 1)
    out.backward(gouts.to(cuda))
    for t, ref, name in zip(tens, want, ("x", "offset", "mask", "weight", "bias")):
        assert t.grad.dtype == dt
        assert rel_l2(t.grad, torch.from_numpy(ref)) <= HALF_REL, (name, rel_l2(t.grad, torch.from_numpy(ref)))


def test_needs_input_grad_subsets(cuda):
    """Only the requested gradients are produced (frozen weight, fixed offsets)."""
    import modulated_deform_conv as mdc
    x, off, mask, w, b = dcn_inputs(51, 1, 16, 8, 8, 8)
    xg = x.to(cuda).requires_grad_()
    out = mdc.modulated_deform_conv2d(xg, off.to(cuda), mask.to(cuda), w.to(cuda), b.to(cuda),
                                      1, 1, 1)
    gout = torch.randn_like(out)
    out.backward(gout)
    want = oracle.dcn_backward(x.numpy(), off.numpy(), mask.numpy(), w.numpy(),
                               gout.cpu().numpy(), 1, 1, 1)
    assert rel_l2(xg.grad, torch.from_numpy(want[0])) <= FP32_REL


def test_split_nhwc_backward(cuda):
    """dcn_split_nhwc (offset conv + fused sigmoid mask) against the oracle's
    DCN backward chained with autograd of the offset convolution, fp32."""
    import torch.nn.functional as F
    from modulated_deform_conv import dcn_split_nhwc
    g = torch.Generator().manual_seed(61)
    B, C, H, W, Cout, T = 2, 32, 9, 10, 24, 9
    x = torch.randn(B, H, W, C, generator=g)
    w_off = torch.randn(3 * T, C, 3, 3, generator=g) * 0.05
    b_off = torch.randn(3 * T, generator=g) * 0.5
    w = torch.randn(Cout, C, 3, 3, generator=g) * 0.1
    b = torch.randn(Cout, generator=g)
    gout = torch.randn(B, H, W, Cout, generator=g)
    # composite CPU reference
    xr, wor, bor = (t.clone().requires_grad_() for t in (x, w_off, b_off))
    y = F.conv2d(xr.permute(0, 3, 1, 2), wor, bor, 1, 1, 1)
    offset, logit = y[:, :2 * T], y[:, 2 * T:]
    mask = torch.sigmoid(logit)
    gx_d, goff, gmask, gw, gb = oracle.dcn_backward(
        x.permute(0, 3, 1, 2).numpy(), offset.detach().numpy(), mask.detach().numpy(),
        w.numpy(), gout.permute(0, 3, 1, 2).numpy(), 1, 1, 1)
    torch.autograd.backward([offset, mask], [torch.from_numpy(goff), torch.from_numpy(gmask)])
    want_x = xr.grad + torch.from_numpy(gx_d).permute(0, 2, 3, 1)
    # GPU; the offset convolution is cuDNN's, which runs fp32 convs as TF32 by
    # default -- switched off so that it matches the fp32 CPU reference
    tens = [t.to(cuda).requires_grad_() for t in (x, w_off, b_off, w, b)]
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        out = dcn_split_nhwc(*tens, 1, 1, 1)
        out.backward(gout.to(cuda))
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    for got, want, name in ((tens[0].grad, want_x, "x"), (tens[1].grad, wor.grad, "w_off"),
                            (tens[2].grad, bor.grad, "b_off"),
                            (tens[3].grad, torch.from_numpy(gw), "weight"),
                            (tens[4].grad, torch.from_numpy(gb), "bias")):
        assert rel_l2(got, want) <= 2e-5, (name, rel_l2(got, want))


def _split_reference(x, w_off, b_off, w, b, bn_scale, bn_shift):
    """CPU composite: offset conv (torch, fp32), oracle DCN forward, BN affine, ReLU."""
    import torch.nn.functional as F
    T = 9
    y = F.conv2d(x.permute(0, 3, 1, 2).float(), w_off.float(), b_off.float(), 1, 1, 1)
    off, mask = y[:, :2 * T], torch.sigmoid(y[:, 2 * T:])
    z = torch.from_numpy(oracle.dcn_forward(x.permute(0, 3, 1, 2).float().numpy(),
                                            off.numpy(), mask.numpy(), w.float().numpy(),
                                            b.float().numpy(), 1, 1, 1))
    z = z * bn_scale.float().view(1, -1, 1, 1) + bn_shift.float().view(1, -1, 1, 1)
    return torch.relu(z).permute(0, 2, 3, 1), y, off, mask


@pytest.mark.parametrize("dt", [torch.float32, torch.float16], ids=["f32_simt", "f16_tc"])
def test_split_nhwc_bn_relu_epilogue(cuda, dt):
    """FrozenBN folded into weight / bias and the ReLU applied in the kernel's
    epilogue (dcn_split_nhwc.py:185-199)."""
    from modulated_deform_conv import dcn_split_nhwc
    g = torch.Generator().manual_seed(71)
    B, C, H, W, Cout, T = 2, 64, 9, 10, 64, 9
    x = torch.randn(B, H, W, C, generator=g)
    w_off = torch.randn(3 * T, C, 3, 3, generator=g) * 0.03
    b_off = torch.randn(3 * T, generator=g) * 0.5
    w = torch.randn(Cout, C, 3, 3, generator=g) * 0.05
    b = torch.randn(Cout, generator=g)
    scale = torch.rand(Cout, generator=g) + 0.5
    shift = torch.randn(Cout, generator=g)
    xs, wos, bos, ws, bs = (t.to(dt) for t in (x, w_off, b_off, w, b))
    want = _split_reference(xs, wos, bos, ws, bs, scale, shift)[0]
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        out = dcn_split_nhwc(*(t.to(cuda) for t in (xs, wos, bos, ws, bs)), 1, 1, 1,
                             scale.to(cuda), shift.to(cuda), True)
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    assert (out >= 0).all()
    tol = FP32_REL * 3 if dt == torch.float32 else HALF_REL
    assert rel_l2(out.float(), want) <= tol, rel_l2(out.float(), want)


def test_split_nhwc_bn_relu_backward(cuda):
    """Backward through the folded BN + ReLU epilogue: dO is masked by the ReLU
    and scaled by the BN scale (dcn_split_nhwc.py:256-266), fp32."""
    from modulated_deform_conv import dcn_split_nhwc
    g = torch.Generator().manual_seed(72)
    B, C, H, W, Cout, T = 1, 16, 8, 9, 12, 9
    x = torch.randn(B, H, W, C, generator=g)
    w_off = torch.randn(3 * T, C, 3, 3, generator=g) * 0.05
    b_off = torch.randn(3 * T, generator=g) * 0.5
    w = torch.randn(Cout, C, 3, 3, generator=g) * 0.1
    b = torch.randn(Cout, generator=g)
    scale = torch.rand(Cout, generator=g) + 0.5
    shift = torch.randn(Cout, generator=g) * 0.2
    gout = torch.randn(B, H, W, Cout, generator=g)
    out_ref, y, off, mask = _split_reference(x, w_off, b_off, w, b, scale, shift)
    dz = (gout * (out_ref > 0)).permute(0, 3, 1, 2) * scale.view(1, -1, 1, 1)   # d/d(conv+bias)
    gx, goff, gmask, gw, gb = oracle.dcn_backward(
        x.permute(0, 3, 1, 2).numpy(), off.numpy(), mask.numpy(), w.numpy(), dz.numpy(), 1, 1, 1)
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        tens = [t.to(cuda).requires_grad_() for t in (x, w, b)]
        out = dcn_split_nhwc(tens[0], w_off.to(cuda), b_off.to(cuda), tens[1], tens[2], 1, 1, 1,
                             scale.to(cuda), shift.to(cuda), True)
        out.backward(gout.to(cuda))
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    assert rel_l2(tens[1].grad, torch.from_numpy(gw)) <= 2e-5
    assert rel_l2(tens[2].grad, torch.from_numpy(gb)) <= 2e-5
