"""BEVFormer's own DCN entry points on real data: ModulatedDeformConv2dPack.forward
(reference modulated_deform_conv/modulated_deform_conv.py:584-626) and
dcn_apply_nchw (modulated_deform_conv/dcn_split_nhwc.py:306-329), against the
unfused CPU composite of the same computation:

    y      = conv_offset(x)            fp32 F.conv2d on the up-cast inputs, rounded
                                       to the input dtype (what the reference's
                                       cuDNN offset conv returns)
    offset = y[:, :2T]                 (chunk(3) + cat of the first two chunks)
    mask   = sigmoid(y[:, 2T:])
    out    = oracle.dcn_forward(x, offset, mask, weight, bias)

for NCHW-contiguous and channels_last input (the output follows the input's
memory format), at BASELINE configs 2 (fp16) and 3 (bf16, offsets pushed out
of the image) full size, with the folded FrozenBN + ReLU epilogue, and for the
grouped / deformable-grouped module (the branch that calls
modulated_deform_conv2d), forward and backward.

Tolerances: fp16/bf16 in -> within 5e-3 relative L2 of the fp32 composite;
fp32 within 1e-5 relative L2 and 1e-4 max-abs.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from helpers import FP32_ABS, FP32_REL, HALF_REL, max_abs, rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _exact_offset_conv():
    """fp32 offset convolutions on cuDNN without TF32 (torch's default allows
    it), so the fp32 cases compare the DCN, not TF32 rounding of the offsets."""
    old = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cudnn.allow_tf32 = old


# BASELINE configs 2 and 3 (B, C, H, W, Cout, dtype, out-of-image offset bias)
CFGS = {
    "cfg2": (6, 512, 29, 50, 512, torch.float16, 0.0),
    "cfg3": (6, 256, 58, 100, 256, torch.bfloat16, 62.0),
}


def _pack_module(seed, C, Cout, dt, device, far=0.0, bias=False, **kw):
    """A Pack module with BEVFormer's geometry whose offset conv yields offsets
    of ~2 px and mask logits ~N(0, 1); with ``far``, the Δh of tap 0 (one of
    the 18 offset channels) is pushed ``far`` pixels down and the Δw of tap 8
    ``far`` pixels left, out of the image."""
    from modulated_deform_conv import ModulatedDeformConv2dPack
    torch.manual_seed(seed)
    m = ModulatedDeformConv2dPack(C, Cout, 3, stride=kw.get("stride", 1),
                                  padding=kw.get("padding", 1), dilation=kw.get("dilation", 1),
                                  groups=kw.get("groups", 1),
                                  deform_groups=kw.get("deform_groups", 1), bias=bias)
    g = torch.Generator().manual_seed(seed + 1)
    cin_g = C // m.groups
    with torch.no_grad():
        m.weight.copy_(torch.randn(m.weight.shape, generator=g) * math.sqrt(2.0 / (cin_g * 9)))
        if bias:
            m.bias.copy_(torch.randn(Cout, generator=g))
        w_off = torch.randn(m.conv_offset.weight.shape, generator=g) / math.sqrt(C * 9)
        n_off = 2 * m.deform_groups * 9
        w_off[:n_off] *= 2.0                      # offsets ~N(0, 2^2) px
        m.conv_offset.weight.copy_(w_off)
        b_off = torch.randn(m.conv_offset.bias.shape, generator=g) * 0.1
        b_off[0] += far
        b_off[17] -= far
        m.conv_offset.bias.copy_(b_off)
    return m.to(device=device, dtype=dt)


def _composite(x, m, y=None):
    """The unfused CPU composite of the module's forward -> fp32 NCHW.  With
    ``y``, the offset-conv output the module produced is used as is."""
    with torch.no_grad():
        xf = x.detach().float().cpu()
        if y is None:
            y = F.conv2d(xf, m.conv_offset.weight.detach().float().cpu(),
                         m.conv_offset.bias.detach().float().cpu(), m.stride, m.padding,
                         m.dilation)
            y = y.to(x.dtype)
        y = y.detach().float().cpu()
        n = 2 * m.deform_groups * m.kernel_size[0] * m.kernel_size[1]
        offset, mask = y[:, :n], torch.sigmoid(y[:, n:])
        b = None if m.bias is None else m.bias.detach().float().cpu().numpy()
        out = oracle.dcn_forward(xf.numpy(), offset.numpy(), mask.numpy(),
                                 m.weight.detach().float().cpu().numpy(), b, m.stride, m.padding,
                                 m.dilation, m.groups, m.deform_groups)
    return torch.from_numpy(out), offset, mask


def _input(seed, B, C, H, W, dt, device, channels_last):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, C, H, W, generator=g).to(dt).to(device)
    return x.contiguous(memory_format=torch.channels_last) if channels_last else x


@pytest.mark.parametrize("channels_last", [False, True], ids=["nchw", "channels_last"])
@pytest.mark.parametrize("cfg", ["cfg2", "cfg3"])
def test_pack_forward_full_size_matches_composite(cuda, cfg, channels_last):
    B, C, H, W, Cout, dt, far = CFGS[cfg]
    m = _pack_module(11, C, Cout, dt, cuda, far=far)
    x = _input(12, B, C, H, W, dt, cuda, channels_last)
    with torch.no_grad():
        out = m(x)
    torch.cuda.synchronize()
    assert out.shape == (B, Cout, H, W) and out.dtype == dt
    # the output keeps the input's memory format (dcn_split_nhwc.py:322-329)
    if channels_last:
        assert out.is_contiguous(memory_format=torch.channels_last)
    else:
        assert out.is_contiguous()
    want, offset, _ = _composite(x, m)
    if far:
        # the pushed taps really leave the image (tap 0 samples row ho - 1 + Δh)
        assert float((offset[:, 0] > H + 1).float().mean()) > 0.9
        assert float((offset[:, 17] < -(H + 1)).float().mean()) > 0.9
    r = rel_l2(out, want)
    assert r <= HALF_REL, r


@pytest.mark.parametrize("channels_last", [False, True], ids=["nchw", "channels_last"])
def test_dcn_apply_nchw_bn_relu_matches_composite(cuda, channels_last):
    """dcn_apply_nchw with a bias and the folded FrozenBN + ReLU epilogue
    (dcn_split_nhwc.py:185-199): relu(scale * (dcn(x) + b) + shift)."""
    from modulated_deform_conv import dcn_apply_nchw
    B, C, H, W, Cout, dt = 2, 128, 21, 30, 192, torch.float16
    m = _pack_module(21, C, Cout, dt, cuda, bias=True)
    x = _input(22, B, C, H, W, dt, cuda, channels_last)
    g = torch.Generator().manual_seed(23)
    scale = (torch.rand(Cout, generator=g) + 0.5).to(cuda)
    shift = (torch.randn(Cout, generator=g) * 0.1).to(cuda)
    with torch.no_grad():
        out = dcn_apply_nchw(x, m.conv_offset.weight, m.conv_offset.bias, m.weight, m.bias,
                             1, 1, 1, scale, shift, True)
    assert out.is_contiguous(memory_format=torch.channels_last if channels_last
                             else torch.contiguous_format)
    conv, _, _ = _composite(x, m)
    want = torch.relu(scale.cpu().view(1, -1, 1, 1) * conv + shift.cpu().view(1, -1, 1, 1))
    r = rel_l2(out, want)
    assert r <= HALF_REL, r
    # the ReLU really clips: about half the outputs are exactly zero
    assert 0.2 < float((out == 0).float().mean()) < 0.8


def test_dcn_apply_nchw_rejects_asymmetric_geometry(cuda):
    from modulated_deform_conv import dcn_apply_nchw
    m = _pack_module(31, 16, 16, torch.float16, cuda)
    x = _input(32, 1, 16, 8, 8, torch.float16, cuda, False)
    with pytest.raises(ValueError, match="stride"):
        dcn_apply_nchw(x, m.conv_offset.weight, m.conv_offset.bias, m.weight, None, (1, 2), 1, 1)
    # a pair with equal components is one value for both axes
    out = dcn_apply_nchw(x, m.conv_offset.weight, m.conv_offset.bias, m.weight, None, (1, 1),
                         (1, 1), (1, 1))
    assert out.shape == (1, 16, 8, 8)


def test_pack_asymmetric_stride_takes_the_general_path(cuda):
    """stride (1, 2): the module computes the asymmetric convolution (the
    reference's NHWC path would silently use stride 1 on both axes)."""
    dt = torch.float32
    m = _pack_module(41, 24, 40, dt, cuda, stride=(1, 2), bias=True)
    x = _input(42, 2, 24, 11, 14, dt, cuda, False)
    with torch.no_grad():
        out = m(x)
    assert out.shape == (2, 40, 11, 7)
    want, _, _ = _composite(x, m)
    assert rel_l2(out, want) <= FP32_REL and max_abs(out, want) <= FP32_ABS


GROUP_CASES = [
    # dtype, B, C, H, W, Cout, groups, deform_groups, channels_last
    (torch.float32, 2, 32, 9, 12, 48, 2, 2, False),
    (torch.float16, 2, 64, 10, 13, 64, 2, 2, True),
]


@pytest.mark.parametrize("case", GROUP_CASES, ids=["f32_g2_dg2", "f16_g2_dg2_cl"])
def test_pack_groups_forward_backward_match_oracle(cuda, case):
    """The grouped module's branch (conv_offset, chunk, cat, sigmoid,
    ModulatedDeformConv2dFunction; modulated_deform_conv.py:610-626), forward
    and .backward(), against the oracle's forward and backward chained through
    the sigmoid and the offset convolution's own gradients (torch autograd in
    fp64 on the CPU).  The oracle takes the offsets and mask logits the
    module's offset conv (cuDNN) produced: a rounding difference there moves
    a sample across a pixel boundary, where the offset gradient jumps."""
    dt, B, C, H, W, Cout, groups, dg, cl = case
    m = _pack_module(51, C, Cout, dt, cuda, bias=True, groups=groups, deform_groups=dg)
    x = _input(52, B, C, H, W, dt, cuda, cl).requires_grad_()
    out = m(x)
    gout = torch.randn(out.shape, generator=torch.Generator().manual_seed(53)).to(dt)
    out.backward(gout.to(cuda))
    with torch.no_grad():
        y_gpu = m.conv_offset(x)
    torch.cuda.synchronize()

    want, offset, mask = _composite(x.detach(), m, y_gpu)
    tol = (lambda a, b: rel_l2(a, b) <= FP32_REL and max_abs(a, b) <= FP32_ABS * max(
        1.0, float(b.abs().max()))) if dt == torch.float32 else (
        lambda a, b: rel_l2(a, b) <= HALF_REL)
    assert tol(out, want), rel_l2(out, want)

    xf = x.detach().float().cpu()
    gx, goff, gm, gw, gb = oracle.dcn_backward(
        xf.numpy(), offset.numpy(), mask.numpy(), m.weight.detach().float().cpu().numpy(),
        gout.float().numpy(), m.stride, m.padding, m.dilation, groups, dg, with_bias=True)
    # chain through mask = sigmoid(y[:, 2T*dg:]) and y = conv_offset(x)
    gy = torch.cat([torch.from_numpy(goff), torch.from_numpy(gm) * mask * (1 - mask)], 1)
    xd = xf.double().requires_grad_()
    wd = m.conv_offset.weight.detach().double().cpu().requires_grad_()
    bd = m.conv_offset.bias.detach().double().cpu().requires_grad_()
    y = F.conv2d(xd, wd, bd, m.stride, m.padding, m.dilation)
    y.backward(gy.double())
    grads = {
        "x": (x.grad, torch.from_numpy(gx).double() + xd.grad),
        "weight": (m.weight.grad, torch.from_numpy(gw)),
        "bias": (m.bias.grad, torch.from_numpy(gb)),
        "conv_offset.weight": (m.conv_offset.weight.grad, wd.grad),
        "conv_offset.bias": (m.conv_offset.bias.grad, bd.grad),
    }
    for name, (got, ref) in grads.items():
        assert got is not None, name
        assert tol(got, ref), (name, rel_l2(got, ref))
