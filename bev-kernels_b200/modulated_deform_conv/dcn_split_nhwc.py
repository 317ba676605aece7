"""NHWC DCNv2 entry points (the reference's default "fuse_c" backend surface,
``modulated_deform_conv/dcn_split_nhwc.py``).

Layouts follow the reference: x [B, H, W, Cin], offset-conv weight
w_off [3T, Cin, kH, kW] (T = kH*kW), b_off [3T], weight [Cout, Cin, kH, kW],
output [B, Ho, Wo, Cout].  The offset/mask convolution stays a cuDNN conv as in
the reference (dcn_split_nhwc.py:171); its raw output y feeds the fused kernel
directly -- offsets from channels [0, 2T), the mask sigmoid applied on load to
channels [2T, 3T) -- and the deformable gather + contraction run as one kernel
with no column matrix in HBM.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .modulated_deform_conv import _load_ext, dcn_forward_into


def out_size(H, pad, dil, k, stride):
    return (H + 2 * pad - (dil * (k - 1) + 1)) // stride + 1


def gather_cols_nhwc(x_nhwc, offset, mask=None, kH=3, kW=3, stride=1, padding=1, dilation=1):
    """Deformable gather -> Col [M, T*Cin] with k = t*Cin + ci
    (dcn_split_nhwc.py:21-45).  ``offset`` is either [B, Ho, Wo, 2T] with a
    post-sigmoid ``mask`` [B, Ho, Wo, T], or the raw offset-conv output
    y [B, Ho, Wo, 3T] with ``mask=None`` (sigmoid applied on load)."""
    ext = _load_ext()
    B, H, W, Cin = x_nhwc.shape
    T = kH * kW
    Ho = out_size(H, padding, dilation, kH, stride)
    Wo = out_size(W, padding, dilation, kW, stride)
    off_c = offset.contiguous()
    mask_c = (mask if mask is not None else offset).contiguous()
    col = torch.empty(B * Ho * Wo, T * Cin, device=x_nhwc.device, dtype=x_nhwc.dtype)
    ext.modulated_deformable_im2col_nhwc_cuda(
        x_nhwc.contiguous(), off_c, mask_c, B, Cin, H, W, Ho, Wo, kH, kW, padding, padding,
        stride, stride, dilation, dilation, 1, col)
    return col


def _fold_bn(weight, bias, bn_scale, bn_shift):
    """relu(scale*(conv(x, w) + b) + shift) == relu(conv(x, w*scale) + (shift + scale*b))
    (the epilogue folding of dcn_split_nhwc.py:185-199)."""
    w_eff = weight * bn_scale.to(weight.dtype).view(-1, 1, 1, 1)
    b_eff = bn_shift if bias is None else bn_shift + bn_scale * bias.to(bn_shift.dtype)
    return w_eff, b_eff


def _forward_nhwc(x_nhwc, w_off, b_off, weight, bias, stride, padding, dilation,
                  bn_scale=None, bn_shift=None, act_relu=False):
    B, H, W, Cin = x_nhwc.shape
    Cout, _, kH, kW = weight.shape
    T = kH * kW
    Ho = out_size(H, padding, dilation, kH, stride)
    Wo = out_size(W, padding, dilation, kW, stride)
    x_view = x_nhwc.permute(0, 3, 1, 2)                       # [B, Cin, H, W] channels-last view
    y = F.conv2d(x_view, w_off, b_off, stride, padding, dilation)   # [B, 3T, Ho, Wo]
    if bn_scale is not None:
        weight, bias = _fold_bn(weight, bias, bn_scale, bn_shift)
    weight = weight.to(x_nhwc.dtype)
    out = torch.empty(B, Ho, Wo, Cout, device=x_nhwc.device, dtype=x_nhwc.dtype)
    dcn_forward_into(x_view, y[:, :2 * T], y[:, 2 * T:], weight,
                     None if bias is None else bias.to(x_nhwc.dtype), out.permute(0, 3, 1, 2),
                     stride, padding, dilation, mask_is_logit=True)
    if bn_scale is not None and act_relu:
        out.relu_()
    return out, y


def dcn_split_forward_nhwc(x_nhwc, w_off, b_off, weight, bias=None, stride=1, padding=1,
                           dilation=1):
    """Forward-only NHWC DCNv2 (dcn_split_nhwc.py:96-128) -> [B, Ho, Wo, Cout]."""
    return _forward_nhwc(x_nhwc, w_off, b_off, weight, bias, stride, padding, dilation)[0]


class DCNSplitNHWCFunction(torch.autograd.Function):
    """NHWC DCNv2 autograd Function (dcn_split_nhwc.py:131-291).

    Inputs: x_nhwc [B,H,W,Cin], w_off [3T,Cin,kH,kW], b_off [3T], weight
    [Cout,Cin,kH,kW], bias [Cout] or None, stride, padding, dilation, and the
    optional folded FrozenBN(+ReLU) epilogue (bn_scale, bn_shift, act_relu).
    Output: [B,Ho,Wo,Cout].
    """

    @staticmethod
    def forward(ctx, x_nhwc, w_off, b_off, weight, bias, stride, padding, dilation,
                bn_scale=None, bn_shift=None, act_relu=False):
        out, y = _forward_nhwc(x_nhwc, w_off, b_off, weight, bias, stride, padding, dilation,
                               bn_scale, bn_shift, act_relu)
        ctx.save_for_backward(x_nhwc, y, w_off, weight)
        ctx.stride, ctx.padding, ctx.dilation = stride, padding, dilation
        ctx.with_bias = bias is not None
        return out

    @staticmethod
    def backward(ctx, grad_out):
        raise NotImplementedError(
            "bev-kernels_b200: DCNSplitNHWCFunction backward is not built yet "
            "(forward-only release)")


def dcn_split_nhwc(x_nhwc, w_off, b_off, weight, bias=None, stride=1, padding=1, dilation=1,
                   bn_scale=None, bn_shift=None, act_relu=False):
    """Autograd-enabled NHWC DCNv2 (dcn_split_nhwc.py:294-301)."""
    return DCNSplitNHWCFunction.apply(x_nhwc, w_off, b_off, weight, bias, stride, padding,
                                      dilation, bn_scale, bn_shift, act_relu)


def _as_int(v):
    return v[0] if isinstance(v, (tuple, list)) else v


def dcn_apply_nchw(x_nchw, w_off, b_off, weight, bias=None, stride=1, padding=1, dilation=1,
                   bn_scale=None, bn_shift=None, act_relu=False):
    """NCHW-in / NCHW-out adapter over the NHWC path (dcn_split_nhwc.py:310-329).

    A channels_last input is viewed as NHWC without a copy and the output is
    returned channels_last; a contiguous NCHW input is copied to NHWC first and
    the output returned contiguous, matching the reference.
    """
    s, p, d = _as_int(stride), _as_int(padding), _as_int(dilation)
    is_cl = x_nchw.is_contiguous(memory_format=torch.channels_last)
    x_nhwc = x_nchw.permute(0, 2, 3, 1)
    if not is_cl:
        x_nhwc = x_nhwc.contiguous()
    out_nhwc = dcn_split_nhwc(x_nhwc, w_off, b_off, weight, bias, s, p, d, bn_scale, bn_shift,
                              act_relu)
    out = out_nhwc.permute(0, 3, 1, 2)
    return out if is_cl else out.contiguous()
