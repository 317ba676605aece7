"""NHWC DCNv2 entry points, forward and backward (the reference's default
"fuse_c" backend surface,
``modulated_deform_conv/dcn_split_nhwc.py``).

Layouts follow the reference: x [B, H, W, Cin], offset-conv weight
w_off [3T, Cin, kH, kW] (T = kH*kW), b_off [3T], weight [Cout, Cin, kH, kW],
output [B, Ho, Wo, Cout].  The offset/mask convolution (3T output channels)
runs for fp16/bf16 NHWC input as one GEMM with fp32 output plus this
library's tap-sum kernel (offset_conv; cuDNN's implicit GEMM is a poor fit
for 27 output channels), elsewhere as a cuDNN conv as in the reference
(dcn_split_nhwc.py:171).  Its output y feeds the fused kernel directly --
offsets from channels [0, 2T), the mask sigmoid applied on load to channels
[2T, 3T) -- and the deformable gather + contraction run as one kernel with no
column matrix in HBM.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .modulated_deform_conv import (_load_ext, _ones_pad, _tap_major_weight, dcn_forward_into,
                                    offset_conv, tensor_cache_key)


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
    (the epilogue folding of dcn_split_nhwc.py:185-199).  Cached on the weight
    tensor, keyed by the version counters and storage addresses of all four
    inputs (FrozenBN buffers and inference weights do not change between
    calls; the reference folds on every call)."""
    srcs = (bias, bn_scale, bn_shift)
    key = (tensor_cache_key(weight),
           tuple(None if t is None else tensor_cache_key(t) for t in srcs))
    cached = getattr(weight, "_bevk_bn_fold", None)
    if (cached is not None and cached[0] == key
            and all(a is b for a, b in zip(cached[1], srcs))):
        return cached[2]
    w_eff = weight.detach() * bn_scale.to(weight.dtype).view(-1, 1, 1, 1)
    b_eff = bn_shift if bias is None else bn_shift + bn_scale * bias.to(bn_shift.dtype)
    try:
        weight._bevk_bn_fold = (key, srcs, (w_eff, b_eff))
    except (AttributeError, RuntimeError):
        pass
    return w_eff, b_eff


def offset_conv_supported(x_nhwc, kernel_size):
    """Whether offset_conv (GEMM + tap sum) replaces cuDNN: contiguous NHWC
    fp16/bf16 on CUDA with kH*kW <= 9.  At the stage-4 shape on B200 it takes
    ~12 us against cuDNN's 21 us."""
    kh, kw = (kernel_size, kernel_size) if isinstance(kernel_size, int) else kernel_size
    return (x_nhwc.is_cuda and x_nhwc.dtype in (torch.float16, torch.bfloat16)
            and x_nhwc.is_contiguous() and kh * kw <= 9)


def _forward_nhwc(x_nhwc, w_off, b_off, weight, bias, stride, padding, dilation,
                  bn_scale=None, bn_shift=None, act_relu=False, gemm_offset=True):
    B, H, W, Cin = x_nhwc.shape
    Cout, _, kH, kW = weight.shape
    T = kH * kW
    Ho = out_size(H, padding, dilation, kH, stride)
    Wo = out_size(W, padding, dilation, kW, stride)
    x_view = x_nhwc.permute(0, 3, 1, 2)                       # [B, Cin, H, W] channels-last view
    if bn_scale is not None:
        weight, bias = _fold_bn(weight, bias, bn_scale, bn_shift)
    weight = weight.to(x_nhwc.dtype)
    bias = None if bias is None else bias.to(x_nhwc.dtype)
    relu = bn_scale is not None and bool(act_relu)
    out = torch.empty(B, Ho, Wo, Cout, device=x_nhwc.device, dtype=x_nhwc.dtype)
    if gemm_offset and B > 0 and offset_conv_supported(x_nhwc, (kH, kW)):
        # [B, 3T, Ho, Wo] view of the [B, Ho, Wo, 3T] offset-conv output
        y = offset_conv(x_nhwc, w_off, b_off, stride, padding, dilation).permute(0, 3, 1, 2)
    else:
        y = F.conv2d(x_view, w_off, b_off, stride, padding, dilation)   # [B, 3T, Ho, Wo]
    # the FrozenBN affine is folded into weight / bias; its ReLU runs in the
    # kernel's epilogue
    dcn_forward_into(x_view, y[:, :2 * T], y[:, 2 * T:], weight, bias, out.permute(0, 3, 1, 2),
                     stride, padding, dilation, mask_is_logit=True, act_relu=relu)
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
        ctx.stride, ctx.padding, ctx.dilation = stride, padding, dilation
        ctx.with_bias = bias is not None
        ctx.has_bn = bn_scale is not None
        ctx.act_relu = bool(act_relu) and ctx.has_bn
        saved = [x_nhwc, y, w_off, weight]
        if ctx.has_bn:
            saved.append(bn_scale)
            if ctx.act_relu:
                saved.append(out > 0)
        ctx.save_for_backward(*saved)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        """dcn_split_nhwc.py:231-291: the BN scale and ReLU mask are folded into
        dO; dCol = dO . W_flat^T (torch.mm); the scatter kernel reads offsets
        and the pre-sigmoid mask straight from the offset-conv output y and
        returns the mask gradient with the sigmoid backward applied;
        grad_weight = Col^T . dO with Col re-gathered; the offset conv's own
        backward is a regular convolution backward."""
        import torch.nn.grad as tnng
        ext = _load_ext()
        saved = list(ctx.saved_tensors)
        x, y, w_off, weight = saved[:4]
        bn_scale = saved[4] if ctx.has_bn else None
        relu_mask = saved[5] if ctx.act_relu else None
        st, pd, dl = ctx.stride, ctx.padding, ctx.dilation
        Cout, _, kH, kW = weight.shape
        B, H, W, Cin = x.shape
        if B == 0:
            # an empty batch: zero gradients
            return (torch.zeros_like(x), torch.zeros_like(w_off),
                    torch.zeros(w_off.shape[0], device=x.device, dtype=w_off.dtype),
                    torch.zeros_like(weight), torch.zeros(Cout, device=x.device, dtype=x.dtype)
                    if ctx.with_bias else None, None, None, None, None, None, None)
        T = kH * kW
        Ho = out_size(H, pd, dl, kH, st)
        Wo = out_size(W, pd, dl, kW, st)
        M = B * Ho * Wo
        K = T * Cin
        dt = x.dtype
        go = grad_out.reshape(M, Cout)
        if ctx.has_bn:
            if ctx.act_relu:
                go = go * relu_mask.reshape(M, Cout)
            go = go * bn_scale.to(go.dtype).view(1, -1)
        dO = go.to(dt)
        w_tap = _tap_major_weight(weight, dt)                             # [Cout, K], k = t*Cin + c
        dcol = torch.mm(dO, w_tap)                                        # [M, K]
        xc = x.contiguous()
        # fp32 gradients: gX meets the offset conv's input gradient, gOff /
        # gMask (one [B, Ho, Wo, 3T] buffer, the offset conv's dY) feed its
        # backward
        gX = torch.empty(B, H, W, Cin, device=x.device, dtype=torch.float32)
        dY_nhwc = torch.empty(B, Ho, Wo, 3 * T, device=x.device, dtype=torch.float32)
        # with a bias, 8 more columns [1, 0, ..., 0]: the grad_weight GEMM then
        # also returns the column sums of dO (grad_bias)
        Kc = K + 8 if ctx.with_bias else K
        cols = torch.empty(M, Kc, device=x.device, dtype=dt)
        # offsets and pre-sigmoid mask read straight from the offset-conv output
        done = ext.dcn_backward_data(
            dcol, xc.permute(0, 3, 1, 2), y[:, :2 * T], y[:, 2 * T:], True, Cin, H, W, kH, kW,
            st, st, pd, pd, dl, dl, 1, gX.permute(0, 3, 1, 2),
            dY_nhwc[..., :2 * T].permute(0, 3, 1, 2), dY_nhwc[..., 2 * T:].permute(0, 3, 1, 2),
            cols[:, :K])
        if done:
            gOff, gMask = dY_nhwc[..., :2 * T], dY_nhwc[..., 2 * T:]
            if Kc > K:
                cols[:, K:].copy_(_ones_pad(dt, x.device).expand(M, 8))
        else:
            y_nhwc = y.permute(0, 2, 3, 1).contiguous()                   # [B, Ho, Wo, 3T]
            gX.zero_()
            gOff = torch.zeros(B, Ho, Wo, 2 * T, device=x.device, dtype=torch.float32)
            gMask = torch.zeros(B, Ho, Wo, T, device=x.device, dtype=torch.float32)
            ext.modulated_deformable_col2im_nhwc_cuda(
                dcol, xc, y_nhwc, y_nhwc, B, Cin, H, W, Ho, Wo, kH, kW, pd, pd, st, st,
                dl, dl, 1, gX, gOff, gMask)
            cols = gather_cols_nhwc(x, y_nhwc, None, kH, kW, st, pd, dl)  # [M, K]
        # fp16/bf16 operands, fp32 products and accumulation: the reference's
        # fp32 GEMM of the up-cast operands without the up-cast copies
        gw32 = (torch.mm(cols.t(), dO, out_dtype=torch.float32)
                if dt in (torch.float16, torch.bfloat16) else torch.mm(cols.t().float(), dO.float()))
        grad_bias = None
        if ctx.with_bias:
            grad_bias = (gw32[K] if cols.shape[1] > K else dO.sum(0, dtype=torch.float32)).to(dt)
        grad_weight = gw32[:K] \
            .view(kH, kW, Cin, Cout).permute(3, 2, 0, 1).contiguous().to(dt)
        # offset / mask convolution backward (regular convolution)
        dY = (dY_nhwc if done else torch.cat([gOff, gMask], dim=-1)) \
            .permute(0, 3, 1, 2).contiguous()                            # [B, 3T, Ho, Wo]
        x_nchw = x.permute(0, 3, 1, 2).float()
        w_off_f = w_off.float()
        grad_x_off = tnng.conv2d_input(x_nchw.shape, w_off_f, dY, st, pd, dl)
        grad_w_off = tnng.conv2d_weight(x_nchw, w_off_f.shape, dY, st, pd, dl)
        grad_b_off = dY.sum(dim=(0, 2, 3))
        grad_x = (gX + grad_x_off.permute(0, 2, 3, 1)).to(dt)
        return (grad_x, grad_w_off.to(w_off.dtype), grad_b_off.to(w_off.dtype), grad_weight,
                grad_bias, None, None, None, None, None, None)


def dcn_split_nhwc(x_nhwc, w_off, b_off, weight, bias=None, stride=1, padding=1, dilation=1,
                   bn_scale=None, bn_shift=None, act_relu=False):
    """Autograd-enabled NHWC DCNv2 (dcn_split_nhwc.py:294-301)."""
    return DCNSplitNHWCFunction.apply(x_nhwc, w_off, b_off, weight, bias, stride, padding,
                                      dilation, bn_scale, bn_shift, act_relu)


def _as_int(v, what):
    """One value for both axes.  The reference keeps the first component of a
    pair (dcn_split_nhwc.py:306-307), which silently computes a different
    convolution when the two differ; this build refuses such a pair."""
    if isinstance(v, (tuple, list)):
        if len(v) != 2 or v[0] != v[1]:
            raise ValueError(f"dcn_apply_nchw: {what}={tuple(v)} differs between the axes; the "
                             "NHWC path takes one value for both (use "
                             "modulated_deform_conv2d for asymmetric geometry)")
        return v[0]
    return v


def dcn_apply_nchw(x_nchw, w_off, b_off, weight, bias=None, stride=1, padding=1, dilation=1,
                   bn_scale=None, bn_shift=None, act_relu=False):
    """NCHW-in / NCHW-out adapter over the NHWC path (dcn_split_nhwc.py:310-329).

    A channels_last input is viewed as NHWC without a copy and the output is
    returned channels_last; a contiguous NCHW input is copied to NHWC first and
    the output returned contiguous, matching the reference.
    """
    s, p, d = _as_int(stride, "stride"), _as_int(padding, "padding"), _as_int(dilation,
                                                                               "dilation")
    is_cl = x_nchw.is_contiguous(memory_format=torch.channels_last)
    x_nhwc = x_nchw.permute(0, 2, 3, 1)
    if not is_cl:
        x_nhwc = x_nhwc.contiguous()
    out_nhwc = dcn_split_nhwc(x_nhwc, w_off, b_off, weight, bias, s, p, d, bn_scale, bn_shift,
                              act_relu)
    out = out_nhwc.permute(0, 3, 1, 2)
    return out if is_cl else out.contiguous()
