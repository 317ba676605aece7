"""Modulated deformable convolution (DCNv2) on B200: the reference's operator
surface over the fused sm_100a kernels.

Drop-in for ``modulated_deform_conv/modulated_deform_conv.py`` of the reference
(itself an mmcv drop-in): same class names, argument orders, defaults, parameter
names (checkpoint compatible) and ``_load_from_state_dict`` migration.

Forward does not materialise the column matrix: ``ModulatedDeformConv2dFunction``
calls the fused kernel (``_modulated_deform_conv_ext.dcn_forward``), which
gathers the modulated bilinear samples straight into shared memory and runs the
contraction on tcgen05 tensor cores (fp16/bf16) or as an exact SIMT implicit GEMM
(fp32/fp64, grouped convolutions).  There is no CPU path: CPU tensors raise.
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn as nn
from torch.autograd import Function
from torch.autograd.function import once_differentiable
from torch.nn.modules.utils import _pair, _single

from bevk import load_extension

_ext = None


def _load_ext():
    """The compiled extension (modulated_deform_conv.py:22-27)."""
    global _ext
    if _ext is None:
        _ext = load_extension("_modulated_deform_conv_ext")
    return _ext


def _out_size(n, pad, dil, k, stride):
    return (n + 2 * pad - (dil * (k - 1) + 1)) // stride + 1


# ---------------------------------------------------------------------------
# Column-matrix wrappers (reference: modulated_deform_conv.py:30-68)
# ---------------------------------------------------------------------------

def ext_modulated_deformable_im2col(data_im, data_offset, data_mask, kernel_h, kernel_w,
                                    pad_h, pad_w, stride_h, stride_w, dilation_h, dilation_w,
                                    deformable_group):
    """Column matrix [C*kH*kW, B, Ho, Wo] (modulated_deform_conv.py:30-48)."""
    ext = _load_ext()
    batch_size, channels, height, width = data_im.shape
    height_col = _out_size(height, pad_h, dilation_h, kernel_h, stride_h)
    width_col = _out_size(width, pad_w, dilation_w, kernel_w, stride_w)
    data_col = data_im.new_empty(channels * kernel_h * kernel_w, batch_size, height_col, width_col)
    ext.modulated_deformable_im2col_cuda(
        data_im.contiguous(), data_offset.contiguous(), data_mask.contiguous(),
        batch_size, channels, height, width, height_col, width_col,
        kernel_h, kernel_w, pad_h, pad_w, stride_h, stride_w, dilation_h, dilation_w,
        deformable_group, data_col)
    return data_col


def ext_modulated_deformable_im2col_opt(data_im, data_offset, data_mask, kernel_h, kernel_w,
                                        pad_h, pad_w, stride_h, stride_w, dilation_h, dilation_w,
                                        deformable_group):
    """Same column matrix via the reference's "opt" entry (modulated_deform_conv.py:51-68)."""
    ext = _load_ext()
    batch_size, channels, height, width = data_im.shape
    height_col = _out_size(height, pad_h, dilation_h, kernel_h, stride_h)
    width_col = _out_size(width, pad_w, dilation_w, kernel_w, stride_w)
    data_col = data_im.new_empty(channels * kernel_h * kernel_w, batch_size, height_col, width_col)
    ext.modulated_deformable_im2col_opt_cuda(
        data_im.contiguous(), data_offset.contiguous(), data_mask.contiguous(),
        batch_size, channels, height, width, height_col, width_col,
        kernel_h, kernel_w, pad_h, pad_w, stride_h, stride_w, dilation_h, dilation_w,
        deformable_group, data_col)
    return data_col


def _col2im(entry, data_col, data_offset, data_mask, batch_size, channels, height, width,
            kernel_h, kernel_w, pad_h, pad_w, stride_h, stride_w, dilation_h, dilation_w,
            deformable_group):
    ext = _load_ext()
    height_col = _out_size(height, pad_h, dilation_h, kernel_h, stride_h)
    width_col = _out_size(width, pad_w, dilation_w, kernel_w, stride_w)
    grad_im = data_col.new_zeros(batch_size, channels, height, width)
    getattr(ext, entry)(data_col.contiguous(), data_offset, data_mask, batch_size, channels,
                        height, width, height_col, width_col, kernel_h, kernel_w, pad_h, pad_w,
                        stride_h, stride_w, dilation_h, dilation_w, deformable_group, grad_im)
    return grad_im


def ext_modulated_deformable_col2im(*args):
    """Column gradient [C*kH*kW, B*Ho*Wo] -> grad_im [B, C, H, W]
    (modulated_deform_conv.py:115-134; same arguments)."""
    return _col2im("modulated_deformable_col2im_cuda", *args)


def ext_modulated_deformable_col2im_opt(*args):
    """As ext_modulated_deformable_col2im (modulated_deform_conv.py:73-92)."""
    return _col2im("modulated_deformable_col2im_opt_cuda", *args)


def ext_modulated_deformable_col2im_smem(*args):
    """As ext_modulated_deformable_col2im (modulated_deform_conv.py:94-113)."""
    return _col2im("modulated_deformable_col2im_smem_cuda", *args)


def _col2im_coord(entry, data_col, data_im, data_offset, data_mask, kernel_h, kernel_w, pad_h,
                  pad_w, stride_h, stride_w, dilation_h, dilation_w, deformable_group):
    ext = _load_ext()
    batch_size, channels, height, width = data_im.shape
    height_col = _out_size(height, pad_h, dilation_h, kernel_h, stride_h)
    width_col = _out_size(width, pad_w, dilation_w, kernel_w, stride_w)
    grad_offset = data_offset.new_zeros(data_offset.shape)
    grad_mask = data_mask.new_zeros(data_mask.shape)
    getattr(ext, entry)(data_col.contiguous(), data_im, data_offset, data_mask, batch_size,
                        channels, height, width, height_col, width_col, kernel_h, kernel_w,
                        pad_h, pad_w, stride_h, stride_w, dilation_h, dilation_w,
                        deformable_group, grad_offset, grad_mask)
    return grad_offset, grad_mask


def ext_modulated_deformable_col2im_coord(*args):
    """Column gradient -> (grad_offset, grad_mask) (modulated_deform_conv.py:136-156)."""
    return _col2im_coord("modulated_deformable_col2im_coord_cuda", *args)


def ext_modulated_deformable_col2im_coord_opt(*args):
    """As ext_modulated_deformable_col2im_coord (modulated_deform_conv.py:158-182)."""
    return _col2im_coord("modulated_deformable_col2im_coord_opt_cuda", *args)


# ---------------------------------------------------------------------------
# Packed weights
# ---------------------------------------------------------------------------

# Attributes under which derived copies of a weight are cached on the tensor.
_CACHE_ATTRS = ("_bevk_packed", "_bevk_offset_gemm", "_bevk_tap_major", "_bevk_bn_fold")


def tensor_cache_key(t: torch.Tensor):
    """What a cached copy derived from ``t`` depends on: the version counter
    (in-place updates through autograd-visible ops, e.g. optimizer steps), the
    storage address (``p.data = new_tensor`` swaps, as EMA hooks and some
    checkpoint loaders do, keep the old version counter), dtype, device and
    shape."""
    return (t._version, t.data_ptr(), t.dtype, t.device, tuple(t.shape))


def invalidate_weight_caches(obj) -> None:
    """Drop the derived copies (packed weight, tap-major weight, offset-conv
    GEMM operand, FrozenBN fold) cached on a tensor, or on every parameter
    and buffer of a module.  Needed only after a write the cache key cannot
    see: ``p.data.copy_(t)`` changes neither the version counter nor the
    storage address."""
    tensors = ([obj] if isinstance(obj, torch.Tensor)
               else list(obj.parameters()) + list(obj.buffers()))
    for t in tensors:
        for a in _CACHE_ATTRS:
            if hasattr(t, a):
                try:
                    delattr(t, a)
                except (AttributeError, RuntimeError):
                    pass


def packed_weight(weight: torch.Tensor, groups: int = 1) -> torch.Tensor:
    """[Cout, Cin/groups, kH, kW] -> the kernels' [Cout][kH*kW][Cin_g_pad] layout.

    Cached on the weight tensor and keyed by its version counter and storage
    address (tensor_cache_key), so a module's parameter is packed once per
    optimizer update instead of once per call (the reference permutes and
    copies the weight on every call, dcn_split_nhwc.py:176).  An update that
    neither bumps the version nor moves the storage -- ``p.data.copy_(t)`` --
    is invisible to the key: call ``invalidate_weight_caches`` after it.
    """
    key = (tensor_cache_key(weight), int(groups))
    cached = getattr(weight, "_bevk_packed", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    packed = _load_ext().dcn_pack_weight(weight.detach(), int(groups))
    try:
        weight._bevk_packed = (key, packed)
    except (AttributeError, RuntimeError):  # e.g. tensors that reject attributes
        pass
    return packed


def dcn_forward_into(input, offset, mask, weight, bias, output, stride, padding, dilation,
                     groups=1, deform_groups=1, mask_is_logit=False, act_relu=False):
    """Fused DCNv2 forward writing into ``output`` ([B, Cout, Ho, Wo], any strides).

    ``input``/``offset``/``mask`` may be NCHW-contiguous or channels-last views;
    ``mask_is_logit`` applies the sigmoid on load (raw offset-conv output);
    ``act_relu`` applies max(0, .) in the kernel's epilogue.
    """
    if input.shape[0] == 0:
        return output  # an empty batch: nothing to compute or write
    kh, kw = weight.shape[2], weight.shape[3]
    sh, sw = _pair(stride)
    ph, pw = _pair(padding)
    dh, dw = _pair(dilation)
    _load_ext().dcn_forward(input, offset, mask, packed_weight(weight, groups), bias, output,
                            kh, kw, sh, sw, ph, pw, dh, dw, int(groups), int(deform_groups),
                            bool(mask_is_logit), bool(act_relu))
    return output


def offset_conv_partials(x_nhwc, w_off):
    """Per-tap partial products of the offset convolution, [B*H*W, ld] fp32
    (ld = T*3T rounded up to a multiple of 32): row p, column t*3T + c holds
    sum_ci x[p, ci] * w_off[c, ci, t] -- one GEMM with fp32 output, the
    channel reduction of the Pack module's conv_offset
    (dcn_split_nhwc.py:171-172).  Columns beyond T*3T are zero."""
    B, H, W, Cin = x_nhwc.shape
    return torch.mm(x_nhwc.reshape(B * H * W, Cin), _offset_gemm_weight(w_off, x_nhwc.dtype).t(),
                    out_dtype=torch.float32)


def _offset_gemm_weight(w_off, dtype):
    """w_off [3T, Cin, kH, kW] as the GEMM operand [ld, Cin] (row t*3T + c,
    zero rows up to ld), cached on w_off like packed_weight."""
    key = (tensor_cache_key(w_off), dtype)
    cached = getattr(w_off, "_bevk_offset_gemm", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    c3, cin, kh, kw = w_off.shape
    n = kh * kw * c3
    wz = torch.zeros((n + 31) // 32 * 32, cin, device=w_off.device, dtype=dtype)
    wz[:n] = w_off.detach().permute(2, 3, 0, 1).reshape(n, cin)
    try:
        w_off._bevk_offset_gemm = (key, wz)
    except (AttributeError, RuntimeError):
        pass
    return wz


def offset_conv(x_nhwc, w_off, b_off, stride, padding, dilation):
    """The Pack module's offset convolution (dcn_split_nhwc.py:171-172) as
    [B, Ho, Wo, 3T] in x's dtype: its channel reduction as one GEMM with fp32
    output (offset_conv_partials), then the tap sum, bias and one rounding in
    a kernel of this library (bevk_dcn_offset_conv_sum)."""
    B, H, W, _ = x_nhwc.shape
    c3, _, kh, kw = w_off.shape
    sh, sw = _pair(stride)
    ph, pw = _pair(padding)
    dh, dw = _pair(dilation)
    Ho = (H + 2 * ph - (dh * (kh - 1) + 1)) // sh + 1
    Wo = (W + 2 * pw - (dw * (kw - 1) + 1)) // sw + 1
    y = torch.empty(B, Ho, Wo, c3, device=x_nhwc.device, dtype=x_nhwc.dtype)
    _load_ext().dcn_offset_conv_sum(offset_conv_partials(x_nhwc, w_off), b_off, y, B, H, W,
                                    kh, kw, sh, sw, ph, pw, dh, dw)
    return y


# ---------------------------------------------------------------------------
# autograd Function (reference: modulated_deform_conv.py:318-502)
# ---------------------------------------------------------------------------

class ModulatedDeformConv2dFunction(Function):
    """Drop-in for mmcv.ops.ModulatedDeformConv2dFunction (reference
    modulated_deform_conv.py:318-499).

    Forward: one fused kernel, output [B, Cout, Ho, Wo] contiguous (as the
    reference's permute(...).contiguous(), :396-398) in the input's dtype.
    """

    @staticmethod
    def forward(ctx, input, offset, mask, weight, bias=None, stride=1, padding=0, dilation=1,
                groups=1, deform_groups=1):
        if input is not None and input.dim() != 4:
            raise ValueError(f'Expected 4D tensor as input, got {input.dim()}D tensor instead.')
        ctx.stride = _pair(stride)
        ctx.padding = _pair(padding)
        ctx.dilation = _pair(dilation)
        ctx.groups = groups
        ctx.deform_groups = deform_groups
        ctx.with_bias = bias is not None
        if not ctx.with_bias:
            bias = input.new_empty(0)

        input = input.type_as(offset)
        weight = weight.type_as(input)
        mask = mask.type_as(input)
        ctx.save_for_backward(input, offset, mask, weight, bias)

        batch, _, height, width = input.shape
        channels_out, _, kernel_h, kernel_w = weight.shape
        height_out = _out_size(height, ctx.padding[0], ctx.dilation[0], kernel_h, ctx.stride[0])
        width_out = _out_size(width, ctx.padding[1], ctx.dilation[1], kernel_w, ctx.stride[1])
        output = input.new_empty(batch, channels_out, height_out, width_out)
        dcn_forward_into(input, offset, mask, weight,
                         bias.type_as(input) if ctx.with_bias else None, output,
                         ctx.stride, ctx.padding, ctx.dilation, groups, deform_groups)
        return output

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        input, offset, mask, weight, bias = ctx.saved_tensors
        need = ctx.needs_input_grad
        grads = dcn_backward(input, offset, mask, weight, grad_output, ctx.stride, ctx.padding,
                             ctx.dilation, ctx.groups, ctx.deform_groups,
                             need_input=need[0], need_offset_mask=need[1] or need[2],
                             need_weight=need[3], need_bias=ctx.with_bias and need[4])
        return grads + (None, None, None, None, None)


def _tap_major_weight(weight, dtype):
    """weight [Cout, Cg, kH, kW] as [Cout, kH*kW*Cg] (k = t*Cg + c) in dtype,
    cached on the weight like packed_weight (the backward's dCol GEMM operand)."""
    key = (tensor_cache_key(weight), dtype)
    cached = getattr(weight, "_bevk_tap_major", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    cout, cg, kh, kw = weight.shape
    wt = weight.detach().to(dtype).permute(0, 2, 3, 1).reshape(cout, kh * kw * cg).contiguous()
    try:
        weight._bevk_tap_major = (key, wt)
    except (AttributeError, RuntimeError):
        pass
    return wt


_ONES_PAD = {}


def _ones_pad(dtype, device):
    """[1, 0, 0, 0, 0, 0, 0, 0]: the extra columns that make the grad_weight
    GEMM return grad_bias (cached per dtype and device)."""
    key = (dtype, device)
    t = _ONES_PAD.get(key)
    if t is None:
        t = torch.zeros(8, dtype=dtype, device=device)
        t[0] = 1
        _ONES_PAD[key] = t
    return t


def dcn_backward(input, offset, mask, weight, grad_output, stride, padding, dilation,
                 groups=1, deform_groups=1, need_input=True, need_offset_mask=True,
                 need_weight=True, need_bias=True):
    """Gradients of the DCNv2 forward (modulated_deform_conv.py:405-499) ->
    (grad_input, grad_offset, grad_mask, grad_weight, grad_bias), None where
    not requested.

    The two contractions are plain GEMMs (cuBLAS through torch.mm, as in the
    reference): the column gradient dcol = dO . W^T in pixel-major NHWC order
    [M, kH*kW*C] (k = t*C + c), and grad_weight = dO^T . col.  The deformable
    part is bevk_dcn_backward_data for fp32/fp16/bf16 with channel counts in
    whole 16-byte vectors (the input is read channels-last, copied once if it
    is not): grad_input summed per destination pixel after a counting sort of
    the samples' corners, grad_offset / grad_mask and col from one pass over
    the samples, all written in the output dtype.  Other cases take the
    bevk_dcn_col2im scatter (fp32 atomics; fp64 for fp64) and the im2col
    kernel.
    """
    ext = _load_ext()
    B, C, H, W = input.shape
    Cout, Cg, kH, kW = weight.shape
    if B == 0:
        # an empty batch: zero gradients of the requested inputs
        acc0 = torch.float64 if input.dtype == torch.float64 else torch.float32
        return (torch.zeros_like(input) if need_input else None,
                torch.zeros_like(offset) if need_offset_mask else None,
                torch.zeros_like(mask) if need_offset_mask else None,
                torch.zeros_like(weight) if need_weight else None,
                torch.zeros(Cout, device=input.device, dtype=acc0).to(input.dtype)
                if need_bias else None)
    T = kH * kW
    sh, sw = _pair(stride)
    ph, pw = _pair(padding)
    dh, dw = _pair(dilation)
    Ho = _out_size(H, ph, dh, kH, sh)
    Wo = _out_size(W, pw, dw, kW, sw)
    M = B * Ho * Wo
    G = groups
    Coutg = Cout // G
    dt = input.dtype
    acc = torch.float64 if dt == torch.float64 else torch.float32
    go = grad_output.to(dt).permute(0, 2, 3, 1).reshape(M, Cout)    # [M, Cout]

    grad_input = grad_offset = grad_mask = grad_weight = grad_bias = None
    col = None
    if need_input or need_offset_mask:
        # dcol[m, t*C + c] = sum_co dO[m, co] * weight[co, c_local, t]  (per conv group)
        wt = _tap_major_weight(weight, dt).view(G, Coutg, T * Cg)          # k = t*Cg + c
        if G == 1:
            dcol = torch.mm(go, wt[0])
        else:
            dcol = torch.stack([torch.mm(go[:, g * Coutg:(g + 1) * Coutg], wt[g])
                                for g in range(G)], 1)                      # [M, G, T*Cg]
            dcol = dcol.view(M, G, T, Cg).permute(0, 2, 1, 3).reshape(M, T * C)
        done = False
        if dt != torch.float64 and (C * input.element_size()) % 16 == 0:
            dev = input.device
            x_cl = None
            if need_offset_mask or need_weight:
                x_cl = input.contiguous(memory_format=torch.channels_last)
            gx = (torch.empty(B, C, H, W, device=dev, dtype=dt).contiguous(
                memory_format=torch.channels_last) if need_input else None)
            goff = torch.empty(offset.shape, device=dev, dtype=dt) if need_offset_mask else None
            gmsk = torch.empty(mask.shape, device=dev, dtype=dt) if need_offset_mask else None
            # with a bias, 8 more columns [1, 0, ..., 0]: the grad_weight GEMM
            # then also returns the column sums of dO (grad_bias)
            K = T * C
            ones_col = need_weight and need_bias and G == 1
            col = (torch.empty(M, K + 8 if ones_col else K, device=dev, dtype=dt)
                   if need_weight else None)
            done = ext.dcn_backward_data(dcol, x_cl, offset, mask, False, C, H, W, kH, kW, sh, sw,
                                         ph, pw, dh, dw, deform_groups, gx, goff, gmsk,
                                         None if col is None else col[:, :K])
            if done:
                grad_input, grad_offset, grad_mask = gx, goff, gmsk
                if ones_col:
                    col[:, K:].copy_(_ones_pad(dt, dev).expand(M, 8))
            else:
                col = None
        if not done:
            fmt = (torch.channels_last if input.is_contiguous(memory_format=torch.channels_last)
                   else torch.contiguous_format)
            gx = (torch.zeros(B, C, H, W, device=input.device, dtype=acc).contiguous(
                memory_format=fmt) if need_input else None)
            goff = (torch.zeros(offset.shape, device=input.device, dtype=acc)
                    if need_offset_mask else None)
            gmsk = (torch.zeros(mask.shape, device=input.device, dtype=acc)
                    if need_offset_mask else None)
            ext.dcn_col2im(dcol, input if need_offset_mask else None, offset, mask, C, H, W, kH,
                           kW, sh, sw, ph, pw, dh, dw, deform_groups, gx, goff, gmsk)
            if need_input:
                grad_input = gx.to(dt)
            if need_offset_mask:
                grad_offset = goff.to(offset.dtype)
                grad_mask = gmsk.to(mask.dtype)
    if need_weight:
        if col is None:
            # NHWC column matrix [M, T*C] (k = t*C + c; aligned leading
            # dimensions for the GEMM) gathered straight from the input in its
            # own layout
            col = ext.dcn_columns(input, offset, mask, kH, kW, sh, sw, ph, pw, dh, dw,
                                  deform_groups, 1)
        if G == 1:
            # col^T . dO ([T*C (+8), Cout]) is the faster cuBLAS form of this
            # product on B200 than dO^T . col (36 vs 42 us at the stage-4 shape)
            gwt = torch.mm(col.t(), go)                                  # [T*C (+8), Cout]
            if gwt.shape[0] > T * C:
                grad_bias = gwt[T * C].contiguous()
                gwt = gwt[:T * C]
            gw = gwt.view(kH, kW, C, Cout).permute(3, 2, 0, 1)
        else:
            colg = col.view(M, T, G, Cg)
            gw = torch.cat([torch.mm(go[:, g * Coutg:(g + 1) * Coutg].t(),
                                     colg[:, :, g].reshape(M, T * Cg)) for g in range(G)], 0)
            gw = gw.view(Cout, kH, kW, Cg).permute(0, 3, 1, 2)
        grad_weight = gw.contiguous().to(weight.dtype)
    if need_bias and grad_bias is None:
        grad_bias = go.sum(0, dtype=acc).to(dt)
    return grad_input, grad_offset, grad_mask, grad_weight, grad_bias


modulated_deform_conv2d = ModulatedDeformConv2dFunction.apply


# The two module classes below keep mmcv's interface so that its checkpoints
# load unchanged: constructor arguments, parameter names and shapes, weight
# initialisation, the conv_offset layer and the version-1 state-dict key
# migration follow mmcv.ops.ModulatedDeformConv2d(Pack) (Copyright (c)
# OpenMMLab, Apache License 2.0; see NOTICE at the repository root).
class ModulatedDeformConv2d(nn.Module):
    """Drop-in for mmcv.ops.ModulatedDeformConv2d (modulated_deform_conv.py:505-543)."""

    def __init__(self, in_channels, out_channels, kernel_size, stride=1, padding=0,
                 dilation=1, groups=1, deform_groups=1, bias=True):
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = _pair(kernel_size)
        self.stride = _pair(stride)
        self.padding = _pair(padding)
        self.dilation = _pair(dilation)
        self.groups = groups
        self.deform_groups = deform_groups
        self.transposed = False
        self.output_padding = _single(0)

        self.weight = nn.Parameter(
            torch.Tensor(out_channels, in_channels // groups, *self.kernel_size))
        if bias:
            self.bias = nn.Parameter(torch.Tensor(out_channels))
        else:
            self.register_parameter('bias', None)
        self.init_weights()

    def init_weights(self):
        n = self.in_channels
        for k in self.kernel_size:
            n *= k
        stdv = 1. / math.sqrt(n)
        self.weight.data.uniform_(-stdv, stdv)
        if self.bias is not None:
            self.bias.data.zero_()

    def forward(self, x, offset, mask):
        return modulated_deform_conv2d(x, offset, mask, self.weight, self.bias, self.stride,
                                       self.padding, self.dilation, self.groups,
                                       self.deform_groups)


class ModulatedDeformConv2dPack(ModulatedDeformConv2d):
    """Self-contained DCNv2 that predicts its own offsets and masks
    (modulated_deform_conv.py:546-643); checkpoint-compatible with mmcv.

    The reference selects among 'fuse_c', 'cuda' and 'tilelang' backends; this
    build has exactly one, so ``backend=`` and ``DCN_BACKEND`` are accepted and
    recorded but do not change the computation.  groups == 1 and
    deform_groups == 1 with the same stride, padding and dilation on both
    axes run the NHWC fused path (offset conv, then the fused kernel reading
    the raw offset-conv output with the mask sigmoid applied on load); other
    geometries compute offsets/masks explicitly and call
    ``modulated_deform_conv2d``, as the reference does (:588-626).  (The
    reference sends asymmetric strides down its NHWC path too, which then
    silently uses the first component for both axes.)
    """

    _version = 2

    def __init__(self, *args, **kwargs):
        self.backend = kwargs.pop('backend', os.environ.get('DCN_BACKEND', 'fuse_c'))
        super().__init__(*args, **kwargs)
        self.conv_offset = nn.Conv2d(
            self.in_channels,
            self.deform_groups * 3 * self.kernel_size[0] * self.kernel_size[1],
            kernel_size=self.kernel_size,
            stride=self.stride,
            padding=self.padding,
            dilation=self.dilation,
            bias=True)
        self.init_weights()

    def init_weights(self):
        super().init_weights()
        if hasattr(self, 'conv_offset'):
            self.conv_offset.weight.data.zero_()
            self.conv_offset.bias.data.zero_()

    def forward(self, x):
        # The NHWC path takes one stride / padding / dilation for both axes
        # (as the reference's, dcn_split_nhwc.py:306-307, which keeps only the
        # first component); asymmetric ones take the general path below, which
        # honours both components.
        square = (self.stride[0] == self.stride[1] and self.padding[0] == self.padding[1]
                  and self.dilation[0] == self.dilation[1])
        if self.groups == 1 and self.deform_groups == 1 and square:
            from .dcn_split_nhwc import dcn_apply_nchw
            return dcn_apply_nchw(x, self.conv_offset.weight, self.conv_offset.bias,
                                  self.weight, self.bias, self.stride, self.padding,
                                  self.dilation)
        out = self.conv_offset(x)
        o1, o2, mask = torch.chunk(out, 3, dim=1)
        offset = torch.cat((o1, o2), dim=1)
        mask = torch.sigmoid(mask)
        return modulated_deform_conv2d(x, offset, mask, self.weight, self.bias, self.stride,
                                       self.padding, self.dilation, self.groups,
                                       self.deform_groups)

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        version = local_metadata.get('version', None)
        if version is None or version < 2:
            # mmcv v1 checkpoints name the offset conv "<prefix>_offset"
            if (prefix + 'conv_offset.weight' not in state_dict
                    and prefix[:-1] + '_offset.weight' in state_dict):
                state_dict[prefix + 'conv_offset.weight'] = state_dict.pop(
                    prefix[:-1] + '_offset.weight')
            if (prefix + 'conv_offset.bias' not in state_dict
                    and prefix[:-1] + '_offset.bias' in state_dict):
                state_dict[prefix + 'conv_offset.bias'] = state_dict.pop(
                    prefix[:-1] + '_offset.bias')
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs)
