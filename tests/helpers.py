"""Shared test helpers: seeded DCN/MSDA problems and C-ABI call wrappers."""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from bevk import cabi

DT = {torch.float32: cabi.DTYPE_F32, torch.float16: cabi.DTYPE_F16,
      torch.bfloat16: cabi.DTYPE_BF16, torch.float64: cabi.DTYPE_F64}

FP32_REL, FP32_ABS = 1e-5, 1e-4      # north_star tolerance, fp32
HALF_REL = 5e-3                      # fp16/bf16 inputs vs fp32 oracle on up-cast inputs


def out_size(n, pad, dil, k, stride):
    return (n + 2 * pad - (dil * (k - 1) + 1)) // stride + 1


def dcn_inputs(seed, B, C, H, W, Cout, k=(3, 3), stride=(1, 1), pad=(1, 1), dil=(1, 1),
               groups=1, dg=1, off_std=2.0, big_frac=0.0, bias=True):
    """Seeded NCHW fp32 CPU tensors with the BASELINE distributions."""
    g = torch.Generator().manual_seed(seed)
    kh, kw = k
    Ho, Wo = out_size(H, pad[0], dil[0], kh, stride[0]), out_size(W, pad[1], dil[1], kw, stride[1])
    T = kh * kw
    x = torch.randn(B, C, H, W, generator=g)
    w = torch.randn(Cout, C // groups, kh, kw, generator=g) * (2.0 / ((C // groups) * T)) ** 0.5
    off = torch.randn(B, 2 * dg * T, Ho, Wo, generator=g) * off_std
    if big_frac:
        sel = torch.rand(off.shape, generator=g) < big_frac
        sign = torch.where(torch.rand(off.shape, generator=g) < 0.5, -1.0, 1.0)
        off = torch.where(sel, sign * (H + 4), off)
    mask = torch.sigmoid(torch.randn(B, dg * T, Ho, Wo, generator=g))
    b = torch.randn(Cout, generator=g) if bias else None
    return x, off, mask, w, b


def problem(x, off, mask, out, Cout, k, stride, pad, dil, groups=1, dg=1, mask_is_logit=False,
            has_bias=False):
    p = cabi.DcnProblem()
    p.dtype = DT[x.dtype]
    p.batch, p.in_channels, p.height, p.width = x.shape
    p.out_channels = Cout
    p.kernel_h, p.kernel_w = k
    p.stride_h, p.stride_w = stride
    p.pad_h, p.pad_w = pad
    p.dilation_h, p.dilation_w = dil
    p.groups, p.deformable_groups = groups, dg
    for i in range(4):
        p.input_strides[i] = x.stride(i)
        p.offset_strides[i] = off.stride(i)
        p.mask_strides[i] = mask.stride(i)
        p.output_strides[i] = out.stride(i)
    p.mask_is_logit = int(mask_is_logit)
    p.has_bias = int(has_bias)
    return p


def cabi_dcn_forward(x, off, mask, w, b, out, stride, pad, dil, groups=1, dg=1,
                     mask_is_logit=False, workspace=True, act_relu=False):
    """Pack + forward through the C ABI (ctypes) on the current stream.
    workspace=False passes no workspace (valid for channel-contiguous input:
    the kernel then takes a schedule without K split)."""
    L = cabi.lib()
    k = (w.shape[2], w.shape[3])
    p = problem(x, off, mask, out, w.shape[0], k, stride, pad, dil, groups, dg, mask_is_logit,
                b is not None)
    p.act_relu = int(act_relu)
    stream = torch.cuda.current_stream().cuda_stream
    nbytes = L.bevk_dcn_packed_weight_bytes(ctypes.byref(p))
    assert nbytes > 0, cabi.last_error()
    wpk = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    wc = w.contiguous()
    cabi.check(L.bevk_dcn_pack_weight(ctypes.byref(p), wc.data_ptr(), wpk.data_ptr(), stream),
               "pack")
    ws_bytes = L.bevk_dcn_forward_workspace_bytes(ctypes.byref(p)) if workspace else 0
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    cabi.check(L.bevk_dcn_forward(ctypes.byref(p), x.data_ptr(), off.data_ptr(), mask.data_ptr(),
                                  wpk.data_ptr(), b.data_ptr() if b is not None else None,
                                  out.data_ptr(), ws.data_ptr() if ws_bytes else None, ws_bytes,
                                  stream), "dcn_forward")
    return out


def cabi_msda_forward(value, shapes, lsi, loc, attn, im2col_step=64):
    L = cabi.lib()
    B, S, M, C = value.shape
    _, Q, _, Lv, P, _ = loc.shape
    out = torch.empty(B, Q, M * C, dtype=value.dtype, device=value.device)
    i64p = ctypes.POINTER(ctypes.c_int64)
    cabi.check(L.bevk_ms_deform_attn_forward(
        value.data_ptr(), ctypes.cast(shapes.data_ptr(), i64p), ctypes.cast(lsi.data_ptr(), i64p),
        loc.data_ptr(), attn.data_ptr(), B, S, M, C, Lv, Q, P, im2col_step, out.data_ptr(),
        DT[value.dtype], torch.cuda.current_stream().cuda_stream), "msda_forward")
    return out


def cabi_msda_backward(value, shapes, lsi, loc, attn, grad_out, grad_value=None,
                       im2col_step=64):
    """Backward through the C ABI -> (grad_value, grad_loc, grad_attn); grad_value
    starts from `grad_value` (f32 accumulates into it) or zeros."""
    L = cabi.lib()
    B, S, M, C = value.shape
    _, Q, _, Lv, P, _ = loc.shape
    gv = torch.zeros_like(value) if grad_value is None else grad_value
    gl = torch.empty_like(loc)
    ga = torch.empty_like(attn)
    ws_bytes = L.bevk_ms_deform_attn_backward_workspace_bytes(B, S, M, C, DT[value.dtype])
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=value.device)
    i64p = ctypes.POINTER(ctypes.c_int64)
    cabi.check(L.bevk_ms_deform_attn_backward(
        value.data_ptr(), ctypes.cast(shapes.data_ptr(), i64p), ctypes.cast(lsi.data_ptr(), i64p),
        loc.data_ptr(), attn.data_ptr(), grad_out.data_ptr(), B, S, M, C, Lv, Q, P, im2col_step,
        gv.data_ptr(), gl.data_ptr(), ga.data_ptr(), ws.data_ptr() if ws_bytes else None,
        ws_bytes, DT[value.dtype], torch.cuda.current_stream().cuda_stream),
        "msda_backward")
    return gv, gl, ga


def msda_inputs(seed, B, shapes, M, C, Q, P, oob_frac=0.02):
    """Seeded MSDA inputs with the BASELINE distributions (CPU fp32)."""
    g = torch.Generator().manual_seed(seed)
    L = len(shapes)
    sizes = [h * w for h, w in shapes]
    S = sum(sizes)
    lsi = torch.tensor(np.concatenate([[0], np.cumsum(sizes)[:-1]]), dtype=torch.int64)
    value = torch.randn(B, S, M, C, generator=g)
    loc = torch.rand(B, Q, M, L, P, 2, generator=g)
    if oob_frac:
        sel = torch.rand(B, Q, M, L, P, 1, generator=g) < oob_frac
        loc = torch.where(sel, loc * 1.4 - 0.2, loc)
    attn = torch.softmax(torch.randn(B, Q, M, L * P, generator=g), -1).view(B, Q, M, L, P)
    return value, torch.tensor(shapes, dtype=torch.int64), lsi, loc, attn


def rel_l2(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def max_abs(a, b):
    return float((a.double().cpu() - b.double().cpu()).abs().max())
