"""Multi-scale deformable attention (MSDA) forward and backward for B200.

Operator surface:
* ``MultiScaleDeformableAttnFunction.apply(value, value_spatial_shapes,
  value_level_start_index, sampling_locations, attention_weights, im2col_step)``
  (the mmcv / BEVFormer convention);
* ``ms_deform_attn_forward(value, spatial_shapes, level_start_index,
  sampling_loc, attn_weight, *, im2col_step=64, force_generic=False)`` and
  ``ms_deform_attn_backward(..., grad_output, *, im2col_step=64,
  force_generic_col2im=False)`` (msda_musa_opt2/msda_musa_opt2/dispatch.py
  :15-69 of the reference).

They run ``_ms_deform_attn_ext.forward`` / ``.backward`` ->
``bevk_ms_deform_attn_forward`` / ``_backward``: all four bilinear corners of
a sample in one vector load, fp32 accumulation (fp32 atomics into grad_value
in the backward).  CUDA tensors only.
"""
from __future__ import annotations

import torch
from torch.autograd import Function
from torch.autograd.function import once_differentiable

from bevk import load_extension

_ext = None


def _load_ext():
    global _ext
    if _ext is None:
        _ext = load_extension("_ms_deform_attn_ext")
    return _ext


def ms_deform_attn_forward(value: torch.Tensor, spatial_shapes: torch.Tensor,
                           level_start_index: torch.Tensor, sampling_loc: torch.Tensor,
                           attn_weight: torch.Tensor, *, im2col_step: int = 64,
                           force_generic: bool = False) -> torch.Tensor:
    """value [B,S,heads,C], spatial_shapes [L,2] int64, level_start_index [L]
    int64, sampling_loc [B,Q,heads,L,P,2], attn_weight [B,Q,heads,L,P]
    -> [B, Q, heads*C] in value's dtype."""
    return _load_ext().forward(value, spatial_shapes, level_start_index, sampling_loc,
                               attn_weight, im2col_step=im2col_step,
                               force_generic=force_generic)


def ms_deform_attn_backward(value: torch.Tensor, spatial_shapes: torch.Tensor,
                            level_start_index: torch.Tensor, sampling_loc: torch.Tensor,
                            attn_weight: torch.Tensor, grad_output: torch.Tensor, *,
                            im2col_step: int = 64, force_generic_col2im: bool = False):
    """-> (grad_value, grad_sampling_loc, grad_attn_weight), each in its
    input's shape and dtype (dispatch.py:38-69 of the reference, which zeroes
    all three; here only grad_value, which the kernel accumulates into -- the
    kernel writes every element of the location and attention gradients)."""
    grad_value = torch.zeros_like(value)
    grad_sampling_loc = torch.empty_like(sampling_loc)
    grad_attn_weight = torch.empty_like(attn_weight)
    _load_ext().backward(value, spatial_shapes, level_start_index, sampling_loc, attn_weight,
                         grad_output, grad_value, grad_sampling_loc, grad_attn_weight,
                         im2col_step=im2col_step, force_generic_col2im=force_generic_col2im)
    return grad_value, grad_sampling_loc, grad_attn_weight


class MultiScaleDeformableAttnFunction(Function):
    """autograd Function with the mmcv signature used by BEVFormer's
    TemporalSelfAttention / SpatialCrossAttention."""

    @staticmethod
    def forward(ctx, value, value_spatial_shapes, value_level_start_index, sampling_locations,
                attention_weights, im2col_step):
        ctx.im2col_step = im2col_step
        output = ms_deform_attn_forward(value, value_spatial_shapes, value_level_start_index,
                                        sampling_locations, attention_weights,
                                        im2col_step=im2col_step)
        ctx.save_for_backward(value, value_spatial_shapes, value_level_start_index,
                              sampling_locations, attention_weights)
        return output

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        value, shapes, level_start, loc, attn = ctx.saved_tensors
        grad_value, grad_loc, grad_attn = ms_deform_attn_backward(
            value, shapes, level_start, loc, attn, grad_output.contiguous(),
            im2col_step=ctx.im2col_step)
        return grad_value, None, None, grad_loc, grad_attn, None


multi_scale_deformable_attn = MultiScaleDeformableAttnFunction.apply

__all__ = ["ms_deform_attn_forward", "ms_deform_attn_backward",
           "MultiScaleDeformableAttnFunction", "multi_scale_deformable_attn"]
