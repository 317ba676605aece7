"""Multi-scale deformable attention (MSDA) forward for B200.

Operator surface:
* ``MultiScaleDeformableAttnFunction.apply(value, value_spatial_shapes,
  value_level_start_index, sampling_locations, attention_weights, im2col_step)``
  (the mmcv / BEVFormer convention);
* ``ms_deform_attn_forward(value, spatial_shapes, level_start_index,
  sampling_loc, attn_weight, *, im2col_step=64, force_generic=False)``
  (msda_musa_opt2/msda_musa_opt2/dispatch.py:15-35 of the reference).

Both run ``_ms_deform_attn_ext.forward`` -> ``bevk_ms_deform_attn_forward``:
one warp per (batch, query, head), all four bilinear corners of a sample in
one vector load, fp32 accumulation.  CUDA tensors only.
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
        raise NotImplementedError(
            "bev-kernels_b200: MultiScaleDeformableAttnFunction backward is not built yet "
            "(forward-only release)")


multi_scale_deformable_attn = MultiScaleDeformableAttnFunction.apply

__all__ = ["ms_deform_attn_forward", "MultiScaleDeformableAttnFunction",
           "multi_scale_deformable_attn"]
