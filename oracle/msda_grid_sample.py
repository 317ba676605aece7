"""Independent MSDA forward formulation via ``F.grid_sample`` -- TEST
INFRASTRUCTURE ONLY.

This restates the published multi-scale deformable attention algorithm
(Deformable DETR, Zhu et al. 2021; the "pytorch" reference formulation that
mmcv ships as ``multi_scale_deformable_attn_pytorch``): per level, bilinear
sampling with ``align_corners=False`` and zero padding at grid = 2*loc - 1,
followed by an attention-weighted sum over levels and points.  It is written
from the algorithm, not copied, and serves as a second formulation to
cross-check the direct-gather oracle (``oracle/bevk_oracle.c``), whose
semantics follow ``csrc_musa/msda/ms_deform_attn_kernels.cuh:559-623``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def msda_forward_grid_sample(value: torch.Tensor, spatial_shapes, sampling_loc: torch.Tensor,
                             attn_weight: torch.Tensor) -> torch.Tensor:
    """value [B,S,M,C], spatial_shapes [L,2] (H,W), sampling_loc [B,Q,M,L,P,2],
    attn_weight [B,Q,M,L,P] -> [B,Q,M*C]."""
    B, S, M, C = value.shape
    _, Q, _, L, P, _ = sampling_loc.shape
    shapes = [(int(h), int(w)) for h, w in torch.as_tensor(spatial_shapes).tolist()]
    sizes = [h * w for h, w in shapes]
    levels = value.split(sizes, dim=1)
    grids = 2.0 * sampling_loc - 1.0
    sampled = []
    for lvl, (h, w) in enumerate(shapes):
        # [B, HW, M, C] -> [B*M, C, H, W]
        v = levels[lvl].permute(0, 2, 3, 1).reshape(B * M, C, h, w)
        # [B, Q, M, P, 2] -> [B*M, Q, P, 2]
        g = grids[:, :, :, lvl].permute(0, 2, 1, 3, 4).reshape(B * M, Q, P, 2)
        sampled.append(F.grid_sample(v, g, mode="bilinear", padding_mode="zeros",
                                     align_corners=False))          # [B*M, C, Q, P]
    stacked = torch.stack(sampled, dim=-2).flatten(-2)              # [B*M, C, Q, L*P]
    a = attn_weight.permute(0, 2, 1, 3, 4).reshape(B * M, 1, Q, L * P)
    out = (stacked * a).sum(-1)                                     # [B*M, C, Q]
    return out.view(B, M * C, Q).transpose(1, 2).contiguous()
