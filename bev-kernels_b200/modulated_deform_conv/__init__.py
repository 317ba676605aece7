"""DCNv2 (modulated deformable convolution) for B200 -- drop-in for the
reference's ``modulated_deform_conv`` package (its ``__init__.py`` exports)."""
from .modulated_deform_conv import (  # noqa: F401
    ModulatedDeformConv2d,
    ModulatedDeformConv2dFunction,
    ModulatedDeformConv2dPack,
    dcn_backward,
    dcn_forward_into,
    ext_modulated_deformable_col2im,
    ext_modulated_deformable_col2im_coord,
    ext_modulated_deformable_col2im_coord_opt,
    ext_modulated_deformable_col2im_opt,
    ext_modulated_deformable_col2im_smem,
    ext_modulated_deformable_im2col,
    ext_modulated_deformable_im2col_opt,
    modulated_deform_conv2d,
    offset_conv,
    offset_conv_partials,
    packed_weight,
)
from .dcn_split_nhwc import (  # noqa: F401
    DCNSplitNHWCFunction,
    dcn_apply_nchw,
    dcn_split_forward_nhwc,
    dcn_split_nhwc,
    gather_cols_nhwc,
)

__all__ = [
    "ModulatedDeformConv2dFunction",
    "ModulatedDeformConv2d",
    "ModulatedDeformConv2dPack",
    "modulated_deform_conv2d",
    "ext_modulated_deformable_im2col",
    "ext_modulated_deformable_im2col_opt",
    "ext_modulated_deformable_col2im",
    "ext_modulated_deformable_col2im_opt",
    "ext_modulated_deformable_col2im_smem",
    "ext_modulated_deformable_col2im_coord",
    "ext_modulated_deformable_col2im_coord_opt",
    "dcn_backward",
    "DCNSplitNHWCFunction",
    "dcn_apply_nchw",
    "dcn_split_nhwc",
    "dcn_split_forward_nhwc",
    "gather_cols_nhwc",
]
