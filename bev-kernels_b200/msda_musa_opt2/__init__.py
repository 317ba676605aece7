"""Import-path alias of the reference's MSDA dispatch package
(msda_musa_opt2/msda_musa_opt2/__init__.py) so existing imports keep working;
the implementation is :mod:`ms_deform_attn` (CUDA, sm_100a)."""
from .dispatch import ms_deform_attn_backward, ms_deform_attn_forward  # noqa: F401

__all__ = ["ms_deform_attn_forward", "ms_deform_attn_backward"]
