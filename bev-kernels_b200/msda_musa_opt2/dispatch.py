"""Alias of msda_musa_opt2/msda_musa_opt2/dispatch.py:15-69 over :mod:`ms_deform_attn`."""
from ms_deform_attn import ms_deform_attn_backward, ms_deform_attn_forward  # noqa: F401
