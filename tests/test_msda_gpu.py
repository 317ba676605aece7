"""MSDA forward and backward parity on the GPU (C ABI and Python surface) vs the CPU oracle.

Tolerances: fp32 within 1e-5 relative L2 and 1e-4 max-abs; fp16/bf16 within
5e-3 relative L2 of the fp32 oracle on the up-cast inputs.
"""
import glob
import os

import numpy as np
import pytest
import torch

from helpers import (FP32_ABS, FP32_REL, HALF_REL, cabi_msda_backward, cabi_msda_forward,
                     max_abs, msda_inputs,
                     rel_l2)
from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

CFG4 = dict(B=2, shapes=[(200, 200)], M=8, C=32, Q=40000, P=4)
CFG5 = dict(B=6, shapes=[(116, 200), (58, 100), (29, 50), (15, 25)], M=8, C=32, Q=10000, P=8)


def _oracle(value, shapes, lsi, loc, attn):
    return torch.from_numpy(oracle.msda_forward(value.float().cpu().numpy(), shapes.cpu().numpy(),
                                                lsi.cpu().numpy(), loc.float().cpu().numpy(),
                                                attn.float().cpu().numpy()))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "msda_*.npz"))),
                         ids=lambda p: os.path.basename(p)[:-4])
def test_fixtures_cabi(cuda, path):
    z = np.load(path)
    value, shapes, lsi, loc, attn = (torch.from_numpy(z[n]).to(cuda) for n in (
        "value", "spatial_shapes", "level_start_index", "sampling_loc", "attn_weight"))
    out = cabi_msda_forward(value, shapes, lsi, loc, attn)
    ref = torch.from_numpy(z["out"])
    assert rel_l2(out, ref) <= FP32_REL and max_abs(out, ref) <= FP32_ABS


SMALL = [
    dict(B=2, shapes=[(20, 30)], M=8, C=32, Q=300, P=4),
    dict(B=3, shapes=[(23, 41), (12, 21), (6, 11), (3, 6)], M=8, C=32, Q=257, P=8),
    dict(B=1, shapes=[(9, 7), (5, 4)], M=4, C=32, Q=100, P=13),      # L*P > 32 samples
    dict(B=2, shapes=[(10, 12), (5, 6)], M=3, C=24, Q=50, P=3),      # generic kernel (C != 32)
    dict(B=1, shapes=[(1, 1), (2, 1)], M=8, C=32, Q=40, P=2),        # degenerate levels
    dict(B=2, shapes=[(15, 17), (8, 9)], M=8, C=32, Q=123, P=4),     # L*P = 8 pass kernel
    dict(B=1, shapes=[(13, 11), (7, 6), (4, 3), (2, 2)], M=8, C=32, Q=77, P=4),  # L*P = 16
    dict(B=1, shapes=[(12, 10), (6, 5)], M=5, C=32, Q=33, P=2),      # units % 8 != 0
]


@pytest.mark.parametrize("cfg", SMALL, ids=[f"s{i}" for i in range(len(SMALL))])
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16],
                         ids=["f32", "f16", "bf16"])
def test_small_cases(cuda, cfg, dt):
    value, shapes, lsi, loc, attn = msda_inputs(7, oob_frac=0.1, **cfg)
    value, loc, attn = (t.to(cuda, dt) for t in (value, loc, attn))
    shapes, lsi = shapes.to(cuda), lsi.to(cuda)
    want = _oracle(value, shapes, lsi, loc, attn)
    out = cabi_msda_forward(value, shapes, lsi, loc, attn)
    if dt == torch.float32:
        assert rel_l2(out, want) <= FP32_REL and max_abs(out, want) <= FP32_ABS
    else:
        assert out.dtype == dt and rel_l2(out, want) <= HALF_REL


# Larger multi-level cases (150k+ units: batch x queries x heads) with partial
# load batches (L*P = 9), two rounds of samples (L*P = 48) and large levels.
LARGE = [
    dict(B=2, shapes=[(40, 60), (20, 30), (10, 15), (5, 8)], M=8, C=32, Q=10000, P=8),
    dict(B=1, shapes=[(30, 50), (15, 25), (8, 13)], M=8, C=32, Q=19000, P=3),
    dict(B=3, shapes=[(16, 20), (8, 10), (4, 5), (2, 3)], M=4, C=32, Q=13000, P=12),
    dict(B=1, shapes=[(120, 160), (60, 80)], M=8, C=32, Q=19500, P=4),
]


@pytest.mark.parametrize("cfg", LARGE, ids=[f"l{i}" for i in range(len(LARGE))])
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16],
                         ids=["f32", "f16", "bf16"])
def test_large_multilevel_cases(cuda, cfg, dt):
    value, shapes, lsi, loc, attn = msda_inputs(11, oob_frac=0.05, **cfg)
    value, loc, attn = (t.to(cuda, dt) for t in (value, loc, attn))
    shapes, lsi = shapes.to(cuda), lsi.to(cuda)
    want = _oracle(value, shapes, lsi, loc, attn)
    out = cabi_msda_forward(value, shapes, lsi, loc, attn)
    if dt == torch.float32:
        assert rel_l2(out, want) <= FP32_REL and max_abs(out, want) <= FP32_ABS
    else:
        assert out.dtype == dt and rel_l2(out, want) <= HALF_REL


# Multi-level problems outside the pass kernel's L*P (4, 8, 16) on the
# warp-per-unit kernel: a head count that does not divide the SM count, a
# small level beside a large one, degenerate levels with two rounds of samples
# (L*P = 36), and more heads than SMs.  Each case runs twice in a row.
MULTI = [
    dict(B=3, shapes=[(36, 64), (18, 32), (9, 16), (5, 8)], M=6, C=32, Q=1200, P=8),
    dict(B=2, shapes=[(50, 70), (25, 35)], M=8, C=32, Q=800, P=5),
    dict(B=1, shapes=[(1, 1), (2, 1), (1, 3), (40, 50)], M=8, C=32, Q=600, P=9),
    dict(B=1, shapes=[(6, 5), (3, 2)], M=160, C=32, Q=20, P=3),
]


@pytest.mark.parametrize("cfg", MULTI, ids=[f"t{i}" for i in range(len(MULTI))])
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16],
                         ids=["f32", "f16", "bf16"])
def test_multilevel_warp_per_unit_cases(cuda, cfg, dt):
    value, shapes, lsi, loc, attn = msda_inputs(13, oob_frac=0.1, **cfg)
    value, loc, attn = (t.to(cuda, dt) for t in (value, loc, attn))
    shapes, lsi = shapes.to(cuda), lsi.to(cuda)
    want = _oracle(value, shapes, lsi, loc, attn)
    for _ in range(2):
        out = cabi_msda_forward(value, shapes, lsi, loc, attn)
        if dt == torch.float32:
            assert rel_l2(out, want) <= FP32_REL and max_abs(out, want) <= FP32_ABS
        else:
            assert out.dtype == dt and rel_l2(out, want) <= HALF_REL


@pytest.mark.parametrize("name", ["cfg4", "cfg5"])
def test_baseline_configs_full_size(cuda, name):
    import ms_deform_attn
    cfg = CFG4 if name == "cfg4" else CFG5
    value, shapes, lsi, loc, attn = msda_inputs(2026, oob_frac=0.02 if name == "cfg4" else 0.0,
                                                **cfg)
    want = _oracle(value, shapes, lsi, loc, attn)
    value, shapes, lsi, loc, attn = (t.to(cuda) for t in (value, shapes, lsi, loc, attn))
    out = ms_deform_attn.MultiScaleDeformableAttnFunction.apply(value, shapes, lsi, loc, attn, 64)
    assert out.shape == (cfg["B"], cfg["Q"], cfg["M"] * cfg["C"])
    assert rel_l2(out, want) <= FP32_REL and max_abs(out, want) <= FP32_ABS


def test_im2col_step_contract(cuda):
    import ms_deform_attn
    value, shapes, lsi, loc, attn = (t.to(cuda) for t in msda_inputs(1, 3, [(6, 6)], 8, 32, 10, 4))
    with pytest.raises(RuntimeError, match="im2col_step"):
        ms_deform_attn.ms_deform_attn_forward(value, shapes, lsi, loc, attn, im2col_step=2)
    out = ms_deform_attn.ms_deform_attn_forward(value, shapes, lsi, loc, attn, im2col_step=3)
    want = _oracle(value, shapes, lsi, loc, attn)
    assert rel_l2(out, want) <= FP32_REL
    with pytest.raises(RuntimeError, match="contiguous"):
        ms_deform_attn.ms_deform_attn_forward(value.transpose(1, 2), shapes, lsi, loc, attn)


# ------------------------------------------------------------------ backward
def _oracle_bwd(value, shapes, lsi, loc, attn, gout):
    return tuple(torch.from_numpy(a) for a in oracle.msda_backward(
        value.float().cpu().numpy(), shapes.cpu().numpy(), lsi.cpu().numpy(),
        loc.float().cpu().numpy(), attn.float().cpu().numpy(), gout.float().cpu().numpy()))


def _bwd_case(cuda, cfg, dt, seed=7, oob=0.1):
    value, shapes, lsi, loc, attn = msda_inputs(seed, oob_frac=oob, **cfg)
    g = torch.Generator().manual_seed(seed + 1)
    gout = torch.randn(cfg["B"], cfg["Q"], cfg["M"] * cfg["C"], generator=g)
    value, loc, attn, gout = (t.to(cuda, dt) for t in (value, loc, attn, gout))
    return value, shapes.to(cuda), lsi.to(cuda), loc, attn, gout


def _check_grads(got, want, dt):
    for name, a, b in zip(("grad_value", "grad_loc", "grad_attn"), got, want):
        if dt == torch.float32:
            assert rel_l2(a, b) <= FP32_REL, (name, rel_l2(a, b))
            scale = float(b.abs().max()) or 1.0
            assert max_abs(a, b) <= FP32_ABS * max(1.0, scale), (name, max_abs(a, b))
        else:
            assert a.dtype == dt and rel_l2(a, b) <= HALF_REL, (name, rel_l2(a, b))


@pytest.mark.parametrize("cfg", SMALL, ids=[f"s{i}" for i in range(len(SMALL))])
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16],
                         ids=["f32", "f16", "bf16"])
def test_backward_small_cases(cuda, cfg, dt):
    value, shapes, lsi, loc, attn, gout = _bwd_case(cuda, cfg, dt)
    want = _oracle_bwd(value, shapes, lsi, loc, attn, gout)
    _check_grads(cabi_msda_backward(value, shapes, lsi, loc, attn, gout), want, dt)


# The multi-level cases through the backward: L*P = 32 (batches of 8 sharing
# one grad_out vector), 10 and 6 (batches of 4 that cross unit boundaries,
# one grad_out vector per sample) and 36 (batches of 4 inside a unit), with
# passes of 32 samples that start mid-unit.
@pytest.mark.parametrize("cfg", MULTI, ids=[f"t{i}" for i in range(len(MULTI))])
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16],
                         ids=["f32", "f16", "bf16"])
def test_backward_multilevel_cases(cuda, cfg, dt):
    value, shapes, lsi, loc, attn, gout = _bwd_case(cuda, cfg, dt, seed=17)
    want = _oracle_bwd(value, shapes, lsi, loc, attn, gout)
    _check_grads(cabi_msda_backward(value, shapes, lsi, loc, attn, gout), want, dt)


@pytest.mark.parametrize("name", ["cfg4", "cfg5"])
def test_backward_baseline_configs_full_size(cuda, name):
    import ms_deform_attn
    cfg = CFG4 if name == "cfg4" else CFG5
    value, shapes, lsi, loc, attn, gout = _bwd_case(cuda, cfg, torch.float32, seed=2026,
                                                    oob=0.02 if name == "cfg4" else 0.0)
    want = _oracle_bwd(value, shapes, lsi, loc, attn, gout)
    got = ms_deform_attn.ms_deform_attn_backward(value, shapes, lsi, loc, attn, gout)
    _check_grads(got, want, torch.float32)


def test_backward_through_autograd(cuda):
    """MultiScaleDeformableAttnFunction.backward returns the op's gradients for
    value, sampling_locations and attention_weights (and None for the rest)."""
    import ms_deform_attn
    cfg = SMALL[1]
    value, shapes, lsi, loc, attn, gout = _bwd_case(cuda, cfg, torch.float32)
    v, l, a = (t.clone().requires_grad_() for t in (value, loc, attn))
    out = ms_deform_attn.MultiScaleDeformableAttnFunction.apply(v, shapes, lsi, l, a, 64)
    out.backward(gout)
    want = _oracle_bwd(value, shapes, lsi, loc, attn, gout)
    _check_grads((v.grad, l.grad, a.grad), want, torch.float32)


def test_backward_f32_accumulates_into_grad_value(cuda):
    """fp32 grad_value is accumulated into (the reference's callers pass zeros)."""
    cfg = SMALL[0]
    value, shapes, lsi, loc, attn, gout = _bwd_case(cuda, cfg, torch.float32)
    base = torch.randn_like(value)
    gv, _, _ = cabi_msda_backward(value, shapes, lsi, loc, attn, gout, grad_value=base.clone())
    want = _oracle_bwd(value, shapes, lsi, loc, attn, gout)[0]
    assert rel_l2(gv - base, want) <= FP32_REL


def test_backward_im2col_step_contract(cuda):
    import ms_deform_attn
    cfg = dict(SMALL[0], B=3)
    value, shapes, lsi, loc, attn, gout = _bwd_case(cuda, cfg, torch.float32)
    with pytest.raises(RuntimeError, match="im2col_step"):
        ms_deform_attn.ms_deform_attn_backward(value, shapes, lsi, loc, attn, gout, im2col_step=2)


@pytest.mark.parametrize("dt", [torch.float32, torch.float16], ids=["f32", "f16"])
def test_zero_queries(cuda, dt):
    """num_query = 0: an empty output, zero grad_value and empty location /
    attention gradients."""
    import ms_deform_attn
    value, shapes, lsi, loc, attn = msda_inputs(3, 2, [(6, 7), (3, 4)], 8, 32, 0, 4)
    value, loc, attn = (t.to(cuda, dt) for t in (value, loc, attn))
    shapes, lsi = shapes.to(cuda), lsi.to(cuda)
    out = ms_deform_attn.ms_deform_attn_forward(value, shapes, lsi, loc, attn)
    assert out.shape == (2, 0, 256) and out.dtype == dt
    gout = torch.zeros(2, 0, 256, device=cuda, dtype=dt)
    gv, gl, ga = ms_deform_attn.ms_deform_attn_backward(value, shapes, lsi, loc, attn, gout)
    torch.cuda.synchronize()
    assert gv.shape == value.shape and not torch.count_nonzero(gv)
    assert gl.shape == loc.shape and ga.shape == attn.shape
