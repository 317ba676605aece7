"""CPU oracle pinned against the reference's own goldens (tests/golden) and
cross-checked against independent formulations.  No GPU needed."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from oracle.msda_grid_sample import msda_forward_grid_sample

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DCN_FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "dcn_*.npz")))
MSDA_FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "msda_*.npz")))


def _meta(z):
    kh, kw, sh, sw, ph, pw, dh, dw, groups, dg = (int(v) for v in z["meta"])
    return (kh, kw), (sh, sw), (ph, pw), (dh, dw), groups, dg


def test_fixture_set_present():
    names = {os.path.basename(p) for p in DCN_FIXTURES + MSDA_FIXTURES}
    assert "dcn_cfg1.npz" in names and len(DCN_FIXTURES) >= 6 and len(MSDA_FIXTURES) >= 2


@pytest.mark.parametrize("path", DCN_FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_dcn_forward_matches_reference_golden(path):
    """oracle vs modulated_deformable_im2col_pytorch + grouped mm (the reference's golden)."""
    z = np.load(path)
    k, st, pd, dl, groups, dg = _meta(z)
    out = oracle.dcn_forward(z["x"], z["offset"], z["mask"], z["weight"], z.get("bias"),
                             st, pd, dl, groups, dg)
    assert oracle.rel_l2(out, z["out"]) <= 1e-6
    assert oracle.max_abs(out, z["out"]) <= 1e-5


@pytest.mark.parametrize("path", [p for p in DCN_FIXTURES if "groups" not in p],
                         ids=lambda p: os.path.basename(p)[:-4])
def test_dcn_nhwc_golden(path):
    """oracle vs the reference's NHWC golden (fused_tl.dcn_forward_golden_nhwc)."""
    z = np.load(path)
    k, st, pd, dl, groups, dg = _meta(z)
    out = oracle.dcn_forward(z["x"], z["offset"], z["mask"], z["weight"], z.get("bias"),
                             st, pd, dl)
    assert oracle.rel_l2(out.transpose(0, 2, 3, 1), z["out_nhwc"]) <= 1e-6


@pytest.mark.parametrize("path", [p for p in DCN_FIXTURES if "columns_nchw" in np.load(p)],
                         ids=lambda p: os.path.basename(p)[:-4])
def test_dcn_columns_match_reference(path):
    z = np.load(path)
    k, st, pd, dl, groups, dg = _meta(z)
    col = oracle.dcn_columns(z["x"], z["offset"], z["mask"], k, st, pd, dl, dg, layout="nchw")
    assert oracle.max_abs(col, z["columns_nchw"]) <= 1e-5
    if "columns_nhwc" in z:
        coln = oracle.dcn_columns(z["x"], z["offset"], z["mask"], k, st, pd, dl, dg,
                                  layout="nhwc")
        assert oracle.max_abs(coln, z["columns_nhwc"]) <= 1e-5


def test_dcn_matches_torchvision():
    """Third formulation: torchvision.ops.deform_conv2d, an independent
    implementation of the same modulated deformable convolution."""
    tv = pytest.importorskip("torchvision")
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 16, 11, 9, generator=g)
    w = torch.randn(12, 16, 3, 3, generator=g)
    off = torch.randn(2, 18, 6, 5, generator=g) * 2
    m = torch.rand(2, 9, 6, 5, generator=g)
    b = torch.randn(12, generator=g)
    want = tv.ops.deform_conv2d(x, off, w, b, stride=2, padding=1, dilation=1, mask=m)
    got = oracle.dcn_forward(x.numpy(), off.numpy(), m.numpy(), w.numpy(), b.numpy(), 2, 1, 1)
    assert oracle.rel_l2(got, want.numpy()) <= 1e-6


def test_dcn_pixel_range_is_a_slice():
    z = np.load(DCN_FIXTURES[0])
    k, st, pd, dl, groups, dg = _meta(z)
    full = oracle.dcn_forward(z["x"], z["offset"], z["mask"], z["weight"], z.get("bias"),
                              st, pd, dl, groups, dg)
    part = oracle.dcn_forward(z["x"], z["offset"], z["mask"], z["weight"], z.get("bias"),
                              st, pd, dl, groups, dg, pix_range=(100, 300))
    B, C, Ho, Wo = full.shape
    flat_full = full.transpose(0, 2, 3, 1).reshape(-1, C)
    flat_part = part.transpose(0, 2, 3, 1).reshape(-1, C)
    assert np.array_equal(flat_part[100:300], flat_full[100:300])
    assert not flat_part[:100].any() and not flat_part[300:].any()


@pytest.mark.parametrize("path", MSDA_FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_msda_matches_fixture(path):
    z = np.load(path)
    out = oracle.msda_forward(z["value"], z["spatial_shapes"], z["level_start_index"],
                              z["sampling_loc"], z["attn_weight"])
    assert oracle.rel_l2(out, z["out"]) <= 1e-6


def test_msda_matches_grid_sample_random():
    g = torch.Generator().manual_seed(11)
    shapes = [(13, 17), (7, 9), (4, 5)]
    sizes = [h * w for h, w in shapes]
    lsi = np.concatenate([[0], np.cumsum(sizes)[:-1]])
    B, M, C, Q, P = 2, 4, 16, 64, 5
    value = torch.randn(B, sum(sizes), M, C, generator=g)
    loc = torch.rand(B, Q, M, 3, P, 2, generator=g) * 1.5 - 0.25      # many points outside
    attn = torch.rand(B, Q, M, 3, P, generator=g)
    want = msda_forward_grid_sample(value, torch.tensor(shapes), loc, attn).numpy()
    got = oracle.msda_forward(value.numpy(), np.array(shapes), lsi, loc.numpy(), attn.numpy())
    assert oracle.rel_l2(got, want) <= 1e-6 and oracle.max_abs(got, want) <= 1e-5


REF_MSDA_CASES = [
    # B, level shapes, heads, C, Q, P, spread of locations beyond [0, 1]
    (2, [(20, 30)], 8, 32, 300, 4, 0.1),
    (3, [(23, 41), (12, 21), (6, 11), (3, 6)], 8, 32, 257, 8, 0.1),
    (1, [(9, 7), (5, 4)], 4, 32, 100, 13, 0.2),
    (2, [(10, 12), (5, 6)], 3, 24, 50, 3, 0.1),
    (1, [(1, 1), (2, 1)], 8, 32, 40, 2, 0.3),       # degenerate levels
    (1, [(29, 50), (15, 25)], 8, 32, 64, 8, 0.0),   # BEVFormer-like level shapes
]


@pytest.mark.parametrize("case", REF_MSDA_CASES, ids=[f"r{i}" for i in range(len(REF_MSDA_CASES))])
def test_msda_matches_reference_kernel(case):
    """The oracle's MSDA forward against the reference's own generic kernel
    (ms_deform_attn_kernels.cuh:559-623) compiled for the host from the
    reference tree (oracle/ref_msda.cpp, oracle/ref_shim)."""
    if not oracle.reference_msda_available():
        pytest.skip("reference tree not present and oracle/_ref not built")
    B, shapes, M, C, Q, P, spread = case
    rng = np.random.default_rng(len(shapes) * 100 + Q)
    L = len(shapes)
    sizes = [h * w for h, w in shapes]
    lsi = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)
    value = rng.standard_normal((B, sum(sizes), M, C)).astype(np.float32)
    loc = rng.uniform(-spread, 1 + spread, (B, Q, M, L, P, 2)).astype(np.float32)
    attn = rng.random((B, Q, M, L, P)).astype(np.float32)
    want = oracle.reference_msda_forward(value, np.array(shapes), lsi, loc, attn)
    got = oracle.msda_forward(value, np.array(shapes), lsi, loc, attn)
    # fp32 rounding only: the two builds contract multiply-adds differently
    assert oracle.rel_l2(got, want) <= 1e-6 and oracle.max_abs(got, want) <= 1e-5


REF_MSDA_BWD_CASES = [
    # B, level shapes, heads, C, Q, P, spread of locations beyond [0, 1]
    (2, [(20, 30)], 8, 32, 24, 4, 0.1),
    (1, [(23, 41), (12, 21), (6, 11), (3, 6)], 8, 32, 12, 8, 0.1),
    (1, [(9, 7), (5, 4)], 4, 32, 16, 13, 0.2),
    (2, [(10, 12), (5, 6)], 3, 24, 10, 3, 0.1),      # C = 24: a block of 24 threads
    (1, [(1, 1), (2, 1)], 8, 32, 8, 2, 0.3),         # degenerate levels
]


@pytest.mark.parametrize("case", REF_MSDA_BWD_CASES,
                         ids=[f"b{i}" for i in range(len(REF_MSDA_BWD_CASES))])
def test_msda_backward_matches_reference_kernel(case):
    """The oracle's MSDA backward against the reference's own generic backward
    kernel (ms_deform_attn_kernels.cuh:1168-1271: a block of C threads per
    (batch, query, head), shared-memory reduction of the location / attention
    gradients, atomics into grad_value) compiled for the host from the
    reference tree and run as one emulated block of C host threads."""
    if not oracle.reference_msda_available():
        pytest.skip("reference tree not present and oracle/_ref not built")
    B, shapes, M, C, Q, P, spread = case
    rng = np.random.default_rng(len(shapes) * 1000 + Q + C)
    L = len(shapes)
    sizes = [h * w for h, w in shapes]
    lsi = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)
    value = rng.standard_normal((B, sum(sizes), M, C)).astype(np.float32)
    loc = rng.uniform(-spread, 1 + spread, (B, Q, M, L, P, 2)).astype(np.float32)
    attn = rng.random((B, Q, M, L, P)).astype(np.float32)
    gout = rng.standard_normal((B, Q, M * C)).astype(np.float32)
    want = oracle.reference_msda_backward(value, np.array(shapes), lsi, loc, attn, gout)
    got = oracle.msda_backward(value, np.array(shapes), lsi, loc, attn, gout)
    # fp32 rounding only (summation orders and atomics differ)
    for name, g, w in zip(("grad_value", "grad_loc", "grad_attn"), got, want):
        scale = max(1.0, float(np.abs(w).max()))
        assert oracle.rel_l2(g, w) <= 1e-5, (name, oracle.rel_l2(g, w))
        assert oracle.max_abs(g, w) <= 1e-4 * scale, (name, oracle.max_abs(g, w))


def test_msda_boundary_coordinates():
    """Points exactly on the gates: h = -1 and h = H (dropped), h = H-1 (kept)."""
    H, W = 4, 5
    value = np.arange(H * W * 1 * 1, dtype=np.float32).reshape(1, H * W, 1, 1) + 1
    # loc_y*H - 0.5 = -1  -> loc_y = -0.5/H ; = H -> (H+0.5)/H ; = H-1 -> (H-0.5)/H
    ys = np.array([-0.5 / H, (H + 0.5) / H, (H - 0.5) / H], np.float32)
    loc = np.zeros((1, 3, 1, 1, 1, 2), np.float32)
    loc[0, :, 0, 0, 0, 0] = 0.5            # x in range
    loc[0, :, 0, 0, 0, 1] = ys
    attn = np.ones((1, 3, 1, 1, 1), np.float32)
    out = oracle.msda_forward(value, [[H, W]], [0], loc, attn)
    assert out[0, 0, 0] == 0 and out[0, 1, 0] == 0 and out[0, 2, 0] != 0


def test_msda_backward_matches_autograd():
    """Oracle backward (the reference's col2im formulas) against torch autograd
    of the independent grid_sample formulation, in float64."""
    g = torch.Generator().manual_seed(12)
    shapes = [(11, 13), (6, 7), (3, 4)]
    sizes = [h * w for h, w in shapes]
    lsi = np.concatenate([[0], np.cumsum(sizes)[:-1]])
    B, M, C, Q, L, P = 2, 3, 8, 40, 3, 4
    value = torch.randn(B, sum(sizes), M, C, generator=g)
    loc = torch.rand(B, Q, M, L, P, 2, generator=g) * 1.4 - 0.2      # some points outside
    attn = torch.rand(B, Q, M, L, P, generator=g)
    gout = torch.randn(B, Q, M * C, generator=g)
    v64, l64, a64 = (t.double().requires_grad_() for t in (value, loc, attn))
    out = msda_forward_grid_sample(v64, torch.tensor(shapes), l64, a64)
    (out * gout.double()).sum().backward()
    gv, gl, ga = oracle.msda_backward(value.numpy(), np.array(shapes), lsi, loc.numpy(),
                                      attn.numpy(), gout.numpy())
    for got, want in ((gv, v64.grad), (gl, l64.grad), (ga, a64.grad)):
        want = want.numpy()
        assert oracle.rel_l2(got, want) <= 1e-5, oracle.rel_l2(got, want)


def test_msda_backward_zero_outside_gate():
    """A sample outside the gate gets zero grad_loc / grad_attn and touches no
    grad_value line (binding_musa.mu:414-543 writes zeros for it)."""
    H, W = 4, 5
    value = np.random.default_rng(0).standard_normal((1, H * W, 1, 2)).astype(np.float32)
    loc = np.full((1, 1, 1, 1, 1, 2), 0.5, np.float32)
    loc[..., 1] = -0.5 / H - 1e-3                       # h just below -1
    attn = np.ones((1, 1, 1, 1, 1), np.float32)
    gout = np.ones((1, 1, 2), np.float32)
    gv, gl, ga = oracle.msda_backward(value, [[H, W]], [0], loc, attn, gout)
    assert not gv.any() and not gl.any() and not ga.any()


@pytest.mark.parametrize("path", DCN_FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_dcn_backward_matches_reference_golden(path):
    """Oracle backward against the reference's col2im / col2im_coord goldens
    (autograd through its differentiable im2col) and autograd grad_weight."""
    z = np.load(path)
    k, st, pd, dl, groups, dg = _meta(z)
    with_bias = "grad_bias" in z.files
    gx, goff, gm, gw, gb = oracle.dcn_backward(z["x"], z["offset"], z["mask"], z["weight"],
                                               z["grad_out"], st, pd, dl, groups, dg,
                                               with_bias=with_bias)
    for name, got in (("grad_x", gx), ("grad_offset", goff), ("grad_mask", gm),
                      ("grad_weight", gw)) + ((("grad_bias", gb),) if with_bias else ()):
        want = z[name]
        assert oracle.rel_l2(got, want) <= 1e-5, (name, oracle.rel_l2(got, want))


def test_dcn_backward_matches_torchvision_autograd():
    """Third formulation: autograd of torchvision.ops.deform_conv2d."""
    tv = pytest.importorskip("torchvision")
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 8, 9, 10, generator=g, dtype=torch.float64)
    w = torch.randn(12, 8, 3, 3, generator=g, dtype=torch.float64) * 0.2
    off = torch.randn(2, 18, 9, 10, generator=g, dtype=torch.float64) * 1.5
    mask = torch.sigmoid(torch.randn(2, 9, 9, 10, generator=g, dtype=torch.float64))
    b = torch.randn(12, generator=g, dtype=torch.float64)
    gout = torch.randn(2, 12, 9, 10, generator=g, dtype=torch.float64)
    xs, ws, os_, ms, bs = (t.clone().requires_grad_() for t in (x, w, off, mask, b))
    out = tv.ops.deform_conv2d(xs, os_, ws, bs, stride=1, padding=1, dilation=1, mask=ms)
    out.backward(gout)
    got = oracle.dcn_backward(x.float().numpy(), off.float().numpy(), mask.float().numpy(),
                              w.float().numpy(), gout.float().numpy(), 1, 1, 1)
    for a, t in zip(got, (xs, os_, ms, ws, bs)):
        assert oracle.rel_l2(a, t.grad.numpy()) <= 2e-5, oracle.rel_l2(a, t.grad.numpy())
