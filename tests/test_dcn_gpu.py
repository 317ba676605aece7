"""DCNv2 forward parity on the GPU: CUDA path (through the C ABI and through the
reference-compatible Python surface) vs the CPU oracle and the reference's own
golden outputs.

Tolerances (north_star): fp32 within 1e-5 relative L2 and 1e-4 max-abs;
fp16/bf16 inputs (fp32 accumulation) within 5e-3 relative L2 of the fp32 oracle
run on the up-cast inputs.
"""
import glob
import os

import numpy as np
import pytest
import torch

from helpers import (FP32_ABS, FP32_REL, HALF_REL, cabi_dcn_forward, dcn_inputs, max_abs,
                     out_size, rel_l2)
from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _golden_cases():
    return sorted(glob.glob(os.path.join(GOLDEN, "dcn_*.npz")))


def _meta(z):
    kh, kw, sh, sw, ph, pw, dh, dw, groups, dg = (int(v) for v in z["meta"])
    return (kh, kw), (sh, sw), (ph, pw), (dh, dw), groups, dg


def _oracle(x, off, mask, w, b, stride, pad, dil, groups=1, dg=1):
    return torch.from_numpy(oracle.dcn_forward(
        x.float().cpu().numpy(), off.float().cpu().numpy(), mask.float().cpu().numpy(),
        w.float().cpu().numpy(), None if b is None else b.float().cpu().numpy(),
        stride, pad, dil, groups, dg))


def _watchdog_clean():
    from bevk import cabi
    import ctypes
    code = ctypes.c_uint(0)
    st = cabi.lib().bevk_device_watchdog(0, ctypes.byref(code))
    assert st == 0 and code.value == 0, f"device watchdog fired: 0x{code.value:x}"


@pytest.mark.parametrize("path", _golden_cases(), ids=lambda p: os.path.basename(p)[:-4])
def test_golden_fp32_cabi(cuda, path):
    """fp32 exact path vs the reference's own golden (NCHW im2col + mm)."""
    z = np.load(path)
    k, st, pd, dl, groups, dg = _meta(z)
    x, off, mask, w = (torch.from_numpy(z[n]).to(cuda) for n in ("x", "offset", "mask", "weight"))
    b = torch.from_numpy(z["bias"]).to(cuda) if "bias" in z else None
    ref = torch.from_numpy(z["out"])
    out = torch.empty_like(ref, device=cuda)
    cabi_dcn_forward(x, off, mask, w, b, out, st, pd, dl, groups, dg)
    torch.cuda.synchronize()
    assert rel_l2(out, ref) <= FP32_REL and max_abs(out, ref) <= FP32_ABS
    _watchdog_clean()


@pytest.mark.parametrize("path", _golden_cases(), ids=lambda p: os.path.basename(p)[:-4])
def test_golden_function_surface(cuda, path):
    """ModulatedDeformConv2dFunction.apply (reference argument order) vs golden."""
    from modulated_deform_conv import modulated_deform_conv2d
    z = np.load(path)
    k, st, pd, dl, groups, dg = _meta(z)
    x, off, mask, w = (torch.from_numpy(z[n]).to(cuda) for n in ("x", "offset", "mask", "weight"))
    b = torch.from_numpy(z["bias"]).to(cuda) if "bias" in z else None
    out = modulated_deform_conv2d(x, off, mask, w, b, st, pd, dl, groups, dg)
    assert out.is_contiguous() and out.dtype == torch.float32
    ref = torch.from_numpy(z["out"])
    assert rel_l2(out, ref) <= FP32_REL and max_abs(out, ref) <= FP32_ABS


@pytest.mark.parametrize("path", [p for p in _golden_cases() if "groups" not in p],
                         ids=lambda p: os.path.basename(p)[:-4])
def test_golden_nhwc_half(cuda, path):
    """Tensor-core path (fp16/bf16, NHWC input and output) vs the reference's NHWC golden."""
    from modulated_deform_conv import dcn_forward_into
    z = np.load(path)
    k, st, pd, dl, groups, dg = _meta(z)
    ref = torch.from_numpy(z["out_nhwc"])
    for dt in (torch.float16, torch.bfloat16):
        x = torch.from_numpy(z["x"]).to(cuda, dt)
        off = torch.from_numpy(z["offset"]).to(cuda, dt)
        mask = torch.from_numpy(z["mask"]).to(cuda, dt)
        w = torch.from_numpy(z["weight"]).to(cuda, dt)
        b = torch.from_numpy(z["bias"]).to(cuda, dt) if "bias" in z else None
        # reference of record on the exact (rounded) inputs
        want = _oracle(x, off, mask, w, b, st, pd, dl).permute(0, 2, 3, 1)
        x_cl = x.contiguous(memory_format=torch.channels_last)
        out = torch.empty(ref.shape, dtype=dt, device=cuda)       # [B, Ho, Wo, Cout]
        dcn_forward_into(x_cl, off, mask, w, b, out.permute(0, 3, 1, 2), st, pd, dl)
        assert rel_l2(out, want) <= HALF_REL, (dt, rel_l2(out, want))
        assert rel_l2(out, ref) <= 3e-2     # sanity vs the fp32 golden of the unrounded data


TC_CASES = [
    # B, C, H, W, Cout, k, stride, pad, dil, off_std, big_frac
    (1, 64, 9, 17, 64, (3, 3), (1, 1), (1, 1), (1, 1), 2.0, 0.0),
    (2, 8, 7, 5, 16, (3, 3), (1, 1), (1, 1), (1, 1), 2.0, 0.0),
    (1, 72, 11, 13, 96, (3, 3), (1, 1), (1, 1), (1, 1), 2.0, 0.05),
    (2, 128, 10, 19, 320, (3, 3), (2, 2), (1, 1), (1, 1), 1.0, 0.0),
    (1, 24, 15, 9, 40, (3, 3), (1, 2), (2, 1), (2, 1), 3.0, 0.0),
    (3, 256, 8, 12, 256, (3, 3), (1, 1), (1, 1), (1, 1), 2.0, 0.05),
    (1, 40, 9, 9, 130, (1, 3), (1, 1), (0, 1), (1, 1), 1.0, 0.0),
]


@pytest.mark.parametrize("case", TC_CASES, ids=[f"tc{i}" for i in range(len(TC_CASES))])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("layout", ["nchw_in", "nhwc_in"])
def test_tensor_core_path(cuda, case, dt, layout):
    B, C, H, W, Cout, k, stride, pad, dil, off_std, big = case
    x, off, mask, w, b = dcn_inputs(11, B, C, H, W, Cout, k, stride, pad, dil, off_std=off_std,
                                    big_frac=big)
    x, off, mask, w, b = (t.to(cuda, dt) for t in (x, off, mask, w, b))
    want = _oracle(x, off, mask, w, b, stride, pad, dil)
    if layout == "nhwc_in":
        x = x.contiguous(memory_format=torch.channels_last)
        out = torch.empty(want.shape, dtype=dt, device=cuda,
                          memory_format=torch.channels_last)
    else:
        out = torch.empty(want.shape, dtype=dt, device=cuda)
    cabi_dcn_forward(x, off, mask, w, b, out, stride, pad, dil)
    torch.cuda.synchronize()
    assert rel_l2(out, want) <= HALF_REL, rel_l2(out, want)
    _watchdog_clean()


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_fused_logit_mask(cuda, dt):
    """Raw offset-conv output y (offsets + pre-sigmoid mask, NHWC) read directly."""
    from modulated_deform_conv import dcn_forward_into
    B, C, H, W, Cout = 2, 64, 12, 14, 128
    x, off, mask, w, b = dcn_inputs(5, B, C, H, W, Cout)
    logits = torch.logit(mask)
    y = torch.cat([off, logits], 1).to(cuda, dt).contiguous(memory_format=torch.channels_last)
    xd, wd, bd = x.to(cuda, dt), w.to(cuda, dt), b.to(cuda, dt)
    want = _oracle(xd, y[:, :18], torch.sigmoid(y[:, 18:].float()), wd, bd, 1, 1, 1)
    out = torch.empty(want.shape, dtype=dt, device=cuda)
    dcn_forward_into(xd.contiguous(memory_format=torch.channels_last), y[:, :18], y[:, 18:], wd,
                     bd, out, 1, 1, 1, mask_is_logit=True)
    assert rel_l2(out, want) <= HALF_REL


@pytest.mark.parametrize("cfg", ["cfg2", "cfg3"])
def test_baseline_configs_full_size(cuda, cfg):
    """BASELINE configs 2 and 3 at full size (NHWC, fp16 / bf16) vs the oracle."""
    from modulated_deform_conv import dcn_forward_into
    if cfg == "cfg2":
        B, C, H, W, Cout, dt, big = 6, 512, 29, 50, 512, torch.float16, 0.0
    else:
        B, C, H, W, Cout, dt, big = 6, 256, 58, 100, 256, torch.bfloat16, 0.05
    x, off, mask, w, _ = dcn_inputs(2026, B, C, H, W, Cout, off_std=2.0, big_frac=big, bias=False)
    x, off, mask, w = (t.to(cuda, dt) for t in (x, off, mask, w))
    want = _oracle(x, off, mask, w, None, 1, 1, 1)
    x_cl = x.contiguous(memory_format=torch.channels_last)
    out = torch.empty(B, Cout, H, W, dtype=dt, device=cuda, memory_format=torch.channels_last)
    dcn_forward_into(x_cl, off, mask, w, None, out, 1, 1, 1)
    torch.cuda.synchronize()
    assert rel_l2(out, want) <= HALF_REL, rel_l2(out, want)
    _watchdog_clean()


def test_fp64_and_grouped_simt(cuda):
    x, off, mask, w, b = dcn_inputs(3, 2, 12, 9, 8, 18, groups=3, dg=2, off_std=1.5)
    x, off, mask, w, b = (t.double().to(cuda) for t in (x, off, mask, w, b))
    want = _oracle(x, off, mask, w, b, 1, 1, 1, groups=3, dg=2)
    out = torch.empty(want.shape, dtype=torch.float64, device=cuda)
    cabi_dcn_forward(x, off, mask, w, b, out, (1, 1), (1, 1), (1, 1), groups=3, dg=2)
    assert rel_l2(out, want) <= FP32_REL


SIMT_CASES = [
    # B, C, H, W, Cout, groups, dg, layout: the small-tile kernel (fewer 64 x 64
    # tiles than two per SM) and, for 313 tiles, the large-tile kernel
    (1, 64, 32, 32, 64, 1, 1, "nchw"),
    (2, 40, 17, 23, 72, 2, 4, "nchw"),          # chunks end at deformable-group edges
    (1, 96, 9, 14, 130, 1, 1, "channels_last"),  # 96 = a full and a partial chunk
    (2, 32, 100, 100, 64, 1, 1, "nchw"),        # large-tile kernel
]


@pytest.mark.parametrize("case", SIMT_CASES, ids=["cfg1", "g2dg4", "c96_cl", "large"])
def test_fp32_simt_kernels(cuda, case):
    B, C, H, W, Cout, groups, dg, layout = case
    x, off, mask, w, b = dcn_inputs(17, B, C, H, W, Cout, groups=groups, dg=dg, off_std=1.0)
    want = _oracle(x, off, mask, w, b, 1, 1, 1, groups=groups, dg=dg)
    x, off, mask, w, b = (t.to(cuda) for t in (x, off, mask, w, b))
    if layout == "channels_last":
        x = x.contiguous(memory_format=torch.channels_last)
    out = torch.full(want.shape, float("nan"), device=cuda)
    cabi_dcn_forward(x, off, mask, w, b, out, (1, 1), (1, 1), (1, 1), groups=groups, dg=dg)
    torch.cuda.synchronize()
    assert rel_l2(out, want) <= FP32_REL and max_abs(out, want) <= FP32_ABS


# Kernel shapes for the small-tile kernel's tap split (three CTAs of a cluster
# take a third of the taps each when there are at least three): 1 x 2 (no
# split), 1 x 4 and 1 x 5 (uneven thirds), 2 x 2 with deformable groups, in
# fp32 and fp64.
TAP_SPLIT_CASES = [
    ((1, 2), (0, 1), 1, torch.float32),
    ((1, 4), (0, 2), 1, torch.float32),
    ((1, 5), (0, 2), 1, torch.float64),
    ((2, 2), (1, 1), 2, torch.float32),
]


@pytest.mark.parametrize("case", TAP_SPLIT_CASES, ids=["k1x2", "k1x4", "k1x5_f64", "k2x2_dg2"])
def test_small_kernel_tap_split_shapes(cuda, case):
    k, pad, dg, dt = case
    x, off, mask, w, b = dcn_inputs(23, 1, 32, 14, 18, 48, k=k, pad=pad, dg=dg, off_std=1.5)
    want = _oracle(x, off, mask, w, b, (1, 1), pad, (1, 1), dg=dg)
    x, off, mask, w, b = (t.to(cuda, dt) for t in (x, off, mask, w, b))
    out = torch.full(want.shape, float("nan"), device=cuda, dtype=dt)
    for _ in range(2):  # the second call overwrites the first's output in full
        cabi_dcn_forward(x, off, mask, w, b, out, (1, 1), pad, (1, 1), dg=dg)
        torch.cuda.synchronize()
        assert rel_l2(out, want) <= FP32_REL and max_abs(out, want) <= FP32_ABS


def test_im2col_compat_ops(cuda):
    """Reference extension column ops vs the reference goldens' column matrices."""
    import _modulated_deform_conv_ext as ext
    for path in _golden_cases():
        z = np.load(path)
        if "columns_nchw" not in z:
            continue
        (kh, kw), (sh, sw), (ph, pw), (dh, dw), groups, dg = _meta(z)
        x, off, mask = (torch.from_numpy(z[n]).to(cuda) for n in ("x", "offset", "mask"))
        B, C, H, W = x.shape
        Ho, Wo = out_size(H, ph, dh, kh, sh), out_size(W, pw, dw, kw, sw)
        col = torch.empty(C * kh * kw, B * Ho * Wo, device=cuda)
        for fn in (ext.modulated_deformable_im2col_cuda, ext.modulated_deformable_im2col_opt_cuda):
            col.fill_(float("nan"))
            fn(x, off, mask, B, C, H, W, Ho, Wo, kh, kw, ph, pw, sh, sw, dh, dw, dg, col)
            ref = torch.from_numpy(z["columns_nchw"])
            assert rel_l2(col, ref) <= FP32_REL and max_abs(col, ref) <= FP32_ABS
        if "columns_nhwc" in z:
            T = kh * kw
            xn = x.permute(0, 2, 3, 1).contiguous()
            offn = off.permute(0, 2, 3, 1).contiguous()
            mkn = mask.permute(0, 2, 3, 1).contiguous()
            coln = torch.full((B * Ho * Wo, T * C), float("nan"), device=cuda)
            ext.modulated_deformable_im2col_nhwc_cuda(xn, offn, mkn, B, C, H, W, Ho, Wo, kh, kw,
                                                      ph, pw, sh, sw, dh, dw, 1, coln)
            ref = torch.from_numpy(z["columns_nhwc"])
            assert rel_l2(coln, ref) <= FP32_REL and max_abs(coln, ref) <= FP32_ABS
            # fused y [B, Ho, Wo, 3T]: offsets + pre-sigmoid mask
            y = torch.cat([offn, torch.logit(mkn.double()).float()], -1).contiguous()
            coln.fill_(float("nan"))
            ext.modulated_deformable_im2col_nhwc_cuda(xn, y, y, B, C, H, W, Ho, Wo, kh, kw,
                                                      ph, pw, sh, sw, dh, dw, 1, coln)
            assert rel_l2(coln, ref) <= FP32_REL


def test_errors_are_raised(cuda):
    from modulated_deform_conv import modulated_deform_conv2d
    x, off, mask, w, b = (t.to(cuda) for t in dcn_inputs(1, 1, 8, 6, 6, 8))
    with pytest.raises(RuntimeError):
        modulated_deform_conv2d(x, off[:, :10], mask, w, b, 1, 1, 1)      # wrong offset channels
    with pytest.raises(RuntimeError):
        modulated_deform_conv2d(x, off, mask, w, b, 1, 1, 1, 3, 1)        # groups must divide


@pytest.mark.parametrize("dt", [torch.float32, torch.float16], ids=["f32", "f16"])
def test_empty_batch(cuda, dt):
    """A batch of zero images gives an empty output and zero gradients, through
    the NCHW Function and through the Pack module (the NHWC split path)."""
    import modulated_deform_conv as mdc
    x = torch.zeros(0, 16, 8, 9, device=cuda, dtype=dt, requires_grad=True)
    off = torch.zeros(0, 18, 8, 9, device=cuda, dtype=dt, requires_grad=True)
    mask = torch.zeros(0, 9, 8, 9, device=cuda, dtype=dt, requires_grad=True)
    w = torch.randn(24, 16, 3, 3, device=cuda, dtype=dt, requires_grad=True)
    b = torch.randn(24, device=cuda, dtype=dt, requires_grad=True)
    out = mdc.modulated_deform_conv2d(x, off, mask, w, b, 1, 1, 1)
    assert out.shape == (0, 24, 8, 9) and out.dtype == dt
    out.sum().backward()
    assert x.grad.shape == x.shape and off.grad.shape == off.shape and mask.grad.shape == mask.shape
    assert not torch.count_nonzero(w.grad) and not torch.count_nonzero(b.grad)
    m = mdc.ModulatedDeformConv2dPack(16, 24, 3, padding=1).to(cuda, dt)
    xp = torch.zeros(0, 16, 8, 9, device=cuda, dtype=dt, requires_grad=True)
    y = m(xp)
    assert y.shape == (0, 24, 8, 9)
    y.sum().backward()
    assert xp.grad.shape == xp.shape
    assert not torch.count_nonzero(m.weight.grad) and not torch.count_nonzero(m.bias.grad)
    assert not torch.count_nonzero(m.conv_offset.weight.grad)


@pytest.mark.parametrize("dt", [torch.float32, torch.float16], ids=["f32_simt", "f16_tc"])
def test_sampling_on_gate_and_edges(cuda, dt):
    """Sampling positions exactly on the bilinear gate and the image edges
    (h or w = -1, -0.5, 0, H-1, H-0.5, H and between): samples at -1 or H are
    dropped, corners outside [0, H-1] x [0, W-1] count as zero -- the
    oracle's semantics, through the exact SIMT path (fp32) and the
    tensor-core path (fp16, forward and backward)."""
    import modulated_deform_conv as mdc
    B, C, H, W, Cout = 1, 32, 6, 7, 32
    g = torch.Generator().manual_seed(91)
    x = torch.randn(B, C, H, W, generator=g)
    w = torch.randn(Cout, C, 3, 3, generator=g) * 0.1
    b = torch.randn(Cout, generator=g)
    mask = torch.sigmoid(torch.randn(B, 9, H, W, generator=g))
    targets_h = [-1.0, -0.5, 0.0, 0.25, H - 1.0, H - 0.5, float(H), 2.75]
    targets_w = [float(W), -1.0, W - 0.5, -0.5, 0.0, W - 1.0, 3.5, 0.75, 1.0]
    off = torch.zeros(B, 18, H, W)
    n = 0
    for oh in range(H):
        for ow in range(W):
            for t in range(9):
                ki, kj = divmod(t, 3)
                off[0, 2 * t, oh, ow] = targets_h[n % len(targets_h)] - (oh - 1 + ki)
                off[0, 2 * t + 1, oh, ow] = targets_w[n % len(targets_w)] - (ow - 1 + kj)
                n += 1
    xs, offs, masks, ws, bs = (t.to(dt) for t in (x, off, mask, w, b))
    # every target is exact in fp16, so both dtypes sample the same positions
    assert torch.equal(offs.float(), off)
    want = _oracle(xs, offs, masks, ws, bs, 1, 1, 1)
    tens = [xs.to(cuda), offs.to(cuda).requires_grad_(), masks.to(cuda).requires_grad_(),
            ws.to(cuda), bs.to(cuda)]
    if dt == torch.float16:
        tens[0] = tens[0].contiguous(memory_format=torch.channels_last)
    tens[0].requires_grad_()
    out = mdc.modulated_deform_conv2d(*tens, 1, 1, 1)
    o = out.detach()
    if dt == torch.float32:
        assert rel_l2(o, want) <= FP32_REL and max_abs(o, want) <= FP32_ABS
    else:
        assert rel_l2(o, want) <= HALF_REL
    gout = torch.randn(out.shape, generator=torch.Generator().manual_seed(92)).to(dt)
    out.backward(gout.to(cuda))
    gw = oracle.dcn_backward(*(t.float().numpy() for t in (xs, offs, masks, ws, gout)), 1, 1, 1)
    tol = FP32_REL if dt == torch.float32 else HALF_REL
    for t, ref, name in zip(tens[:3], gw[:3], ("x", "offset", "mask")):
        assert rel_l2(t.grad, torch.from_numpy(ref)) <= tol, (name, rel_l2(t.grad, torch.from_numpy(ref)))


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_back_to_back_layers_read_their_predecessor(cuda, dt):
    """A chain of layers, each reading the previous launch's output with no
    synchronisation in between.  Every launch lets the next one start its
    set-up early (programmatic dependent launch) and waits for its
    predecessor before touching memory, so the chain equals, bit for bit, the
    same chain with the device synchronised between layers -- launched
    eagerly and replayed from a CUDA graph."""
    import _modulated_deform_conv_ext as ext
    import modulated_deform_conv as mdc
    B, C, H, W, L = 2, 256, 29, 50, 6
    g = torch.Generator(device=cuda).manual_seed(31)
    x0 = torch.randn(B, C, H, W, device=cuda, generator=g).to(dt).contiguous(
        memory_format=torch.channels_last)
    offs = [(torch.randn(B, 18, H, W, device=cuda, generator=g) * 2).to(dt) for _ in range(L)]
    masks = [torch.rand(B, 9, H, W, device=cuda, generator=g).to(dt) for _ in range(L)]
    wpk = [mdc.packed_weight((torch.randn(C, C, 3, 3, device=cuda, generator=g)
                              * (2.0 / (9 * C)) ** 0.5).to(dt)) for _ in range(L)]

    def chain(outs, sync):
        h = x0
        for i in range(L):
            ext.dcn_forward(h, offs[i], masks[i], wpk[i], None, outs[i], 3, 3, 1, 1, 1, 1, 1, 1,
                            1, 1, False)
            if sync:
                torch.cuda.synchronize()
            h = outs[i]

    want = [torch.empty_like(x0) for _ in range(L)]
    chain(want, True)
    assert all(torch.isfinite(o).all() for o in want)
    got = [torch.full_like(x0, float("nan")) for _ in range(L)]
    for _ in range(3):
        for o in got:
            o.fill_(float("nan"))
        chain(got, False)
        torch.cuda.synchronize()
        assert all(torch.equal(a, b) for a, b in zip(got, want))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        for o in got:
            o.fill_(float("nan"))
        with torch.cuda.graph(graph, stream=side):
            chain(got, False)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        for o in got:
            o.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert all(torch.equal(a, b) for a, b in zip(got, want))
    del graph
