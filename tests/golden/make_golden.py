"""Generate the golden fixtures in tests/golden from the reference's own goldens.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference <path-to-bev-kernels>

The reference ships no test vectors; its only correctness oracles are the
pure-PyTorch golden functions inside its modules.  This script imports those
modules by file path and records their outputs on small seeded inputs:

* ``modulated_deform_conv/modulated_deform_conv.py:216-266``
  (``modulated_deformable_im2col_pytorch``, NCHW columns) followed by the grouped
  ``mm`` + bias of ``ModulatedDeformConv2dFunction.forward`` (:380-401);
* ``modulated_deform_conv/fused_tl.py:177-227`` (``dcn_columns_golden_nhwc`` /
  ``dcn_forward_golden_nhwc``, NHWC, k = t*Cin + ci);
* the backward goldens ``modulated_deformable_col2im_pytorch`` and
  ``modulated_deformable_col2im_coord_pytorch`` (:269-312: autograd through the
  differentiable im2col golden) on the column gradient W^T . grad_out, and
  grad_weight / grad_bias by autograd through the same golden forward.

MSDA has no reference golden (the reference's MSDA exists only as MUSA kernels);
``msda_*.npz`` are produced by the independent grid_sample formulation in
``oracle/msda_grid_sample.py`` and only guard the C oracle against regressions.

Each fixture is an ``.npz`` with the inputs, the expected output and the
convolution parameters; float32 throughout.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _load_module(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _dcn_inputs(g, B, C, H, W, Cout, k, stride, pad, dil, groups, dg, off_std,
                big_frac=0.0, integer_taps=False, bias=True):
    kh, kw = k
    Ho = (H + 2 * pad[0] - (dil[0] * (kh - 1) + 1)) // stride[0] + 1
    Wo = (W + 2 * pad[1] - (dil[1] * (kw - 1) + 1)) // stride[1] + 1
    T = kh * kw
    x = torch.randn(B, C, H, W, generator=g)
    fan_in = (C // groups) * T
    w = torch.randn(Cout, C // groups, kh, kw, generator=g) * (2.0 / fan_in) ** 0.5
    off = torch.randn(B, 2 * dg * T, Ho, Wo, generator=g) * off_std
    if integer_taps:
        # taps landing exactly on integer / boundary coordinates (h_im in {-1, 0, H-1, H})
        off = torch.randint(-3, 4, off.shape, generator=g).float()
        off[..., 0, :] = -1.0
        off[..., -1, :] = float(H)
    if big_frac > 0:
        sel = torch.rand(off.shape, generator=g) < big_frac
        sign = torch.where(torch.rand(off.shape, generator=g) < 0.5, -1.0, 1.0)
        off = torch.where(sel, sign * (H + 4), off)
    mask = torch.sigmoid(torch.randn(B, dg * T, Ho, Wo, generator=g))
    b = torch.randn(Cout, generator=g) if bias else None
    return x, off, mask, w, b


def dcn_cases():
    # name, B, C, H, W, Cout, k, stride, pad, dil, groups, dg, off_std, extra
    return [
        ("dcn_cfg1", 1, 64, 32, 32, 64, (3, 3), (1, 1), (1, 1), (1, 1), 1, 1, 1.0, {}),
        ("dcn_boundary_taps", 2, 8, 6, 7, 8, (3, 3), (1, 1), (1, 1), (1, 1), 1, 1, 1.0,
         {"integer_taps": True}),
        ("dcn_far_offsets", 2, 16, 9, 11, 16, (3, 3), (1, 1), (1, 1), (1, 1), 1, 1, 2.0,
         {"big_frac": 0.05}),
        ("dcn_stride2_dil2", 2, 8, 13, 10, 12, (3, 3), (2, 2), (2, 2), (2, 2), 1, 1, 1.5, {}),
        ("dcn_groups2_dg2", 1, 16, 8, 9, 8, (3, 3), (1, 1), (1, 1), (1, 1), 2, 2, 1.0, {}),
        ("dcn_k3x1_nobias", 2, 8, 7, 6, 6, (3, 1), (1, 1), (1, 0), (1, 1), 1, 1, 1.0,
         {"bias": False}),
        ("dcn_asym_stride", 1, 24, 10, 12, 16, (3, 3), (2, 1), (1, 2), (1, 2), 1, 1, 1.0, {}),
    ]


def make_dcn(ref_mdc, ref_tl, out_dir):
    g = torch.Generator().manual_seed(20261201)
    for name, B, C, H, W, Cout, k, st, pd, dl, groups, dg, off_std, extra in dcn_cases():
        x, off, mask, w, b = _dcn_inputs(g, B, C, H, W, Cout, k, st, pd, dl, groups, dg,
                                         off_std, **extra)
        kh, kw = k
        col = ref_mdc.modulated_deformable_im2col_pytorch(
            x, off, mask, kh, kw, pd[0], pd[1], st[0], st[1], dl[0], dl[1], dg)
        Ho, Wo = col.shape[2], col.shape[3]
        col2 = col.reshape(C * kh * kw, B * Ho * Wo)
        cg = col2.view(groups, -1, B * Ho * Wo)
        wg = w.view(groups, Cout // groups, -1)
        out = torch.cat([wg[i] @ cg[i] for i in range(groups)], 0)
        out = out.view(Cout, B, Ho, Wo).permute(1, 0, 2, 3).contiguous()
        if b is not None:
            out = out + b.view(1, -1, 1, 1)
        arrays = dict(x=x, offset=off, mask=mask, weight=w, out=out)
        # ---- backward goldens
        gout = torch.randn(out.shape, generator=g)
        dcol = torch.cat([wg[i].t() @ gout.permute(1, 0, 2, 3).reshape(groups, Cout // groups, -1)[i]
                          for i in range(groups)], 0).view(C * kh * kw, B, Ho, Wo)
        grad_x = ref_mdc.modulated_deformable_col2im_pytorch(
            dcol, x, off, mask, kh, kw, pd[0], pd[1], st[0], st[1], dl[0], dl[1], dg)
        grad_off, grad_mask = ref_mdc.modulated_deformable_col2im_coord_pytorch(
            dcol, x, off, mask, kh, kw, pd[0], pd[1], st[0], st[1], dl[0], dl[1], dg)
        w_var = w.detach().clone().requires_grad_(True)
        cg_fwd = col2.detach().view(groups, -1, B * Ho * Wo)
        out_w = torch.cat([w_var.view(groups, Cout // groups, -1)[i] @ cg_fwd[i]
                           for i in range(groups)], 0)
        (grad_w,) = torch.autograd.grad(out_w, [w_var], grad_outputs=gout.permute(
            1, 0, 2, 3).reshape(Cout, B * Ho * Wo))
        arrays.update(grad_out=gout, grad_x=grad_x, grad_offset=grad_off, grad_mask=grad_mask,
                      grad_weight=grad_w)
        if b is not None:
            arrays["grad_bias"] = gout.sum(dim=(0, 2, 3))
        small = col2.numel() <= 200_000          # keep the fixture set small
        if small:
            arrays["columns_nchw"] = col2
        if b is not None:
            arrays["bias"] = b
        if groups == 1 and dg == 1:
            # NHWC goldens (fused_tl.py) on the same data, channel-last layouts
            x_nhwc = x.permute(0, 2, 3, 1).contiguous()
            off_nhwc = off.permute(0, 2, 3, 1).contiguous()
            mask_nhwc = mask.permute(0, 2, 3, 1).contiguous()
            cols_nhwc = ref_tl.dcn_columns_golden_nhwc(
                x_nhwc, off_nhwc, mask_nhwc, kh, kw, st[0], st[1], pd[0], pd[1], dl[0], dl[1])
            out_nhwc = ref_tl.dcn_forward_golden_nhwc(
                x_nhwc, off_nhwc, mask_nhwc, w, b, stride=st, padding=pd, dilation=dl)
            if small:
                arrays["columns_nhwc"] = cols_nhwc
            arrays["out_nhwc"] = out_nhwc
        meta = np.array([kh, kw, st[0], st[1], pd[0], pd[1], dl[0], dl[1], groups, dg],
                        np.int64)
        np.savez_compressed(os.path.join(out_dir, name + ".npz"), meta=meta,
                            **{k_: v.detach().numpy().astype(np.float32)
                               for k_, v in arrays.items()})
        print("wrote", name, tuple(out.shape))


def make_msda(out_dir):
    sys.path.insert(0, REPO)
    from oracle.msda_grid_sample import msda_forward_grid_sample

    g = torch.Generator().manual_seed(7)
    cases = [
        ("msda_small_4lvl", 2, 8, 8, 30, 4, [(12, 20), (6, 10), (3, 5), (2, 3)]),
        ("msda_small_1lvl", 2, 8, 32, 40, 4, [(8, 10)]),
    ]
    for name, B, M, C, Q, P, shapes in cases:
        L = len(shapes)
        sizes = [h * w for h, w in shapes]
        S = sum(sizes)
        lsi = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)
        value = torch.randn(B, S, M, C, generator=g)
        loc = torch.rand(B, Q, M, L, P, 2, generator=g)
        out_sel = torch.rand(B, Q, M, L, P, 2, generator=g) < 0.05
        loc = torch.where(out_sel, loc * 1.6 - 0.3, loc)       # some points outside [0,1]
        attn = torch.softmax(torch.randn(B, Q, M, L * P, generator=g), -1).view(B, Q, M, L, P)
        out = msda_forward_grid_sample(value, torch.tensor(shapes), loc, attn)
        np.savez_compressed(os.path.join(out_dir, name + ".npz"),
                            value=value.numpy(), spatial_shapes=np.array(shapes, np.int64),
                            level_start_index=lsi, sampling_loc=loc.numpy(),
                            attn_weight=attn.numpy(), out=out.numpy())
        print("wrote", name, tuple(out.shape))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("BEVK_REFERENCE"),
                    help="root of the reference checkout (or set BEVK_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or BEVK_REFERENCE) is required")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    pkg = os.path.join(args.reference, "modulated_deform_conv")
    ref_mdc = _load_module("_bevk_ref_mdc", os.path.join(pkg, "modulated_deform_conv.py"))
    ref_tl = _load_module("_bevk_ref_fused_tl", os.path.join(pkg, "fused_tl.py"))
    make_dcn(ref_mdc, ref_tl, args.out)
    make_msda(args.out)


if __name__ == "__main__":
    main()
