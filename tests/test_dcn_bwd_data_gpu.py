"""bevk_dcn_backward_data (grad_input by bucketed gather, grad_offset /
grad_mask and the column matrix from one pass over the samples) against the
CPU oracle's DCN backward, and its column matrix against bevk_dcn_columns.

Tolerances: fp32 within 1e-5 relative L2; fp16/bf16 within 5e-3 relative L2 of
the fp32 oracle on the up-cast inputs; the column matrix bit-identical to the
im2col kernel's for fp32 (fp32 interpolation, rounded once), and for fp16 /
bf16 built as the fused forward builds its tiles (weights in the input type,
a packed multiply and three packed FMAs, each step rounded to the type):
within 2e-3 relative L2 of the im2col kernel's for fp16 and 1e-2 for bf16
(an 8-bit mantissa rounded four times; grad_weight, which sums the column
matrix over the pixels, is checked against the oracle at 5e-3 elsewhere).
"""
import ctypes

import pytest
import torch

from bevk import cabi
from helpers import DT, FP32_REL, HALF_REL, dcn_inputs, problem, rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu

CASES = [
    # B, C, H, W, Cout, k, stride, pad, dil, dg, big_frac
    (2, 32, 9, 11, 16, (3, 3), (1, 1), (1, 1), (1, 1), 1, 0.0),
    (2, 64, 10, 13, 24, (3, 3), (2, 2), (1, 1), (1, 1), 2, 0.1),     # deformable groups, stride 2
    (1, 72, 8, 9, 40, (3, 3), (1, 1), (2, 2), (2, 2), 1, 0.05),      # 9 vectors / pixel (fp16)
    (1, 48, 7, 12, 8, (1, 3), (1, 1), (0, 1), (1, 1), 3, 0.0),       # 1x3, 16 channels / group
    (1, 512, 6, 7, 32, (3, 3), (1, 1), (1, 1), (1, 1), 1, 0.0),      # two channel chunks
]


def _dcol(go_nchw, w, dt):
    """dcol [M, T*C] (k = t*C + c) = dO . W_tap in dtype dt."""
    Cout, C, kh, kw = w.shape
    go = go_nchw.permute(0, 2, 3, 1).reshape(-1, Cout).to(dt)
    wt = w.permute(0, 2, 3, 1).reshape(Cout, kh * kw * C).to(dt)
    return (go @ wt).contiguous()


def _run(case, dt, grad_dt, cuda, seed=5):
    from modulated_deform_conv.modulated_deform_conv import _load_ext
    ext = _load_ext()
    B, C, H, W, Cout, k, st, pd, dl, dg, big = case
    x, off, mask, w, _ = dcn_inputs(seed, B, C, H, W, Cout, k, st, pd, dl, dg=dg,
                                    big_frac=big, bias=False)
    Ho, Wo = off.shape[2], off.shape[3]
    gout = torch.randn(B, Cout, Ho, Wo, generator=torch.Generator().manual_seed(seed + 1))
    xs, offs, masks, ws, gos = (t.to(dt) for t in (x, off, mask, w, gout))
    want = oracle.dcn_backward(*(t.float().numpy() for t in (xs, offs, masks, ws, gos)),
                               st, pd, dl, 1, dg, with_bias=False)
    xg = xs.to(cuda).contiguous(memory_format=torch.channels_last)
    og, mg = offs.to(cuda), masks.to(cuda)
    dcol = _dcol(gos.to(cuda), ws.to(cuda), dt)
    T = k[0] * k[1]
    gx = torch.full((B, C, H, W), float("nan"), device=cuda, dtype=grad_dt).contiguous(
        memory_format=torch.channels_last)
    goff = torch.full(og.shape, float("nan"), device=cuda, dtype=grad_dt)
    gm = torch.full(mg.shape, float("nan"), device=cuda, dtype=grad_dt)
    col = torch.empty(B * Ho * Wo, T * C, device=cuda, dtype=dt)
    done = ext.dcn_backward_data(dcol, xg, og, mg, False, C, H, W, k[0], k[1], st[0], st[1],
                                 pd[0], pd[1], dl[0], dl[1], dg, gx, goff, gm, col)
    assert done
    torch.cuda.synchronize()
    ref_col = ext.dcn_columns(xg, og, mg, k[0], k[1], st[0], st[1], pd[0], pd[1], dl[0], dl[1],
                              dg, 1)
    return (gx, goff, gm), want, col, ref_col


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16],
                         ids=["f32", "f16", "bf16"])
def test_matches_oracle(cuda, case, dt):
    got, want, col, ref_col = _run(case, dt, dt, cuda)
    tol = FP32_REL if dt == torch.float32 else HALF_REL
    for name, g, ref in zip(("grad_input", "grad_offset", "grad_mask"), got, want[:3]):
        assert g.dtype == dt
        assert not torch.isnan(g).any(), name          # every element written
        assert rel_l2(g, torch.from_numpy(ref)) <= tol, (name, rel_l2(g, torch.from_numpy(ref)))
    if dt == torch.float16:
        assert rel_l2(col, ref_col) <= 2e-3, rel_l2(col, ref_col)
    elif dt == torch.bfloat16:
        assert rel_l2(col, ref_col) <= 1e-2, rel_l2(col, ref_col)
    else:
        assert torch.equal(col, ref_col)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_fp32_gradients_of_half_inputs(cuda, dt):
    got, want, _, _ = _run(CASES[1], dt, torch.float32, cuda, seed=8)
    for name, g, ref in zip(("grad_input", "grad_offset", "grad_mask"), got, want[:3]):
        assert g.dtype == torch.float32
        assert rel_l2(g, torch.from_numpy(ref)) <= HALF_REL, name


def test_subsets_and_unsupported_layouts(cuda):
    """grad_input alone (no input), the column matrix alone (no dcol), and a
    channel count that is not whole 16-byte vectors (returns False, writes
    nothing)."""
    from modulated_deform_conv.modulated_deform_conv import _load_ext
    ext = _load_ext()
    B, C, H, W, Cout = 1, 32, 8, 10, 8
    x, off, mask, w, _ = dcn_inputs(11, B, C, H, W, Cout, bias=False, big_frac=0.1)
    gout = torch.randn(B, Cout, H, W, generator=torch.Generator().manual_seed(12))
    want = oracle.dcn_backward(x.numpy(), off.numpy(), mask.numpy(), w.numpy(), gout.numpy(),
                               1, 1, 1, with_bias=False)
    xg = x.to(cuda).contiguous(memory_format=torch.channels_last)
    og, mg = off.to(cuda), mask.to(cuda)
    dcol = _dcol(gout.to(cuda), w.to(cuda), torch.float32)
    gx = torch.full((B, C, H, W), float("nan"), device=cuda).contiguous(
        memory_format=torch.channels_last)
    assert ext.dcn_backward_data(dcol, None, og, mg, False, C, H, W, 3, 3, 1, 1, 1, 1, 1, 1, 1,
                                 gx, None, None, None)
    assert rel_l2(gx, torch.from_numpy(want[0])) <= FP32_REL
    col = torch.empty(B * H * W, 9 * C, device=cuda)
    assert ext.dcn_backward_data(None, xg, og, mg, False, C, H, W, 3, 3, 1, 1, 1, 1, 1, 1, 1,
                                 None, None, None, col)
    assert torch.equal(col, ext.dcn_columns(xg, og, mg, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1))
    # fp16 with 20 channels: 40-byte pixel rows are not whole 16-byte vectors
    C2 = 20
    x2, off2, mask2, _, _ = dcn_inputs(13, B, C2, H, W, Cout, bias=False)
    x2g = x2.to(cuda).half().contiguous(memory_format=torch.channels_last)
    gx2 = torch.full((B, C2, H, W), 7.0, device=cuda, dtype=torch.half)
    dcol2 = torch.zeros(B * H * W, 9 * C2, device=cuda, dtype=torch.half)
    assert not ext.dcn_backward_data(dcol2, x2g, off2.to(cuda).half(), mask2.to(cuda).half(),
                                     False, C2, H, W, 3, 3, 1, 1, 1, 1, 1, 1, 1, gx2, None, None,
                                     None)
    torch.cuda.synchronize()
    assert bool((gx2 == 7.0).all())


def test_cabi_contract(cuda):
    """Through ctypes: NULL tensors and a short workspace are rejected; the
    full call matches the oracle."""
    L = cabi.lib()
    B, C, H, W, Cout = 2, 16, 7, 9, 8
    x, off, mask, w, _ = dcn_inputs(21, B, C, H, W, Cout, bias=False, big_frac=0.05)
    gout = torch.randn(B, Cout, H, W, generator=torch.Generator().manual_seed(22))
    want = oracle.dcn_backward(x.numpy(), off.numpy(), mask.numpy(), w.numpy(), gout.numpy(),
                               1, 1, 1, with_bias=False)
    xg = x.to(cuda).contiguous(memory_format=torch.channels_last)
    og, mg = off.to(cuda), mask.to(cuda)
    dcol = _dcol(gout.to(cuda), w.to(cuda), torch.float32)
    gx = torch.empty(B, C, H, W, device=cuda).contiguous(memory_format=torch.channels_last)
    goff, gm = torch.empty_like(og), torch.empty_like(mg)
    col = torch.empty(B * H * W, 9 * C, device=cuda)
    a = cabi.DcnBackwardDataArgs()
    a.problem = problem(xg, og, mg, gx, 1, (3, 3), (1, 1), (1, 1), (1, 1))
    a.grad_dtype = DT[torch.float32]
    a.dcol_ld, a.col_ld = dcol.stride(0), col.stride(0)
    for i in range(4):
        a.grad_input_strides[i] = gx.stride(i)
        a.grad_offset_strides[i] = goff.stride(i)
        a.grad_mask_strides[i] = gm.stride(i)
    nbytes = L.bevk_dcn_backward_data_workspace_bytes(ctypes.byref(a.problem))
    assert nbytes >= 4 * (B * H * W * 9) * 8
    ws = torch.empty(nbytes, device=cuda, dtype=torch.uint8)
    stream = torch.cuda.current_stream().cuda_stream

    def call(input_ptr, dcol_ptr, ws_bytes):
        return L.bevk_dcn_backward_data(ctypes.byref(a), input_ptr, og.data_ptr(), mg.data_ptr(),
                                        dcol_ptr, gx.data_ptr(), goff.data_ptr(), gm.data_ptr(),
                                        col.data_ptr(), ws.data_ptr(), ws_bytes, stream)

    assert call(None, dcol.data_ptr(), nbytes) == cabi.ERR_INVALID_ARGUMENT
    assert call(xg.data_ptr(), None, nbytes) == cabi.ERR_INVALID_ARGUMENT
    assert call(xg.data_ptr(), dcol.data_ptr(), nbytes - 16) == cabi.ERR_WORKSPACE
    assert call(xg.data_ptr(), dcol.data_ptr(), nbytes) == cabi.OK, cabi.last_error()
    torch.cuda.synchronize()
    for g, ref in zip((gx, goff, gm), want[:3]):
        assert rel_l2(g, torch.from_numpy(ref)) <= FP32_REL
