"""The tensor-core DCN forward's K-split schedule against the oracle.

Problems with more than 256 output channels whose tiles fill at most one wave
of the GPU run as 2-CTA clusters with paired M=256 MMAs into two 256-column
accumulators, the K loop split in two: the two clusters of a tile each finish
half of the 512 columns from the other's handed-over fp32 partial sums (the
forward workspace holds them and the per-tile tickets).  Without a workspace
the same problems take the N-split schedule; both must match the oracle, as
must runs whose workspace starts out as garbage and CUDA-graph replays (the
tickets carry the launch's grid id and are cleared after the exchange, so
they need no initialisation).
"""
import ctypes

import pytest
import torch

from bevk import cabi
from helpers import HALF_REL, cabi_dcn_forward, dcn_inputs, problem, rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu

SPLIT_CASES = [
    # B, C, H, W, Cout, stride, bias, relu
    (1, 128, 9, 11, 512, 1, True, False),     # one tile, rows 99 of 256
    (2, 136, 13, 17, 520, 1, True, True),     # odd K stages (27), 2 column tiles, ReLU
    (3, 256, 16, 30, 768, 1, False, False),   # 12 tiles, second column tile half empty
    (2, 128, 10, 19, 320, 2, True, False),    # strided, 320 of 512 columns
]


def _oracle(x, off, mask, w, b, stride, relu=False):
    y = torch.from_numpy(oracle.dcn_forward(
        x.float().cpu().numpy(), off.float().cpu().numpy(), mask.float().cpu().numpy(),
        w.float().cpu().numpy(), None if b is None else b.float().cpu().numpy(),
        stride, 1, 1))
    return y.clamp_min(0) if relu else y


def _watchdog_clean():
    code = ctypes.c_uint(0)
    st = cabi.lib().bevk_device_watchdog(0, ctypes.byref(code))
    assert st == 0 and code.value == 0, f"device watchdog fired: 0x{code.value:x}"


def _split_bytes(p):
    return cabi.lib().bevk_dcn_forward_workspace_bytes(ctypes.byref(p))


def _setup(cuda, case, dt, seed=7):
    B, C, H, W, Cout, s, bias, relu = case
    x, off, mask, w, b = dcn_inputs(seed, B, C, H, W, Cout, stride=(s, s), off_std=2.0,
                                    big_frac=0.02, bias=bias)
    x, off, mask, w = (t.to(cuda, dt) for t in (x, off, mask, w))
    b = b.to(cuda, dt) if b is not None else None
    want = _oracle(x, off, mask, w, b, s, relu)
    return x, off, mask, w, b, want


@pytest.mark.parametrize("case", SPLIT_CASES, ids=[f"k{i}" for i in range(len(SPLIT_CASES))])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_split_and_unsplit_match_the_oracle(cuda, case, dt):
    x, off, mask, w, b, want = _setup(cuda, case, dt)
    s, relu = case[5], case[7]
    x_cl = x.contiguous(memory_format=torch.channels_last)
    p = problem(x_cl, off, mask, torch.empty(want.shape, device=cuda, dtype=dt,
                                             memory_format=torch.channels_last),
                want.shape[1], (3, 3), (s, s), (1, 1), (1, 1), has_bias=b is not None)
    assert _split_bytes(p) > 0      # channel-contiguous input: the K-split scratch alone
    for workspace in (True, False):
        out = torch.full(want.shape, float("nan"), device=cuda, dtype=dt).contiguous(
            memory_format=torch.channels_last)
        cabi_dcn_forward(x_cl, off, mask, w, b, out, (s, s), (1, 1), (1, 1),
                         workspace=workspace, act_relu=relu)
        torch.cuda.synchronize()
        assert rel_l2(out, want) <= HALF_REL, (workspace, rel_l2(out, want))
    _watchdog_clean()


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_split_with_nchw_input(cuda, dt):
    """NCHW input: the workspace holds the NHWC copy, then the K-split scratch."""
    x, off, mask, w, b, want = _setup(cuda, SPLIT_CASES[1], dt, seed=9)
    out = torch.empty(want.shape, device=cuda, dtype=dt)
    cabi_dcn_forward(x, off, mask, w, b, out, (1, 1), (1, 1), (1, 1), act_relu=True)
    torch.cuda.synchronize()
    assert rel_l2(out, want) <= HALF_REL
    _watchdog_clean()


def test_garbage_workspace(cuda):
    """Tickets and partial sums need no initialisation by the caller."""
    L = cabi.lib()
    dt = torch.float16
    x, off, mask, w, b, want = _setup(cuda, SPLIT_CASES[2], dt, seed=11)
    x = x.contiguous(memory_format=torch.channels_last)
    out = torch.empty(want.shape, device=cuda, dtype=dt).contiguous(
        memory_format=torch.channels_last)
    p = problem(x, off, mask, out, w.shape[0], (3, 3), (1, 1), (1, 1), (1, 1),
                has_bias=b is not None)
    stream = torch.cuda.current_stream().cuda_stream
    wpk = torch.empty(L.bevk_dcn_packed_weight_bytes(ctypes.byref(p)), dtype=torch.uint8,
                      device=cuda)
    cabi.check(L.bevk_dcn_pack_weight(ctypes.byref(p), w.contiguous().data_ptr(),
                                      wpk.data_ptr(), stream), "pack")
    nb = _split_bytes(p)
    ws = torch.full((nb,), 0xFF, dtype=torch.uint8, device=cuda)
    for fill in (0x5A, 0x00, None):
        out.fill_(float("nan"))
        cabi.check(L.bevk_dcn_forward(ctypes.byref(p), x.data_ptr(), off.data_ptr(),
                                      mask.data_ptr(), wpk.data_ptr(),
                                      b.data_ptr() if b is not None else None, out.data_ptr(),
                                      ws.data_ptr(), nb, stream), "dcn_forward")
        torch.cuda.synchronize()
        assert rel_l2(out, want) <= HALF_REL
        if fill is not None:
            ws.fill_(fill)       # the next call starts from other garbage
    _watchdog_clean()


def test_split_in_cuda_graph(cuda):
    """Replays of a captured call reuse its workspace and stay correct."""
    from modulated_deform_conv import dcn_forward_into
    dt = torch.float16
    x, off, mask, w, b, want = _setup(cuda, SPLIT_CASES[0], dt, seed=13)
    x = x.contiguous(memory_format=torch.channels_last)
    out = torch.empty(want.shape, device=cuda, dtype=dt).contiguous(
        memory_format=torch.channels_last)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        dcn_forward_into(x, off, mask, w, b, out, 1, 1, 1)       # packs and caches the weight
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dcn_forward_into(x, off, mask, w, b, out, 1, 1, 1)
    for _ in range(3):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert rel_l2(out, want) <= HALF_REL
    del g
    _watchdog_clean()


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_half_sums_that_cancel(cuda, dt):
    """The K parts hand each other fp32 sums: here each part's sum is ~69000
    (past fp16's 65504, rounded there by a few tens) while the output, where
    the two parts cancel, is a few hundred."""
    B, C, H, W, Cout = 1, 128, 12, 12, 512
    g = torch.Generator().manual_seed(5)
    x = torch.randn(B, C, H, W, generator=g) * 8.0
    x[:, :64] += 120.0     # channel chunk 0: K part 0 (18 stages = 2 chunks x 9 taps)
    x[:, 64:] -= 120.0     # channel chunk 1: K part 1
    off = torch.zeros(B, 18, H, W)           # integer sample points: exact interpolation
    mask = torch.ones(B, 9, H, W)
    w = 1.0 + 0.01 * torch.randn(Cout, C, 3, 3, generator=g)
    x, off, mask, w = (t.to(cuda, dt) for t in (x, off, mask, w))
    want = _oracle(x, off, mask, w, None, 1)
    part0 = _oracle(x[:, :64].contiguous(), off, mask, w[:, :64].contiguous(), None, 1)
    assert float(part0.abs().max()) > 65520.0
    x_cl = x.contiguous(memory_format=torch.channels_last)
    out = torch.full(want.shape, float("nan"), device=cuda, dtype=dt).contiguous(
        memory_format=torch.channels_last)
    cabi_dcn_forward(x_cl, off, mask, w, None, out, (1, 1), (1, 1), (1, 1))
    torch.cuda.synchronize()
    assert bool(torch.isfinite(out).all())
    assert rel_l2(out, want) <= HALF_REL, rel_l2(out, want)
    _watchdog_clean()


def test_concurrent_calls_on_two_streams(cuda):
    """Two K-split calls at once on two streams, each with its own workspace:
    together their clusters exceed one wave, so some CTAs wait for partners
    that start only when the other call's CTAs finish."""
    dt = torch.float16
    B, C, H, W, Cout = 6, 512, 29, 50, 512        # 136 CTAs each: cfg2
    runs = []
    for seed in (21, 22):
        x, off, mask, w, _ = dcn_inputs(seed, B, C, H, W, Cout, off_std=2.0, bias=False)
        x, off, mask, w = (t.to(cuda, dt) for t in (x, off, mask, w))
        want = _oracle(x, off, mask, w, None, 1)
        x = x.contiguous(memory_format=torch.channels_last)
        out = torch.empty(want.shape, device=cuda, dtype=dt).contiguous(
            memory_format=torch.channels_last)
        runs.append((x, off, mask, w, out, want))
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    for rep in range(3):
        for (x, off, mask, w, out, want), st in zip(runs, streams):
            out.fill_(float("nan"))
        torch.cuda.synchronize()
        for (x, off, mask, w, out, want), st in zip(runs, streams):
            with torch.cuda.stream(st):
                cabi_dcn_forward(x, off, mask, w, None, out, (1, 1), (1, 1), (1, 1))
        torch.cuda.synchronize()
        for x, off, mask, w, out, want in runs:
            assert rel_l2(out, want) <= HALF_REL, (rep, rel_l2(out, want))
    _watchdog_clean()


def test_no_split_beyond_one_wave(cuda):
    """Tiles that do not fit in one wave (here 4 x 38 CTAs) take no K split."""
    B, C, H, W, Cout = 4, 256, 40, 60, 512
    x = torch.empty(B, C, H, W, device=cuda, dtype=torch.float16,
                    memory_format=torch.channels_last)
    off = torch.empty(B, 18, H, W, device=cuda, dtype=torch.float16)
    mask = torch.empty(B, 9, H, W, device=cuda, dtype=torch.float16)
    out = torch.empty(B, Cout, H, W, device=cuda, dtype=torch.float16,
                      memory_format=torch.channels_last)
    p = problem(x, off, mask, out, Cout, (3, 3), (1, 1), (1, 1), (1, 1))
    assert _split_bytes(p) == 0
    # one tile fewer than a wave's worth (37 x 4 = 148 CTAs): split
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    tiles = sms // 4
    Hs = (tiles * 256) // (W * B)
    x2 = torch.empty(B, C, Hs, W, device=cuda, dtype=torch.float16,
                     memory_format=torch.channels_last)
    off2 = torch.empty(B, 18, Hs, W, device=cuda, dtype=torch.float16)
    mask2 = torch.empty(B, 9, Hs, W, device=cuda, dtype=torch.float16)
    out2 = torch.empty(B, Cout, Hs, W, device=cuda, dtype=torch.float16,
                       memory_format=torch.channels_last)
    p2 = problem(x2, off2, mask2, out2, Cout, (3, 3), (1, 1), (1, 1), (1, 1))
    n_tiles = -(-(B * Hs * W) // 256)
    assert n_tiles <= tiles
    tickets = (n_tiles * 2 * 16 + 255) // 256 * 256
    assert _split_bytes(p2) == tickets + n_tiles * 4 * 256 * 128 * 4
