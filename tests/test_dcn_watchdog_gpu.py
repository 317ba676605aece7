"""Failure detection in the fused DCN forward: a barrier wait that runs out.

Every barrier wait in the tensor-core kernel is bounded; a wait that gives up
records its site in the per-device watchdog word, raises the CTA's abort flag
so the other warp roles unwind, lets its in-flight copies land and frees its
tensor memory.  Here the pipeline waits get a limit of one nanosecond
(bevk_set_wait_limit_ns), so the first wait that does not pass at once gives
up: the call must be reported through bevk_device_watchdog with one of the
kernel's site codes, the CUDA context must stay usable, and the next call
with the normal limit must match the oracle again.  No GPU fault is involved:
the kernel returns normally and the host reads the status.

Runs on the single-CTA schedule (output channels <= 128), fp16, NHWC.
"""
import ctypes

import pytest
import torch

from bevk import cabi
from helpers import HALF_REL, cabi_dcn_forward, dcn_inputs, rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu

SITES = {0xB0C1, 0xB0C2, 0xB0C3, 0xB0C4}   # gather-empty, TMA-empty, MMA-full, epilogue


def _watchdog():
    code = ctypes.c_uint(0)
    st = cabi.lib().bevk_device_watchdog(0, ctypes.byref(code))
    return st, code.value


def _problem(cuda, seed):
    B, C, H, W, Cout = 2, 64, 12, 16, 64
    x, off, mask, w, b = dcn_inputs(seed, B, C, H, W, Cout)
    want = torch.from_numpy(oracle.dcn_forward(
        x.half().float().numpy(), off.half().float().numpy(), mask.half().float().numpy(),
        w.half().float().numpy(), b.half().float().numpy(), 1, 1, 1))
    x, off, mask, w, b = (t.to(cuda, torch.float16) for t in (x, off, mask, w, b))
    x = x.contiguous(memory_format=torch.channels_last)
    return x, off, mask, w, b, want


def test_expired_wait_is_reported_and_the_device_recovers(cuda):
    L = cabi.lib()
    x, off, mask, w, b, want = _problem(cuda, 61)
    assert _watchdog() == (0, 0)
    out = torch.empty(want.shape, device=cuda, dtype=torch.float16)
    cabi.check(L.bevk_set_wait_limit_ns(0, 1), "set_wait_limit")
    try:
        cabi_dcn_forward(x, off, mask, w, b, out, (1, 1), (1, 1), (1, 1))
        st, code = _watchdog()
    finally:
        cabi.check(L.bevk_set_wait_limit_ns(0, 0), "set_wait_limit")
    assert st == cabi.ERR_DEVICE_TIMEOUT, (st, cabi.last_error())
    assert code in SITES, hex(code)
    # the watchdog word was cleared by the read
    assert _watchdog() == (0, 0)
    # the context is intact: ordinary CUDA work and the next call succeed
    torch.cuda.synchronize()
    assert float(torch.ones(4, device=cuda).sum()) == 4.0
    for seed in (62, 63):
        x, off, mask, w, b, want = _problem(cuda, seed)
        out = torch.full(want.shape, float("nan"), device=cuda, dtype=torch.float16)
        cabi_dcn_forward(x, off, mask, w, b, out, (1, 1), (1, 1), (1, 1))
        torch.cuda.synchronize()
        assert rel_l2(out, want) <= HALF_REL
    assert _watchdog() == (0, 0)


def test_wait_limit_rejects_a_bad_device(cuda):
    st = cabi.lib().bevk_set_wait_limit_ns(10_000, 1)
    assert st == cabi.ERR_INVALID_ARGUMENT
