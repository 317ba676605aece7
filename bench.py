#!/usr/bin/env python
"""Benchmark of the B200 deformable-sampling hot path (DCNv2 / MSDA forward).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Headline workload: DCNv2 forward of the BEVFormer
ResNet-101-DCN stage-4 conv2 -- 6 cameras x 512 -> 512 channels, 29 x 50, 3x3,
stride 1, pad 1, NHWC fp16 with fp32 accumulation, offsets ~N(0, 2^2) px,
mask = sigmoid(N(0, 1)).  A step is one forward over one 6-camera batch; each
rank runs its own batch (cameras sharded by rank, no collective on the data
path), so scaling is weak and ``value`` is the aggregate TFLOP/s of all ranks.

Timing: W untimed warm-up steps, then exactly K steps replayed from a CUDA
graph and timed with CUDA events on the launching stream, bracketed by a
barrier and cuda.synchronize(); the max over ranks is reported.  Inputs rotate
through enough independent sets that the working set exceeds the 126 MB L2,
so no step finds its inputs in L2 from the step before.  SM clocks and clock
event reasons are sampled through NVML during the timed region.

Also reported on the same line: ``e2e`` (the same metric through the public
``modulated_deform_conv2d`` call with inputs copied from pinned host memory and
the output copied back every step), the roofline of the fused kernel against
MEASURED_PEAKS.json, the CPU oracle timed on a bounded sample (rank 0, N = 1),
``legs`` (the Pack forward, the DCN and MSDA backward, the 5-chain: 48 images,
each a cfg5 MSDA camera slice and a cfg3 DCN image, in contiguous blocks per
rank, strong scaling, per-image checksums all-gathered and checked on rank 0
outside the timed region) and, last, ``configs``: for each BASELINE config
(1-5) the device us/call, its roofline fraction (tensor peak for DCN, HBM for
MSDA), the end-to-end us/step through the public call with pinned host
buffers, the CPU oracle's us/call on all host threads, and for MSDA the
fp16/bf16 variants.  A spin kernel queued ahead of each start event keeps the
host's submission latency out of the timed region.

``--impl reference`` times the reference algorithm on the host cores instead
(the CPU oracle restatement in oracle/, all threads) on the same workload and
metric; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "bev-kernels_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "DCNv2 fwd TFLOP/s & MSDA fwd µs/call on B200, as % of roofline"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

DCN_CFGS = {
    "cfg1": dict(B=1, C=64, H=32, W=32, Cout=64, dtype="float32", big=0.0, off_std=1.0,
                 bias=True, layout="nchw",
                 desc="DCNv2 plumbing fwd: 1x64->64, 32x32, 3x3 s1 p1, bias, NCHW fp32"),
    "cfg2": dict(B=6, C=512, H=29, W=50, Cout=512, dtype="float16", big=0.0,
                 desc="DCNv2 stage-4 conv2 fwd: 6x512->512, 29x50, 3x3 s1 p1, NHWC fp16"),
    "cfg3": dict(B=6, C=256, H=58, W=100, Cout=256, dtype="bfloat16", big=0.05,
                 desc="DCNv2 stage-3 conv2 fwd: 6x256->256, 58x100, 3x3 s1 p1, NHWC bf16, "
                      "5% offsets at +-(H+4)"),
}
MSDA_CFGS = {
    "cfg4": dict(B=2, shapes=[(200, 200)], M=8, C=32, Q=40000, P=4, oob=0.02,
                 desc="MSDA TSA fwd: bs 2, 1 level 200x200, 8x32, Q=40000, P=4, fp32"),
    "cfg5": dict(B=6, shapes=[(116, 200), (58, 100), (29, 50), (15, 25)], M=8, C=32, Q=10000,
                 P=8, oob=0.0,
                 desc="MSDA SCA fwd: 6 cams, 4 levels, 8x32, Q=10000, P=8, fp32"),
}


# ----------------------------------------------------------------------------- helpers
def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def _traffic(key):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, or None."""
    path = os.path.join(REPO, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(key)
    except (OSError, ValueError):
        return None


def _out(n, pad, dil, k, stride):
    return (n + 2 * pad - (dil * (k - 1) + 1)) // stride + 1


_ESZ = {"float32": 4, "float16": 2, "bfloat16": 2}


def dcn_work(cfg):
    """Algorithmic FLOPs and unique bytes of one DCN forward: 2*M*N*K FLOPs; input,
    offset, mask, weight, bias and output each read or written once."""
    B, C, H, W, Co = cfg["B"], cfg["C"], cfg["H"], cfg["W"], cfg["Cout"]
    Ho, Wo = _out(H, 1, 1, 3, 1), _out(W, 1, 1, 3, 1)
    flops = 2.0 * B * Ho * Wo * Co * C * 9
    e = _ESZ[cfg["dtype"]]
    nbytes = e * (B * C * H * W + Co * C * 9 + B * 18 * Ho * Wo + B * 9 * Ho * Wo +
                  B * Co * Ho * Wo + (Co if cfg.get("bias") else 0))
    return flops, nbytes


def msda_bytes(cfg, esz=4):
    B, M, C, Q, P = cfg["B"], cfg["M"], cfg["C"], cfg["Q"], cfg["P"]
    L = len(cfg["shapes"])
    S = sum(h * w for h, w in cfg["shapes"])
    return esz * (B * S * M * C + B * Q * M * L * P * 2 + B * Q * M * L * P + B * Q * M * C)


def cpu_info():
    """Host CPU model and logical core count (for the CPU baselines)."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"model": model, "logical_cores": os.cpu_count()}


class ClockSampler:
    """Polls SM clock and clock-event reasons through NVML in a thread."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, device_index: int, period_s: float = 0.0005):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        self._period = period_s
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report nothing rather than guess
            self._nv = None

    def _sample(self):
        nv = self._nv
        mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
        try:
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except AttributeError:
            bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
        self.samples.append(mhz)
        for bit, name in self.REASONS.items():
            if bits & bit:
                self.reasons.add(name)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                self._ready.set()
                return
            self._ready.set()
            time.sleep(self._period)

    def __enter__(self):
        if self._nv is not None:
            self._ready = threading.Event()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
            # the timed region starts only once the sampler is running, so a
            # region of a few milliseconds still gets several samples
            self._ready.wait(1.0)
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
            if not self.samples:
                self._sample()

    def summary(self):
        if self._nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        busy = [s for s in self.samples]
        return {"sm_mhz": statistics.median(busy) if busy else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons - {"gpu_idle"}),
                "samples": len(busy)}


# ----------------------------------------------------------------------------- data
def dcn_sets(cfg, n_sets, seed, img0, device):
    """n_sets independent input sets; camera b of a set is generated from
    (seed, global image index img0 + b) so any rank can regenerate its shard."""
    import torch
    from bevk.sharding import image_seed
    dt = getattr(torch, cfg["dtype"])
    B, C, H, W, Co = cfg["B"], cfg["C"], cfg["H"], cfg["W"], cfg["Cout"]
    sets = []
    for s in range(n_sets):
        g = torch.Generator(device=device)
        xs, offs, masks = [], [], []
        for b in range(B):
            g.manual_seed(image_seed(seed, img0 + b, s))
            xs.append(torch.randn(1, C, H, W, generator=g, device=device))
            off = torch.randn(1, 18, H, W, generator=g, device=device) * cfg.get("off_std", 2.0)
            if cfg["big"]:
                sel = torch.rand(off.shape, generator=g, device=device) < cfg["big"]
                sign = torch.where(torch.rand(off.shape, generator=g, device=device) < 0.5,
                                   -1.0, 1.0)
                off = torch.where(sel, sign * (H + 4), off)
            offs.append(off)
            masks.append(torch.sigmoid(torch.randn(1, 9, H, W, generator=g, device=device)))
        g.manual_seed(seed * 7919 + s)
        w = torch.randn(Co, C, 3, 3, generator=g, device=device) * math.sqrt(2.0 / (C * 9))
        bias = (torch.randn(Co, generator=g, device=device).to(dt) if cfg.get("bias")
                else None)
        fmt = (torch.contiguous_format if cfg.get("layout") == "nchw"
               else torch.channels_last)
        x = torch.cat(xs).to(dt).contiguous(memory_format=fmt)
        out = torch.empty(B, Co, H, W, dtype=dt, device=device, memory_format=fmt)
        sets.append(dict(x=x, off=torch.cat(offs).to(dt), mask=torch.cat(masks).to(dt),
                         w=w.to(dt), b=bias, out=out))
    return sets


def msda_sets(cfg, n_sets, seed, device, dtype=None):
    """n_sets independent MSDA input sets (value, locations, attention weights
    generated in fp32, then cast to ``dtype`` when given)."""
    import torch
    sets = []
    B, M, C, Q, P = cfg["B"], cfg["M"], cfg["C"], cfg["Q"], cfg["P"]
    shapes = cfg["shapes"]
    L = len(shapes)
    sizes = [h * w for h, w in shapes]
    lsi = [0]
    for s in sizes[:-1]:
        lsi.append(lsi[-1] + s)
    for s in range(n_sets):
        g = torch.Generator(device=device)
        g.manual_seed(seed * 31 + s)
        value = torch.randn(B, sum(sizes), M, C, generator=g, device=device)
        loc = torch.rand(B, Q, M, L, P, 2, generator=g, device=device)
        if cfg["oob"]:
            sel = torch.rand(B, Q, M, L, P, 1, generator=g, device=device) < cfg["oob"]
            loc = torch.where(sel, loc * 1.4 - 0.2, loc)
        attn = torch.softmax(torch.randn(B, Q, M, L * P, generator=g, device=device), -1)
        if dtype is not None:
            value, loc, attn = value.to(dtype), loc.to(dtype), attn.to(dtype)
        sets.append(dict(value=value, loc=loc, attn=attn.view(B, Q, M, L, P),
                         shapes=torch.tensor(shapes, dtype=torch.int64, device=device),
                         lsi=torch.tensor(lsi, dtype=torch.int64, device=device)))
    return sets


CHAIN_IMAGES = 48
CHAIN_DESC = ("5-chain: 48 images (8 samples x 6 cameras); per image one cfg5 MSDA camera "
              "slice (4 levels, Q=10000, 8x32, P=8, fp32) and one cfg3 DCN image (256 -> 256 "
              "ch, 58x100, bf16, 5% offsets at +-(H+4)); contiguous image blocks per rank")


def chain_inputs(img0, n, seed, device):
    """Inputs of global images [img0, img0 + n) of the 5-chain: per image a cfg5
    MSDA camera slice and a cfg3 DCN image, each generated from (seed, image
    index) alone, so a rank's block holds exactly the same images as the
    world-1 run (the DCN weight is shared, from the seed)."""
    import torch
    from bevk.sharding import image_seed
    m5 = MSDA_CFGS["cfg5"]
    M, C, Q, P = m5["M"], m5["C"], m5["Q"], m5["P"]
    shapes = m5["shapes"]
    L = len(shapes)
    sizes = [h * w for h, w in shapes]
    lsi = [0]
    for sz in sizes[:-1]:
        lsi.append(lsi[-1] + sz)
    values, locs, attns = [], [], []
    for img in range(img0, img0 + n):
        g = torch.Generator(device=device)
        g.manual_seed(image_seed(seed, img, 5))
        values.append(torch.randn(1, sum(sizes), M, C, generator=g, device=device))
        locs.append(torch.rand(1, Q, M, L, P, 2, generator=g, device=device))
        attns.append(torch.softmax(torch.randn(1, Q, M, L * P, generator=g, device=device), -1)
                     .view(1, Q, M, L, P))
    msda = dict(value=torch.cat(values), loc=torch.cat(locs), attn=torch.cat(attns),
                shapes=torch.tensor(shapes, dtype=torch.int64, device=device),
                lsi=torch.tensor(lsi, dtype=torch.int64, device=device))
    dcn = dcn_sets(dict(DCN_CFGS["cfg3"], B=n), 1, seed, img0, device)[0]
    return msda, dcn


def chain_step(msda, dcn):
    """One 5-chain step over a block of images: the MSDA call and the DCN call."""
    import _ms_deform_attn_ext as ext
    import modulated_deform_conv as mdc
    out = ext.forward(msda["value"], msda["shapes"], msda["lsi"], msda["loc"], msda["attn"], 64,
                      False)
    mdc.dcn_forward_into(dcn["x"], dcn["off"], dcn["mask"], dcn["w"], None, dcn["out"], 1, 1, 1)
    return out, dcn["out"]


def chain_checksums(msda_out, dcn_out):
    """Per-image fp64 sums of both outputs -> [images, 2]."""
    import torch
    n = msda_out.shape[0]
    if n == 0:
        return torch.zeros(0, 2, dtype=torch.float64, device=msda_out.device)
    return torch.stack([msda_out.double().reshape(n, -1).sum(1),
                        dcn_out.double().reshape(n, -1).sum(1)], 1)


def gather_rows(local, total, rank, world, dist):
    """Rows [b0, b1) of a [total, k] table held by each rank (its shard_range
    block) -> the whole table on every rank (an all_gather of equal-size,
    padded blocks; NCCL or gloo)."""
    import torch
    from bevk.sharding import shard_range
    if dist is None:
        return local
    width = max(shard_range(total, r, world)[1] - shard_range(total, r, world)[0]
                for r in range(world))
    pad = torch.full((width, local.shape[1]), float("nan"), dtype=local.dtype,
                     device=local.device)
    pad[:local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    rows = []
    for r in range(world):
        b0, b1 = shard_range(total, r, world)
        rows.append(parts[r][:b1 - b0])
    return torch.cat(rows)


def bench_chain(steps, warmup, device, seed, stream, rank, world, dist):
    """The 5-chain over the ranks: this rank's contiguous block of the 48 images
    (no collective on the data path), K steps captured in graphs and timed
    between events, max over ranks.  Outside the timed region, per-image output
    checksums are all-gathered and rank 0 regenerates and recomputes every
    rank's block (same block sizes, so the same kernels) and compares them."""
    import torch
    from bevk.sharding import shard_range
    b0, b1 = shard_range(CHAIN_IMAGES, rank, world)
    msda, dcn = chain_inputs(b0, b1 - b0, seed, device)
    torch.cuda.synchronize()            # generated on the default stream, used on `stream`
    ms = graph_time([lambda: chain_step(msda, dcn)], steps, warmup, stream, dist=dist)
    with torch.cuda.stream(stream):
        mine = chain_checksums(*chain_step(msda, dcn))
    torch.cuda.synchronize()
    del msda, dcn
    table = gather_rows(mine, CHAIN_IMAGES, rank, world, dist)
    verified = None
    if rank == 0:
        ok = bool(torch.isfinite(table).all())
        for r in range(world):
            r0, r1 = shard_range(CHAIN_IMAGES, r, world)
            if r1 == r0:
                continue
            m, d = chain_inputs(r0, r1 - r0, seed, device)
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                again = chain_checksums(*chain_step(m, d))
            torch.cuda.synchronize()
            ok = ok and torch.equal(again.cpu(), table[r0:r1].cpu())
            del m, d
        verified = ok
        torch.cuda.empty_cache()
    return dict(ms=ms, per_step_s=ms / 1e3 / steps, images_per_rank=b1 - b0,
                verified=verified)


def n_sets_for(set_bytes, lo=2, hi=16):
    return max(lo, min(hi, math.ceil(2 * L2_BYTES / max(set_bytes, 1))))


# ----------------------------------------------------------------------------- timing
def graph_time(step_fns, steps, warmup, stream, clocks=None, dist=None):
    """Warm up, capture `steps` launches (cycling step_fns) in CUDA graphs, replay them
    once between events; returns (elapsed_ms max over ranks, launches)."""
    import torch
    with torch.cuda.stream(stream):
        for i in range(warmup):
            step_fns[i % len(step_fns)]()
    torch.cuda.synchronize()
    chunk = min(steps, 1024)
    graphs = []
    done = 0
    while done < steps:
        n = min(chunk, steps - done)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                step_fns[(done + i) % len(step_fns)]()
        graphs.append(g)
        done += n
    # one untimed replay so graph upload is outside the timed region
    with torch.cuda.stream(stream):
        graphs[0].replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ctx = clocks if clocks is not None else _Null()
    with ctx:
        with torch.cuda.stream(stream):
            _cover_launch_gap(stream)
            start.record(stream)
            for g in graphs:
                g.replay()
            end.record(stream)
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = start.elapsed_time(end)
    del graphs
    return _max_over_ranks(ms, dist)


def _prime(step_fns, stream):
    """Run every input set's step once, untimed, so that per-weight caches
    (packed weight, BN fold, tap-major weight) are filled before capture:
    a set first used inside the captured graph would put its one-time weight
    transforms into every replay."""
    import torch
    with torch.cuda.stream(stream):
        for fn in step_fns:
            fn()
    torch.cuda.synchronize()


def _cover_launch_gap(stream):
    """Queue a ~2 ms spin kernel ahead of the start event, so the GPU is busy
    while the host submits the timed graphs / copies: the events then bracket
    only the device's work on the K steps, not the host's submission latency
    (which otherwise adds its own length / K to every step of a short run)."""
    import torch
    with torch.cuda.stream(stream):
        torch.cuda._sleep(4_000_000)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def _max_over_ranks(v, dist):
    if dist is None:
        return v
    import torch
    # NCCL reduces device tensors; gloo (CPU runs of the multi-rank logic) host ones
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- workloads
def bench_dcn(cfg_name, steps, warmup, device, seed, img0, stream, dist=None, clocks=None):
    import _modulated_deform_conv_ext as ext
    import modulated_deform_conv as mdc
    cfg = DCN_CFGS[cfg_name]
    flops, nbytes = dcn_work(cfg)
    n_sets = n_sets_for(nbytes)
    sets = dcn_sets(cfg, n_sets, seed, img0, device)
    for s in sets:
        s["wpk"] = mdc.packed_weight(s["w"])

    def make(s):
        return lambda: ext.dcn_forward(s["x"], s["off"], s["mask"], s["wpk"], s["b"], s["out"],
                                       3, 3, 1, 1, 1, 1, 1, 1, 1, 1, False)

    ms = graph_time([make(s) for s in sets], steps, warmup, stream, clocks, dist)
    per_launch_s = ms / 1e3 / steps
    return dict(ms=ms, flops=flops, bytes=nbytes, per_launch_s=per_launch_s, n_sets=n_sets,
                sets=sets)


def bench_dcn_pack(cfg_name, steps, warmup, device, seed, stream, fused):
    """The Pack module's forward as BEVFormer calls it (DCNSplitNHWCFunction:
    offset conv -> sigmoid mask -> DCN -> FrozenBN + ReLU), NHWC.  fused=False
    runs the offset conv on cuDNN (the reference's structure,
    dcn_split_nhwc.py:171-205); fused=True runs its channel reduction as one
    GEMM with fp32 output and the tap sum in this library's kernel.  Either
    way its output feeds the fused DCN kernel (sigmoid on load, BN folded,
    ReLU in the epilogue).  Offset-conv weights are scaled so that the
    offsets have a standard deviation of 2 px, as in the BASELINE configs."""
    import torch
    from modulated_deform_conv.dcn_split_nhwc import _forward_nhwc
    cfg = DCN_CFGS[cfg_name]
    dt = getattr(torch, cfg["dtype"])
    B, C, H, W, Co = cfg["B"], cfg["C"], cfg["H"], cfg["W"], cfg["Cout"]
    flops, nbytes = dcn_work(cfg)
    flops += 2 * B * H * W * 27 * C * 9
    sets = []
    for i in range(n_sets_for(nbytes)):
        g = torch.Generator(device=device)
        g.manual_seed(seed * 31 + i)
        x = torch.randn(B, H, W, C, generator=g, device=device).to(dt)
        w_off = (torch.randn(27, C, 3, 3, generator=g, device=device) *
                 (2.0 / math.sqrt(9 * C))).to(dt)
        b_off = torch.zeros(27, device=device, dtype=dt)
        w = (torch.randn(Co, C, 3, 3, generator=g, device=device) *
             math.sqrt(2.0 / (C * 9))).to(dt)
        scale = torch.rand(Co, generator=g, device=device) + 0.5
        shift = torch.randn(Co, generator=g, device=device) * 0.1
        sets.append((x, w_off, b_off, w, scale, shift))

    def make(s):
        x, w_off, b_off, w, scale, shift = s
        return lambda: _forward_nhwc(x, w_off, b_off, w, None, 1, 1, 1, scale, shift, True,
                                     gemm_offset=fused)

    fns = [make(s) for s in sets]
    _prime(fns, stream)
    ms = graph_time(fns, steps, warmup, stream)
    return dict(ms=ms, flops=flops, per_launch_s=ms / 1e3 / steps, n_sets=len(sets))


def bench_dcn_bwd(cfg_name, steps, warmup, device, seed, stream):
    """DCN backward as autograd runs it: dO . W^T (GEMM), the data side
    (bevk_dcn_backward_data: grad_input by a counting sort of the sample
    corners and a gather, grad_offset / grad_mask and the grad_weight columns
    from one pass over the samples) and [dO^T . col | ones] (GEMM) for
    grad_weight and grad_bias.  FLOPs counted: the two GEMMs (2 x the
    forward's 2*M*N*K)."""
    import torch
    import modulated_deform_conv as mdc
    cfg = DCN_CFGS[cfg_name]
    flops, nbytes = dcn_work(cfg)
    sets = dcn_sets(cfg, max(2, n_sets_for(3 * nbytes)), seed, 0, device)
    for i, s in enumerate(sets):
        g = torch.Generator(device=device)
        g.manual_seed(seed * 17 + i)
        s["gout"] = torch.randn(s["out"].shape, generator=g, device=device).to(
            s["out"].dtype).contiguous(memory_format=torch.channels_last)

    def make(s):
        return lambda: mdc.dcn_backward(s["x"], s["off"], s["mask"], s["w"], s["gout"],
                                        1, 1, 1)

    fns = [make(s) for s in sets]
    _prime(fns, stream)
    ms = graph_time(fns, steps, warmup, stream)
    return dict(ms=ms, flops=2 * flops, per_launch_s=ms / 1e3 / steps, n_sets=len(sets))


def e2e_time(host_in, run, steps, warmup, stream, clocks=None, dist=None):
    """Public-API end-to-end time of `steps` steps: every step copies its inputs
    (``host_in``, pinned host tensors) to the device, runs ``run(dev_inputs)``
    (the public call; it allocates and returns its output) and reads the output
    back into pinned host memory.  The steps are pipelined the way an
    inference loop runs them: the host->device copy of step k+1 and the
    device->host copy of step k-1 run on their own streams while step k
    computes (two buffer sets, ordered by events), so the per-step time is
    that of the slowest of the three, not their sum.
    Returns (ms max over ranks, h2d bytes per step, d2h bytes per step)."""
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    dev_in = [[torch.empty_like(h, device=dev) for h in host_in] for _ in range(2)]
    with torch.cuda.stream(stream):
        probe = run(dev_in[0])
    torch.cuda.synchronize()
    hout = [torch.empty(probe.shape, dtype=probe.dtype).pin_memory() for _ in range(2)]
    del probe
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = hout[0].numel() * hout[0].element_size()
    s_in, s_comp, s_out = torch.cuda.Stream(), stream, torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    ys = [None, None]   # step k's output stays referenced until step k+2 (read back by then)

    def step(k):
        i = k % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_comp[i])               # step k-2 has consumed buffer set i
            for d, h in zip(dev_in[i], host_in):
                d.copy_(h, non_blocking=True)
            ev_in[i].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_in[i])
            s_comp.wait_event(ev_out[i])              # step k-2's output has been read back
            ys[i] = run(dev_in[i])
            ev_comp[i].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[i])
            hout[i].copy_(ys[i], non_blocking=True)
            ev_out[i].record(s_out)

    for k in range(warmup):
        step(k)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ctx = clocks if clocks is not None else _Null()
    with ctx:
        _cover_launch_gap(s_in)
        start.record(s_in)
        for k in range(steps):
            step(k)
        end.record(s_out)                             # after the last read-back
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = _max_over_ranks(start.elapsed_time(end), dist)
    return ms, h2d, d2h


def bench_dcn_e2e(cfg_name, steps, warmup, sets, stream, clocks=None, dist=None):
    """DCN forward end to end through modulated_deform_conv2d (the reference
    Function's public call) with x / offset / mask from pinned host memory."""
    import modulated_deform_conv as mdc
    s0 = sets[0]
    host = [s0[k].cpu().pin_memory() for k in ("x", "off", "mask")]  # keeps x's strides
    w, b = s0["w"], s0["b"]
    return e2e_time(host, lambda d: mdc.modulated_deform_conv2d(d[0], d[1], d[2], w, b, 1, 1, 1),
                    steps, warmup, stream, clocks, dist)


def bench_msda_e2e(cfg_name, steps, warmup, device, seed, stream, dist=None):
    """MSDA forward end to end through MultiScaleDeformableAttnFunction.apply
    with value / locations / attention weights from pinned host memory (the
    level shapes and start indices are per-model constants kept on the device)."""
    import ms_deform_attn
    s0 = msda_sets(MSDA_CFGS[cfg_name], 1, seed, device)[0]
    host = [s0[k].cpu().pin_memory() for k in ("value", "loc", "attn")]
    shapes, lsi = s0["shapes"], s0["lsi"]
    del s0
    fn = ms_deform_attn.MultiScaleDeformableAttnFunction.apply
    return e2e_time(host, lambda d: fn(d[0], shapes, lsi, d[1], d[2], 64), steps, warmup,
                    stream, None, dist)


def bench_msda(cfg_name, steps, warmup, device, seed, stream, dtype=None):
    import torch
    import _ms_deform_attn_ext as ext
    cfg = MSDA_CFGS[cfg_name]
    nbytes = msda_bytes(cfg, 4 if dtype in (None, torch.float32) else 2)
    sets = msda_sets(cfg, n_sets_for(nbytes, lo=2, hi=4), seed, device, dtype)

    def make(s):
        return lambda: ext.forward(s["value"], s["shapes"], s["lsi"], s["loc"], s["attn"], 64,
                                   False)

    ms = graph_time([make(s) for s in sets], steps, warmup, stream)
    return dict(ms=ms, bytes=nbytes, per_launch_s=ms / 1e3 / steps, n_sets=len(sets))


def msda_bwd_bytes(cfg):
    """Algorithmic bytes of one MSDA backward: value, loc, attn and grad_out
    read once; grad_value, grad_loc and grad_attn written once."""
    B, M, C, Q, P = cfg["B"], cfg["M"], cfg["C"], cfg["Q"], cfg["P"]
    L = len(cfg["shapes"])
    S = sum(h * w for h, w in cfg["shapes"])
    return 4 * (2 * B * S * M * C + 2 * (B * Q * M * L * P * 3) + B * Q * M * C)


def bench_msda_bwd(cfg_name, steps, warmup, device, seed, stream):
    """The backward op as a caller pays for it: grad_value zeroed (the
    reference's wrapper allocates it with zeros_like) and the backward kernel."""
    import torch
    import _ms_deform_attn_ext as ext
    cfg = MSDA_CFGS[cfg_name]
    nbytes = msda_bwd_bytes(cfg)
    sets = msda_sets(cfg, n_sets_for(nbytes, lo=2, hi=4), seed, device)
    for i, s in enumerate(sets):
        g = torch.Generator(device=device)
        g.manual_seed(seed * 131 + i)
        B, Q, M, C = cfg["B"], cfg["Q"], cfg["M"], cfg["C"]
        s["gout"] = torch.randn(B, Q, M * C, generator=g, device=device)
        s["gv"] = torch.empty_like(s["value"])
        s["gl"] = torch.empty_like(s["loc"])
        s["ga"] = torch.empty_like(s["attn"])

    def make(s):
        def step():
            s["gv"].zero_()
            ext.backward(s["value"], s["shapes"], s["lsi"], s["loc"], s["attn"], s["gout"],
                         s["gv"], s["gl"], s["ga"], 64, False)
        return step

    ms = graph_time([make(s) for s in sets], steps, warmup, stream)
    return dict(ms=ms, bytes=nbytes, per_launch_s=ms / 1e3 / steps, n_sets=len(sets))


# ----------------------------------------------------------------------------- CPU legs
def _median_calls(fn, calls=5):
    """Median wall time of `calls` calls of fn(i) after one warm-up call."""
    fn(0)
    times = []
    for i in range(calls):
        t0 = time.perf_counter()
        fn(i)
        times.append(time.perf_counter() - t0)
    return statistics.median(times)


def cpu_dcn(cfg_name, target_s, seed):
    """The CPU oracle (oracle/bevk_oracle.c: the reference's DCN forward in fp32
    math, double accumulation) on all host threads over a bounded range of
    output pixels of the workload, median of 5 calls after a warm-up.
    Returns dict(us per full call, TFLOP/s, pixels per call, threads)."""
    import torch
    from oracle import oracle
    cfg = DCN_CFGS[cfg_name]
    s = dcn_sets(cfg, 1, seed, 0, torch.device("cpu"))[0]
    x = s["x"].float().contiguous().numpy()
    off, mask, w = (s[k].float().contiguous().numpy() for k in ("off", "mask", "w"))
    b = None if s["b"] is None else s["b"].float().numpy()
    B, C, H, W, Co = cfg["B"], cfg["C"], cfg["H"], cfg["W"], cfg["Cout"]
    M = B * H * W
    per_px = 2.0 * Co * C * 9
    probe = min(M, 256)
    t0 = time.perf_counter()
    oracle.dcn_forward(x, off, mask, w, b, 1, 1, 1, pix_range=(0, probe))
    t_px = max((time.perf_counter() - t0) / probe, 1e-8)
    npix = int(min(M, max(probe, target_s / t_px)))

    def call(i):
        lo = (i * npix) % max(1, M - npix + 1)
        oracle.dcn_forward(x, off, mask, w, b, 1, 1, 1, pix_range=(lo, lo + npix))

    t = _median_calls(call)
    return dict(us=t / npix * M * 1e6, tflops=per_px * npix / t / 1e12, npix=npix, M=M,
                threads=oracle.max_threads())


def cpu_msda(cfg_name, target_s, seed):
    """The CPU oracle's MSDA forward (the reference kernel's math,
    ms_deform_attn_kernels.cuh:559-623) on all host threads over a bounded range
    of (batch, query, head) units, median of 5 calls after a warm-up.
    Returns dict(us per full call, GB/s algorithmic, units per call, threads)."""
    import torch
    from oracle import oracle
    cfg = MSDA_CFGS[cfg_name]
    s = msda_sets(cfg, 1, seed, torch.device("cpu"))[0]
    args = [s[k].numpy() for k in ("value", "shapes", "lsi", "loc", "attn")]
    units = cfg["B"] * cfg["Q"] * cfg["M"]
    probe = min(units, 4096)
    t0 = time.perf_counter()
    oracle.msda_forward(*args, unit_range=(0, probe))
    t_u = max((time.perf_counter() - t0) / probe, 1e-9)
    n = int(min(units, max(probe, target_s / t_u)))

    def call(i):
        lo = (i * n) % max(1, units - n + 1)
        oracle.msda_forward(*args, unit_range=(lo, lo + n))

    t = _median_calls(call)
    full_s = t / n * units
    return dict(us=full_s * 1e6, gbps=msda_bytes(cfg) / full_s / 1e9, units=n, total=units,
                threads=oracle.max_threads())


def cpu_torch_golden(cfg_name, seed):
    """The reference's golden semantics on CPU through PyTorch, all host
    threads, median of 5 calls after a warm-up: DCN as
    torchvision.ops.deform_conv2d (bit-identical to the reference's golden,
    modulated_deform_conv.py:216-266 + mm, on fp32), MSDA as the grid_sample
    formulation (oracle/msda_grid_sample.py).  fp16/bf16 configs run in fp32
    on the up-cast inputs.  Returns us per call, or None when torchvision is
    missing."""
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    if cfg_name in DCN_CFGS:
        try:
            from torchvision.ops import deform_conv2d
        except ImportError:
            return None
        cfg = DCN_CFGS[cfg_name]
        st = dcn_sets(cfg, 1, seed, 0, torch.device("cpu"))[0]
        x, off, mask, w = (st[k].float().contiguous() for k in ("x", "off", "mask", "w"))
        b = None if st["b"] is None else st["b"].float()
        with torch.no_grad():
            t = _median_calls(lambda i: deform_conv2d(x, off, w, b, (1, 1), (1, 1), (1, 1), mask))
    else:
        from oracle.msda_grid_sample import msda_forward_grid_sample
        st = msda_sets(MSDA_CFGS[cfg_name], 1, seed, torch.device("cpu"))[0]
        with torch.no_grad():
            t = _median_calls(lambda i: msda_forward_grid_sample(st["value"], st["shapes"],
                                                                 st["loc"], st["attn"]))
    return t * 1e6


def headline_config(world):
    """The headline's `config` (shared by both arms, so the driver can compare
    them): BASELINE cfg2, weak-scaled over the ranks."""
    cfg = DCN_CFGS["cfg2"]
    _, nbytes = dcn_work(cfg)
    n_sets = n_sets_for(nbytes)
    return {"workload": cfg["desc"] + " (fp32 accumulate)", "global_batch": cfg["B"] * world,
            "parallelism": f"dp{world} (cameras sharded across ranks, no collective on the "
                           "data path)",
            "l2": f"inputs rotate over {n_sets} independent sets "
                  f"({n_sets * nbytes / 2**20:.0f} MiB > 126 MB L2)"}


def run_reference(args, world):
    """--impl reference: the reference algorithm (the oracle port of the DCN
    forward) on all host threads, same metric, unit and config as our arm; a
    step is a bounded sample of the cfg2 workload."""
    from oracle import oracle
    import torch
    cfg = DCN_CFGS["cfg2"]
    s = dcn_sets(cfg, 1, 2026, 0, torch.device("cpu"))[0]
    x = s["x"].float().contiguous().numpy()
    off, mask, w = (s[k].float().contiguous().numpy() for k in ("off", "mask", "w"))
    B, C, H, W, Co = cfg["B"], cfg["C"], cfg["H"], cfg["W"], cfg["Cout"]
    M = B * H * W
    per_px = 2.0 * Co * C * 9
    t0 = time.perf_counter()
    oracle.dcn_forward(x, off, mask, w, None, 1, 1, 1, pix_range=(0, 128))
    t_px = max((time.perf_counter() - t0) / 128, 1e-7)
    budget_s = 90.0
    npix = int(min(M, max(64, budget_s / (args.steps + args.warmup) / t_px)))
    for i in range(args.warmup):
        oracle.dcn_forward(x, off, mask, w, None, 1, 1, 1, pix_range=(0, npix))
    t0 = time.perf_counter()
    for i in range(args.steps):
        lo = (i * npix) % max(1, M - npix + 1)
        oracle.dcn_forward(x, off, mask, w, None, 1, 1, 1, pix_range=(lo, lo + npix))
    el = time.perf_counter() - t0
    value = per_px * npix * args.steps / el / 1e12
    threads = oracle.max_threads()
    cpu = cpu_info()
    sample = (f"{npix} of {M} output pixels of cfg2 per step (C oracle, fp32 math, "
              f"double accumulation, {threads} OpenMP threads on {cpu['model']})")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; BASELINE cfg2 "
        "shapes and distributions)",
        "config": headline_config(world),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _r(v, nd=3):
    """Round to `nd` significant digits for the compact per-config record."""
    if v is None:
        return None
    if v == 0:
        return 0.0
    return float(f"{v:.{nd}g}")


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--only", choices=("cfg1", "cfg2", "cfg3", "cfg4", "cfg5", "cfg4_f16",
                                       "cfg5_f16", "cfg4_bf16", "cfg5_bf16", "bwd_cfg2",
                                       "bwd_cfg3", "bwd_cfg4", "bwd_cfg5", "pack_cfg2",
                                       "pack_cfg3", "chain"),
                    help="time one workload's kernel only (profiling runs: no e2e, "
                         "legs, per-config record or CPU legs; prints a reduced line)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            run_reference(args, world)
        return

    import datetime
    import torch
    import torch.distributed as dist_mod
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                    device_id=device)
        dist = dist_mod
    stream = torch.cuda.Stream(device=device)
    peaks, peaks_src = _peaks()
    seed = 2026
    half = {"f16": torch.float16, "bf16": torch.bfloat16}

    if args.only:
        if args.only == "chain":
            r = bench_chain(args.steps, args.warmup, device, seed, stream, rank, world, dist)
            r["per_launch_s"] = r["per_step_s"]
            extra = {"images_per_s": CHAIN_IMAGES / r["per_step_s"], "verified": r["verified"],
                     "n_gpus": world}
        elif args.only in DCN_CFGS:
            r = bench_dcn(args.only, args.steps, args.warmup, device, seed, 0, stream, dist)
            del r["sets"]
            extra = {"tflops": r["flops"] / r["per_launch_s"] / 1e12}
        elif args.only.startswith("pack_"):
            r = bench_dcn_pack(args.only[5:], args.steps, args.warmup, device, seed, stream, True)
            r0 = bench_dcn_pack(args.only[5:], args.steps, args.warmup, device, seed, stream,
                                False)
            extra = {"tflops": r["flops"] / r["per_launch_s"] / 1e12,
                     "cudnn_offset_conv_us_per_call": r0["per_launch_s"] * 1e6}
        elif args.only in ("bwd_cfg2", "bwd_cfg3"):
            r = bench_dcn_bwd(args.only[4:], args.steps, args.warmup, device, seed, stream)
            extra = {"tflops": r["flops"] / r["per_launch_s"] / 1e12}
        elif args.only.startswith("bwd_"):
            r = bench_msda_bwd(args.only[4:], args.steps, args.warmup, device, seed, stream)
            extra = {"algorithmic_GBps": r["bytes"] / r["per_launch_s"] / 1e9}
        else:
            name, _, dt = args.only.partition("_")
            r = bench_msda(name, args.steps, args.warmup, device, seed, stream, half.get(dt))
            extra = {"algorithmic_GBps": r["bytes"] / r["per_launch_s"] / 1e9}
        if rank == 0:
            print(json.dumps({"profile_run": True, "workload": args.only,
                              "us_per_call": r["per_launch_s"] * 1e6, **extra}), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return

    # headline: cfg2 DCN, this rank's 6 cameras are global images [6*rank, 6*rank+6)
    clocks = ClockSampler(local_rank)
    cfg_name = "cfg2"
    cfg = DCN_CFGS[cfg_name]
    res = bench_dcn(cfg_name, args.steps, args.warmup, device, seed, cfg["B"] * rank, stream,
                    dist, clocks)
    flops, nbytes = res["flops"], res["bytes"]
    ms = res["ms"]
    value = world * flops * args.steps / (ms / 1e3) / 1e12
    achieved = flops / res["per_launch_s"] / 1e12
    roof = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
            "traffic": _traffic("dcn_fwd_tc cfg2"),
            "peak_source": f"{peaks_src} bf16_tflops (burst; kernel timed alone)",
            "algorithmic_bytes": nbytes}

    e2e_clocks = ClockSampler(local_rank)
    e2e_steps = min(args.steps, 200)
    e2e_ms, h2d, d2h = bench_dcn_e2e(cfg_name, e2e_steps, args.warmup, res["sets"], stream,
                                     e2e_clocks, dist)
    e2e_value = world * flops * e2e_steps / (e2e_ms / 1e3) / 1e12
    del res["sets"]
    torch.cuda.empty_cache()

    # compact per-config record, printed last on the line
    tens_peak, hbm = peaks["bf16_tflops"], peaks["hbm_gbs"]
    configs = {"cfg2": {"us": _r(res["per_launch_s"] * 1e6),
                        "frac": _r(achieved / tens_peak),
                        "e2e_us": _r(e2e_ms * 1e3 / e2e_steps)}}
    legs = {}
    k2 = min(args.steps, 500)
    ke = min(args.steps, 20)
    if not args.no_secondary:
        r1 = bench_dcn("cfg1", k2, args.warmup, device, seed + 1, 0, stream)
        e1 = bench_dcn_e2e("cfg1", ke, args.warmup, r1["sets"], stream)
        del r1["sets"]
        configs["cfg1"] = {"us": _r(r1["per_launch_s"] * 1e6), "frac": None,
                           "e2e_us": _r(e1[0] * 1e3 / ke)}
        r3 = bench_dcn("cfg3", k2, args.warmup, device, seed + 1, cfg["B"] * rank, stream)
        e3 = bench_dcn_e2e("cfg3", ke, args.warmup, r3["sets"], stream)
        del r3["sets"]
        configs["cfg3"] = {"us": _r(r3["per_launch_s"] * 1e6),
                           "frac": _r(r3["flops"] / r3["per_launch_s"] / 1e12 / tens_peak),
                           "e2e_us": _r(e3[0] * 1e3 / ke)}
        torch.cuda.empty_cache()
        for name in ("cfg4", "cfg5"):
            r = bench_msda(name, k2, args.warmup, device, seed + 2, stream)
            roof_us = r["bytes"] / (hbm * 1e9) * 1e6
            em = bench_msda_e2e(name, ke, args.warmup, device, seed + 2, stream)
            entry = {"us": _r(r["per_launch_s"] * 1e6),
                     "frac": _r(roof_us / (r["per_launch_s"] * 1e6)),
                     "e2e_us": _r(em[0] * 1e3 / ke)}
            torch.cuda.empty_cache()
            for tag, dt in half.items():
                rh = bench_msda(name, k2, args.warmup, device, seed + 2, stream, dt)
                entry[f"{tag}_us"] = _r(rh["per_launch_s"] * 1e6)
                entry[f"{tag}_frac"] = _r(rh["bytes"] / (hbm * 1e3) / (rh["per_launch_s"] * 1e6))
                torch.cuda.empty_cache()
            configs[name] = entry
        for name in ("cfg2", "cfg3"):
            r = bench_dcn_pack(name, min(k2, 200), args.warmup, device, seed + 5, stream, True)
            legs[f"pack{name[-1]}_us"] = _r(r["per_launch_s"] * 1e6)
            torch.cuda.empty_cache()
        for name in ("cfg2", "cfg3"):
            r = bench_dcn_bwd(name, min(k2, 100), args.warmup, device, seed + 4, stream)
            legs[f"dcn_bwd{name[-1]}_us"] = _r(r["per_launch_s"] * 1e6)
            torch.cuda.empty_cache()
        for name in ("cfg4", "cfg5"):
            r = bench_msda_bwd(name, min(k2, 200), args.warmup, device, seed + 3, stream)
            legs[f"msda_bwd{name[-1]}_us"] = _r(r["per_launch_s"] * 1e6)
            torch.cuda.empty_cache()
        rc = bench_chain(min(k2, 20), args.warmup, device, seed + 6, stream, rank, world, dist)
        legs["chain5_ms"] = _r(rc["per_step_s"] * 1e3)
        legs["chain5_img_s"] = _r(CHAIN_IMAGES / rc["per_step_s"])
        legs["chain5_ok"] = rc["verified"]
        torch.cuda.empty_cache()

    cpu = None
    cpu_host = cpu_info()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        c2 = cpu_dcn(cfg_name, 1.5, seed)
        cpu = {"value": c2["tflops"], "unit": "TFLOP/s", "cores": c2["threads"], "kind": "port",
               "sample": f"C oracle (oracle/bevk_oracle.c) on {c2['npix']} of {c2['M']} output "
                         f"pixels of cfg2 per call, median of 5 after a warm-up, fp32 math "
                         f"with double accumulation, {c2['threads']} threads on "
                         f"{cpu_host['model']}"}
        configs["cfg2"]["cpu_us"] = _r(c2["us"])
        configs["cfg2"]["cpu_torch_us"] = _r(cpu_torch_golden("cfg2", seed))
        if not args.no_secondary:
            for name in ("cfg1", "cfg3"):
                c = cpu_dcn(name, 1.5, seed)
                configs[name]["cpu_us"] = _r(c["us"])
                configs[name]["cpu_torch_us"] = _r(cpu_torch_golden(name, seed))
            for name in ("cfg4", "cfg5"):
                c = cpu_msda(name, 1.5, seed)
                configs[name]["cpu_us"] = _r(c["us"])
                configs[name]["cpu_torch_us"] = _r(cpu_torch_golden(name, seed))

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded; BASELINE cfg2 shapes and distributions)",
            "config": headline_config(world),
            "roofline": roof,
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "api": "modulated_deform_conv2d, pinned host in/out every step, copies "
                           "overlapped on two streams"},
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "cpu_host": cpu_host,
            "legs": legs,
            # per BASELINE config: device us/call, roofline fraction (tensor for
            # DCN, HBM for MSDA; of measured peaks), e2e us/step (pinned host
            # in/out), CPU us/call on all host threads -- the C oracle
            # (cpu_us) and the reference's golden semantics through PyTorch
            # (cpu_torch_us: torchvision deform_conv2d / grid_sample MSDA) --
            # and fp16/bf16 MSDA
            "configs": {k: configs[k] for k in sorted(configs)},
        }
        print(json.dumps(line, separators=(",", ":")), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
