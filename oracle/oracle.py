"""CPU oracle for the DCNv2 / MSDA forward path -- TEST INFRASTRUCTURE ONLY.

Thin ctypes wrapper over ``oracle/_build/liboracle.so`` (``bevk_oracle.c``, a
plain-C restatement of the reference's algorithms).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs
may import this module; the product package never does.

Parity status:
  * DCNv2 forward and backward: pinned against the reference's own PyTorch
    goldens through the fixtures in ``tests/golden`` (see
    ``tests/golden/make_golden.py``).
  * MSDA forward: pinned against the reference's own generic forward kernel
    (``csrc_musa/msda/ms_deform_attn_kernels.cuh:559-623`` with its bilinear
    helper :7-49) compiled for the host from the reference tree with the
    stand-ins in ``oracle/ref_shim`` (``reference_msda_forward``; built into
    ``oracle/_ref`` by ``make -C oracle ref``), and cross-checked against the
    independent grid_sample formulation in ``oracle/msda_grid_sample.py``.
  * MSDA backward: restated from :425-494 and :638-788 and pinned against the
    reference's own generic backward kernel (:1168-1271, block-cooperative)
    run on the host as one emulated block of C threads
    (``reference_msda_backward``, same ``oracle/_ref`` build), and checked
    against torch autograd of the grid_sample formulation.

All functions take and return numpy arrays (float32 compute; inputs of other
float dtypes are up-cast, which is how fp16/bf16 kernel outputs are checked).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)


def build() -> str:
    """Compile the oracle with its Makefile (gcc only; seconds)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        lib = ctypes.CDLL(_LIB_PATH)
        i, i64 = ctypes.c_int, ctypes.c_int64
        lib.oracle_max_threads.restype = i
        lib.oracle_dcn_columns.restype = i
        lib.oracle_dcn_columns.argtypes = [_f32p] * 3 + [i] * 13 + [_f32p, i]
        lib.oracle_dcn_forward.restype = i
        lib.oracle_dcn_forward.argtypes = [_f32p] * 5 + [i] * 15 + [_f32p, i64, i64, i]
        lib.oracle_msda_forward.restype = i
        lib.oracle_msda_forward.argtypes = (
            [_f32p, _i64p, _i64p, _f32p, _f32p] + [i] * 7 + [_f32p, i64, i64, i])
        lib.oracle_dcn_backward.restype = i
        lib.oracle_dcn_backward.argtypes = [_f32p] * 5 + [i] * 15 + [_f32p] * 5 + [i]
        lib.oracle_msda_backward.restype = i
        lib.oracle_msda_backward.argtypes = (
            [_f32p, _i64p, _i64p, _f32p, _f32p, _f32p] + [i] * 7 + [_f32p] * 3 + [i])
        _lib = lib
    return _lib


def max_threads() -> int:
    return int(_load().oracle_max_threads())


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _p(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def _pair(v):
    return (int(v[0]), int(v[1])) if isinstance(v, (tuple, list)) else (int(v), int(v))


def out_size(n, pad, dil, k, stride):
    return (n + 2 * pad - (dil * (k - 1) + 1)) // stride + 1


def dcn_columns(x, offset, mask, kernel_size, stride=1, padding=0, dilation=1,
                deform_groups=1, layout="nchw", nthreads=0):
    """Deformable columns of NCHW inputs.

    layout="nchw": the reference's [C*kH*kW, B*Ho*Wo] matrix
    (modulated_deform_conv.py:370, row c*T + t).
    layout="nhwc": the NHWC gather's [B*Ho*Wo, T*C] matrix, k = t*C + c
    (dcn_split_nhwc.py:21-45).
    """
    x, offset, mask = _f32(x), _f32(offset), _f32(mask)
    B, C, H, W = x.shape
    kH, kW = _pair(kernel_size)
    sh, sw = _pair(stride)
    ph, pw = _pair(padding)
    dh, dw = _pair(dilation)
    Ho, Wo = out_size(H, ph, dh, kH, sh), out_size(W, pw, dw, kW, sw)
    T = kH * kW
    col = np.empty((B * Ho * Wo, C * T), np.float32)
    rc = _load().oracle_dcn_columns(_p(x), _p(offset), _p(mask), B, C, H, W, kH, kW,
                                    sh, sw, ph, pw, dh, dw, int(deform_groups),
                                    _p(col), int(nthreads))
    if rc != 0:
        raise ValueError("oracle_dcn_columns: invalid arguments")
    if layout == "nchw":
        return np.ascontiguousarray(col.T)
    if layout == "nhwc":
        return np.ascontiguousarray(
            col.reshape(B * Ho * Wo, C, T).transpose(0, 2, 1).reshape(B * Ho * Wo, T * C))
    raise ValueError(layout)


def dcn_forward(x, offset, mask, weight, bias=None, stride=1, padding=0, dilation=1,
                groups=1, deform_groups=1, pix_range=None, nthreads=0):
    """DCNv2 forward on NCHW arrays -> NCHW float32 output
    (modulated_deform_conv.py:331-403 semantics, double accumulation)."""
    x, offset, mask, weight = _f32(x), _f32(offset), _f32(mask), _f32(weight)
    B, C, H, W = x.shape
    Cout, _, kH, kW = weight.shape
    sh, sw = _pair(stride)
    ph, pw = _pair(padding)
    dh, dw = _pair(dilation)
    Ho, Wo = out_size(H, ph, dh, kH, sh), out_size(W, pw, dw, kW, sw)
    out = np.zeros((B, Cout, Ho, Wo), np.float32)
    bptr = None
    if bias is not None:
        bias = _f32(bias)
        bptr = _p(bias)
    lo, hi = (0, -1) if pix_range is None else (int(pix_range[0]), int(pix_range[1]))
    rc = _load().oracle_dcn_forward(_p(x), _p(offset), _p(mask), _p(weight), bptr,
                                    B, C, H, W, Cout, kH, kW, sh, sw, ph, pw, dh, dw,
                                    int(groups), int(deform_groups), _p(out), lo, hi,
                                    int(nthreads))
    if rc != 0:
        raise ValueError("oracle_dcn_forward: invalid arguments")
    return out


def dcn_backward(x, offset, mask, weight, grad_out, stride=1, padding=0, dilation=1,
                 groups=1, deform_groups=1, with_bias=True, nthreads=0):
    """DCNv2 backward on NCHW arrays -> (grad_x, grad_offset, grad_mask,
    grad_weight, grad_bias or None), float32 (modulated_deform_conv.py:269-312
    / :405-499 semantics, double accumulation)."""
    x, offset, mask, weight = _f32(x), _f32(offset), _f32(mask), _f32(weight)
    go = _f32(grad_out)
    B, C, H, W = x.shape
    Cout, _, kH, kW = weight.shape
    sh, sw = _pair(stride)
    ph, pw = _pair(padding)
    dh, dw = _pair(dilation)
    gx = np.zeros(x.shape, np.float32)
    goff = np.zeros(offset.shape, np.float32)
    gm = np.zeros(mask.shape, np.float32)
    gw = np.zeros(weight.shape, np.float32)
    gb = np.zeros((Cout,), np.float32) if with_bias else None
    rc = _load().oracle_dcn_backward(_p(x), _p(offset), _p(mask), _p(weight), _p(go),
                                     B, C, H, W, Cout, kH, kW, sh, sw, ph, pw, dh, dw,
                                     int(groups), int(deform_groups), _p(gx), _p(goff), _p(gm),
                                     _p(gw), _p(gb) if gb is not None else None, int(nthreads))
    if rc != 0:
        raise ValueError("oracle_dcn_backward: invalid arguments")
    return gx, goff, gm, gw, gb


def msda_forward(value, spatial_shapes, level_start_index, sampling_loc, attn_weight,
                 unit_range=None, nthreads=0):
    """MSDA forward -> [B, Q, heads*C] float32
    (ms_deform_attn_kernels.cuh:559-623 semantics)."""
    value, loc, attn = _f32(value), _f32(sampling_loc), _f32(attn_weight)
    shapes = np.ascontiguousarray(np.asarray(spatial_shapes, dtype=np.int64))
    lsi = np.ascontiguousarray(np.asarray(level_start_index, dtype=np.int64))
    B, S, M, C = value.shape
    _, Q, _, L, P, _ = loc.shape
    out = np.zeros((B, Q, M * C), np.float32)
    lo, hi = (0, -1) if unit_range is None else (int(unit_range[0]), int(unit_range[1]))
    rc = _load().oracle_msda_forward(_p(value), shapes.ctypes.data_as(_i64p),
                                     lsi.ctypes.data_as(_i64p), _p(loc), _p(attn),
                                     B, S, M, C, L, Q, P, _p(out), lo, hi, int(nthreads))
    if rc != 0:
        raise ValueError("oracle_msda_forward: invalid arguments")
    return out


_REF_PATH = os.path.join(_HERE, "_ref", "libmsda_ref.so")


def reference_tree():
    """The reference checkout, if there is one: $BEVK_REFERENCE_DIR, else a
    directory named ``reference`` beside this repository; None otherwise."""
    cand = os.environ.get("BEVK_REFERENCE_DIR") or os.path.join(
        os.path.dirname(os.path.dirname(_HERE)), "reference")
    return cand if os.path.isdir(os.path.join(cand, "csrc_musa", "msda")) else None


def build_reference() -> bool:
    """Compile the reference's MSDA kernels for the host into oracle/_ref
    (`make -C oracle ref REF_DIR=...`) when the reference tree is present."""
    tree = reference_tree()
    if tree is not None:
        subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF_DIR={tree}"], check=False)
    return os.path.exists(_REF_PATH)


def reference_msda_available() -> bool:
    """Whether the reference's own MSDA kernel is built for the host
    (oracle/_ref); built here on demand when the reference tree is present."""
    return os.path.exists(_REF_PATH) or build_reference()


def reference_msda_forward(value, spatial_shapes, level_start_index, sampling_loc,
                           attn_weight):
    """The reference's generic MSDA forward kernel
    (csrc_musa/msda/ms_deform_attn_kernels.cuh:559-623) run on the host, fp32
    -> [B, Q, heads*C]; the pin for msda_forward."""
    lib = ctypes.CDLL(_REF_PATH)
    value, loc, attn = _f32(value), _f32(sampling_loc), _f32(attn_weight)
    shapes = np.ascontiguousarray(np.asarray(spatial_shapes, dtype=np.int64))
    lsi = np.ascontiguousarray(np.asarray(level_start_index, dtype=np.int64))
    B, S, M, C = value.shape
    _, Q, _, L, P, _ = loc.shape
    out = np.zeros((B, Q, M * C), np.float32)
    rc = lib.ref_msda_forward_f32(_p(value), shapes.ctypes.data_as(_i64p),
                                  lsi.ctypes.data_as(_i64p), _p(loc), _p(attn), B, S, M, C, L,
                                  Q, P, _p(out))
    if rc != 0:
        raise ValueError("ref_msda_forward_f32: problem too large")
    return out


def reference_msda_backward(value, spatial_shapes, level_start_index, sampling_loc,
                            attn_weight, grad_output):
    """The reference's generic MSDA backward kernel
    (csrc_musa/msda/ms_deform_attn_kernels.cuh:1168-1271 with :426-491, one
    block of C threads per (batch, query, head) as binding_musa.mu:266-282
    launches it) run on the host as one emulated block of C threads ->
    (grad_value, grad_loc, grad_attn) float32, grad_value from zero; the pin
    for msda_backward."""
    lib = ctypes.CDLL(_REF_PATH)
    value, loc, attn = _f32(value), _f32(sampling_loc), _f32(attn_weight)
    g = _f32(grad_output)
    shapes = np.ascontiguousarray(np.asarray(spatial_shapes, dtype=np.int64))
    lsi = np.ascontiguousarray(np.asarray(level_start_index, dtype=np.int64))
    B, S, M, C = value.shape
    _, Q, _, L, P, _ = loc.shape
    gv = np.zeros(value.shape, np.float32)
    gl = np.zeros(loc.shape, np.float32)
    ga = np.zeros(attn.shape, np.float32)
    rc = lib.ref_msda_backward_f32(_p(value), shapes.ctypes.data_as(_i64p),
                                   lsi.ctypes.data_as(_i64p), _p(loc), _p(attn), _p(g), B, S, M,
                                   C, L, Q, P, _p(gv), _p(gl), _p(ga))
    if rc != 0:
        raise ValueError("ref_msda_backward_f32: problem too large or channels > 1024")
    return gv, gl, ga


def msda_backward(value, spatial_shapes, level_start_index, sampling_loc, attn_weight,
                  grad_output, nthreads=0):
    """MSDA backward -> (grad_value [B,S,M,C], grad_loc [B,Q,M,L,P,2],
    grad_attn [B,Q,M,L,P]) float32, grad_value starting from zero
    (ms_deform_attn_kernels.cuh:425-494 / :638-788 semantics)."""
    value, loc, attn = _f32(value), _f32(sampling_loc), _f32(attn_weight)
    g = _f32(grad_output)
    shapes = np.ascontiguousarray(np.asarray(spatial_shapes, dtype=np.int64))
    lsi = np.ascontiguousarray(np.asarray(level_start_index, dtype=np.int64))
    B, S, M, C = value.shape
    _, Q, _, L, P, _ = loc.shape
    gv = np.zeros(value.shape, np.float32)
    gl = np.zeros(loc.shape, np.float32)
    ga = np.zeros(attn.shape, np.float32)
    rc = _load().oracle_msda_backward(_p(value), shapes.ctypes.data_as(_i64p),
                                      lsi.ctypes.data_as(_i64p), _p(loc), _p(attn), _p(g),
                                      B, S, M, C, L, Q, P, _p(gv), _p(gl), _p(ga),
                                      int(nthreads))
    if rc != 0:
        raise ValueError("oracle_msda_backward: invalid arguments")
    return gv, gl, ga


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (d if d > 0 else 1.0))


def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0
