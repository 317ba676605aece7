"""Build the B200 kernels in-tree.

    python bev-kernels_b200/build.py            # libbevk.so + torch extensions

1. ``libbevk.so``: every ``csrc/*.cu`` compiled by nvcc for sm_100a only
   (``-gencode arch=compute_100a,code=sm_100a``), exporting the C ABI of
   ``include/bevk.h``.
2. The torch extensions ``_modulated_deform_conv_ext`` and ``_ms_deform_attn_ext``
   (thin C++ layers over the C ABI; no CUDA code of their own), built with
   ``setup.py build_ext --inplace`` next to this file.

Outputs stay inside this directory so they travel with the source tree.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libbevk.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_lib(verbose: bool = False, extra_flags=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    objs = []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if _stale(obj, [src, *headers]):
            cmd = [nvcc, *NVCC_FLAGS, *extra_flags, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if _stale(LIB, objs):
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", LIB]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def build_torch_ext(verbose: bool = False) -> None:
    srcs = glob.glob(os.path.join(CSRC, "torch_ext_*.cpp"))
    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    outs = [os.path.join(HERE, n + suffix) for n in ("_modulated_deform_conv_ext", "_ms_deform_attn_ext")]
    deps = srcs + [LIB, os.path.join(INCLUDE, "bevk.h"), os.path.join(HERE, "setup.py")]
    if not any(_stale(o, deps) for o in outs):
        return
    cmd = [sys.executable, "setup.py", "build_ext", "--inplace", "--build-temp", os.path.join(BUILD, "ext")]
    subprocess.run(cmd, check=True, cwd=HERE,
                   stdout=None if verbose else subprocess.DEVNULL)


def build(verbose: bool = False) -> None:
    build_lib(verbose)
    build_torch_ext(verbose)


if __name__ == "__main__":
    build(verbose="-q" not in sys.argv)
