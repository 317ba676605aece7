"""Builds the torch extensions in place (invoked by build.py):

    python setup.py build_ext --inplace

Both are plain C++ over libbevk.so (the C ABI in include/bevk.h); they hold
no CUDA kernels of their own and are linked with an $ORIGIN rpath so the
library is found next to them.
"""
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
INCLUDE = os.path.join(os.path.dirname(HERE), "include")


def ext(name, src):
    return CUDAExtension(
        name,
        sources=[os.path.join("csrc", src)],
        include_dirs=[INCLUDE, os.path.join(HERE, "csrc")],
        library_dirs=[HERE],
        libraries=["bevk"],
        extra_compile_args={"cxx": ["-O2", "-std=c++17"]},
        extra_link_args=["-Wl,-rpath,$ORIGIN"],
    )


setup(
    name="bev_kernels_b200_ext",
    ext_modules=[
        ext("_modulated_deform_conv_ext", "torch_ext_dcn.cpp"),
        ext("_ms_deform_attn_ext", "torch_ext_msda.cpp"),
    ],
    cmdclass={"build_ext": BuildExtension},
)
