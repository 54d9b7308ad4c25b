"""Builds the sm_100a CUDA extension in-tree: ``python setup.py build_ext --inplace``.

The extension lands at ``air_rs/_C*.so`` so it travels with the source tree; the arch is
passed explicitly (``-gencode arch=compute_100a,code=sm_100a``), bypassing torch's arch list.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension, CppExtension

HERE = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    srcs = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + sorted(glob.glob(os.path.join("csrc", "*.cpp")))
    return [s for s in srcs if not os.path.basename(s).startswith("_")]


ext = CUDAExtension(
    name="air_rs._C",
    sources=sources(),
    include_dirs=[os.path.join(HERE, "csrc")],
    libraries=["dl"],        # libcufile is dlopen'ed at run time (GPUDirect Storage reads)
    extra_compile_args={
        "cxx": ["-O3", "-std=c++17"],
        "nvcc": ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
                 "-Xptxas=-v" if os.environ.get("AIR_PTXAS_V") else "-DAIR_QUIET"] + ARCH,
    },
)

host = CppExtension(
    name="air_rs._host",
    sources=sorted(glob.glob(os.path.join("csrc", "host", "*.cpp"))),
    extra_compile_args={"cxx": ["-O3", "-std=c++17"]},
)

setup(name="air_rs", version="0.1.0", packages=["air_rs"], ext_modules=[ext, host],
      cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)})
