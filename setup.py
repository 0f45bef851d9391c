"""Builds the in-tree native extension ``thundersync_b200._C`` for sm_100a.

    python setup.py build_ext --inplace

Every CUDA source is compiled for ``compute_100a``/``sm_100a`` only (B200);
the explicit ``-gencode`` bypasses torch's own architecture list.
"""

import glob
import os
import subprocess

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
SOURCES = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + sorted(glob.glob(os.path.join("csrc", "*.cpp")))

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
CXX_FLAGS = ["-O3", "-std=c++17"]
if os.environ.get("TS_BOUNDS_CHECK"):
    # bounds-checked debug build: the TS_BOUND_DEBUG index checks (csrc/bounds.cuh) are compiled in
    NVCC_FLAGS.append("-DTS_BOUNDS_CHECK=1")
    CXX_FLAGS.append("-DTS_BOUNDS_CHECK=1")
if os.environ.get("TS_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")

HOST_TOOLS = {
    # host-side helper executables, built beside the package modules that run them
    os.path.join("thundersync_b200", "rollout", "ts_netguard"): os.path.join("csrc", "host", "netguard.c"),
}


class Build(BuildExtension.with_options(use_ninja=True)):
    def run(self):
        for out, src in HOST_TOOLS.items():
            subprocess.check_call(["gcc", "-O2", "-Wall", "-o", os.path.join(ROOT, out), os.path.join(ROOT, src)])
        super().run()


setup(
    name="thundersync_b200_native",
    ext_modules=[
        CUDAExtension(
            "thundersync_b200._C",
            SOURCES,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": Build},
)
