"""Build the sm_100a kernel library in-tree: ``python setup.py build_ext --inplace``.

Produces ``graspo_b200/_C*.so``.  Only Blackwell datacenter parts (sm_100a)
are targeted; there is no fallback architecture.  ``GRASPO_KERNEL_CHECKS=1``
compiles in index checks (an out-of-table index sets the device error word
and is clamped instead of faulting); ``graspo_b200._C.kernel_checks()``
reports which build is loaded.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CHECKS = ["-DGRASPO_KERNEL_CHECKS"] if os.environ.get("GRASPO_KERNEL_CHECKS") == "1" else []

sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + [os.path.join("csrc", "bindings.cpp")]

setup(
    name="graspo_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="graspo_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={
                "cxx": ["-O3", "-std=c++17"] + CHECKS,
                "nvcc": ARCH + CHECKS + ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
                                "-Xptxas=-v" if os.environ.get("GRASPO_PTXAS_VERBOSE") else "-Xptxas=-O3"],
            },
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
