"""Builds the framework's native extensions in-tree.

    python setup.py build_ext --inplace

``rocket_b200._C``  sm_100a CUDA kernels (tcgen05 / TMA) + torch bindings
``rocket_b200._rt`` host runtime in C++ (page pool, radix prefix tree,
                    scheduler core, prefix store) + pybind11 bindings
"""
import glob
import os

import pybind11
from setuptools import Extension, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("rocket_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-warn-spills",
]
CXX_FLAGS = ["-O3", "-std=c++17"]
if os.environ.get("ROCKET_DEBUG_BOUNDS"):
    # debug build: data-dependent indices are range-checked in the kernels (kErrBounds)
    NVCC_FLAGS.append("-DRKT_DEBUG_BOUNDS")
# programmatic dependent launch: every hot kernel starts with griddepcontrol.wait /
# launch_dependents (both return at once in a launch without the PDL attribute), so the
# runtime switch (ops.set_pdl, ROCKET_PDL) alone decides whether launches overlap
NVCC_FLAGS.append("-DRKT_PDL")

cuda_sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]
rt_sources = sorted(glob.glob(os.path.join(CSRC, "runtime", "*.cc")))

ext_modules = [
    CUDAExtension(
        "rocket_b200._C",
        cuda_sources,
        include_dirs=[os.path.join(HERE, CSRC)],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    ),
]
if rt_sources:
    # plain pybind11 module: no torch linkage, imports without torch loaded
    ext_modules.append(Extension(
        "rocket_b200._rt",
        rt_sources,
        include_dirs=[os.path.join(HERE, CSRC, "runtime"), pybind11.get_include()],
        extra_compile_args=CXX_FLAGS + ["-fvisibility=hidden"],
        language="c++",
    ))

setup(
    name="rocket_b200",
    version="0.1.0",
    packages=["rocket_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
