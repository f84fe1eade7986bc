"""Build the psrl_b200 CUDA extension in-tree for sm_100a.

    python setup.py build_ext --inplace

produces ``psrl_b200/_C*.so`` (kernels) next to the sources so that the
built library travels with the repository snapshot.
"""

import glob
import os

from setuptools import find_packages, setup
from pybind11.setup_helpers import Pybind11Extension
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "psrl_b200", "csrc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__",
]
if os.environ.get("PSRL_KERNEL_CHECKS"):
    NVCC_FLAGS.append("-DPSRL_KERNEL_CHECKS=1")
if os.environ.get("PSRL_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp"),
                                                          os.path.join(CSRC, "vmm.cpp"),
                                                          os.path.join(CSRC, "green.cpp")]

setup(
    name="psrl_b200",
    version="0.1.0",
    packages=find_packages(include=["psrl_b200", "psrl_b200.*"]),
    package_data={"psrl_b200": ["config/*.yaml", "config/presets/*.yaml"]},
    ext_modules=[
        CUDAExtension(
            name="psrl_b200._C",
            sources=[os.path.relpath(s, ROOT) for s in sources],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            # no libcuda link: driver-API calls are resolved at run time
            # (csrc/driver_api.h), so the module imports on driver-less hosts
        ),
        # host-only runtime pieces (plain pybind11, no CUDA or torch linkage):
        # they load on CPU-only machines too
        Pybind11Extension(
            "psrl_b200._router",
            [os.path.relpath(os.path.join(ROOT, "psrl_b200", "csrc_host", "router_core.cpp"), ROOT)],
            cxx_std=17,
            extra_compile_args=["-O3"],
        ),
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
