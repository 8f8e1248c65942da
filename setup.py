"""Build the rl_b200 native extension in-tree for sm_100a.

    python setup.py build_ext --inplace

produces ``rl_b200/_C*.so``.  Every CUDA source is compiled for
``arch=compute_100a,code=sm_100a`` only (B200); torch's own arch list is not used.
"""

import glob
import os

from setuptools import setup

from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
# Keep torch from adding its own -gencode list: the flags below are the only targets.
os.environ["TORCH_CUDA_ARCH_LIST"] = ""

CUDA_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_HALF2_OPERATORS__",
]

sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + ["csrc/bindings.cpp"]

# RL_B200_DEBUG_BOUNDS=1 builds the bounds-checked debug variant rl_b200._C_debug
# (data-dependent indices checked and reported instead of dereferenced); it is
# loaded instead of rl_b200._C when the same variable is set at run time.
DEBUG_BOUNDS = os.environ.get("RL_B200_DEBUG_BOUNDS", "0") == "1"
EXT_NAME = "rl_b200._C_debug" if DEBUG_BOUNDS else "rl_b200._C"
DEFINES = ["-DRLB_DEBUG_BOUNDS"] if DEBUG_BOUNDS else []

setup(
    name="rl_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name=EXT_NAME,
            sources=sources,
            include_dirs=[os.path.join(HERE, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"] + DEFINES, "nvcc": CUDA_FLAGS + DEFINES},
            libraries=["cuda"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    # the debug variant keeps its objects apart from the release build's
    options={"build_ext": {"build_temp": os.path.join("build", "debug_bounds")}} if DEBUG_BOUNDS else {},
)
