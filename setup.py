"""Build of the sm_100a extension, in-tree: ``python setup.py build_ext --inplace``.

Every CUDA source is compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``); torch's own arch list is
bypassed by passing the gencode flag explicitly and clearing TORCH_CUDA_ARCH_LIST.
"""
import glob
import os

from setuptools import setup

os.environ["TORCH_CUDA_ARCH_LIST"] = ""          # no arch from torch's list: only the gencode below
from torch.utils.cpp_extension import BuildExtension, CUDAExtension  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("faster_yoco_b200", "csrc")

NVCC = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr", "-Xptxas", "-v" if os.environ.get("FYB_PTXAS_V") else "-O3",
    "-DNDEBUG",
]
if os.environ.get("FYB_BOUNDS_CHECK"):
    NVCC.append("-DFYB_BOUNDS_CHECK=1")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))

setup(
    name="faster_yoco_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="faster_yoco_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
