"""Build the sm_100a extension in place: ``python setup.py build_ext --inplace``.

Produces ``libra_b200/_C*.so``.  Only ``sm_100a`` code is generated; torch's
own arch list is bypassed by passing ``-gencode`` explicitly.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("libra_b200", "ops", "csrc")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("LIBRA_PTXAS_VERBOSE") else "-O3",
    "-DNDEBUG",
]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"

setup(
    name="libra_b200",
    ext_modules=[
        CUDAExtension(
            name="libra_b200._C",
            sources=sources,
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
