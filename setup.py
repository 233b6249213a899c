"""Build the in-tree native extension ``synthefy_nori_b200._C`` for sm_100a only.

    python setup.py build_ext --inplace
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("synthefy_nori_b200", "csrc")

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
if os.environ.get("NORI_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

setup(
    name="synthefy_nori_b200",
    version="0.1.0",
    packages=[d.replace(os.sep, ".") for d, _, files in os.walk("synthefy_nori_b200") if "__init__.py" in files],
    package_data={"synthefy_nori_b200.configs": ["*.json"], "synthefy_nori_b200.evaluation.benchmark_lists": ["*.csv"]},
    entry_points={"console_scripts": [
        "synthefy-nori-b200-train = synthefy_nori_b200.training.cli:main",
        "synthefy-nori-b200-eval = synthefy_nori_b200.evaluation.cli:main",
        "synthefy-nori-b200-download = synthefy_nori_b200.hf:download_cli",
        "synthefy-nori-b200-upload = synthefy_nori_b200.hf:upload_cli",
        "synthefy-nori-b200-serve = synthefy_nori_b200.serving:main",
    ]},
    ext_modules=[
        CUDAExtension(
            name="synthefy_nori_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
