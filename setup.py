"""Build the in-tree sm_100a kernel library ``inference_systems_b200/_C``.

    python setup.py build_ext --inplace

Only ``sm_100a`` code is generated (``-gencode arch=compute_100a,code=sm_100a``);
the extension is placed next to the package sources so it travels with the
repository checkout.
"""

import os
from pathlib import Path

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

CSRC = Path("inference_systems_b200") / "csrc"
SOURCES = ["ops.cpp", "gemm.cu", "norm.cu", "gdn.cu", "gdn_chunk.cu", "attention.cu", "attention_tc.cu", "state.cu", "comm.cu"]

NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("ISB_PTXAS_VERBOSE") else "-O3",
]

setup(
    name="inference_systems_b200",
    version="0.1.0",
    packages=["inference_systems_b200"],
    ext_modules=[
        CUDAExtension(
            name="inference_systems_b200._C",
            sources=[str(CSRC / s) for s in SOURCES],
            include_dirs=[str(CSRC.resolve())],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(no_python_abi_suffix=True, use_ninja=True)},
)
