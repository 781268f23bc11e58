"""Build the meshtrain_b200 CUDA extension in-tree for sm_100a.

    python setup.py build_ext --inplace      # -> meshtrain_b200/ops/_C*.so

Only Blackwell (sm_100a) code is generated; the arch flags are passed in
``extra_compile_args`` so torch's own arch list is bypassed.
"""

import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("meshtrain_b200", "ops", "csrc")

# Compiling the kernels needs no GPU; torch's arch autodetection would refuse
# without one, so state the architecture explicitly.
os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]

# Diagnostic builds: MT_ATTN_TRACE=1 compiles clock64() timestamps into the attention kernels.
if os.environ.get("MT_ATTN_TRACE") == "1":
    NVCC_FLAGS.append("-DMT_ATTN_TRACE")

SOURCES = [
    os.path.join(CSRC, f)
    for f in ("bindings.cpp", "gemm_tcgen05.cu", "norms.cu", "elementwise.cu", "cross_entropy.cu", "adam.cu",
              "attention.cu")
    if os.path.exists(os.path.join(HERE, CSRC, f))
]

EXTENSIONS = [
    CUDAExtension(
        name="meshtrain_b200.ops._C",
        sources=SOURCES,
        include_dirs=[os.path.join(HERE, CSRC)],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    )
]
# Debug-checks build: MT_DEBUG_CHECKS=1 also builds meshtrain_b200.ops._C_debug, whose kernels check
# the indices they read from data and the TMEM / TMA addresses they form, record failures in a
# check word (ops.read_checks()) and skip the access; selected at run time by MT_OPS_DEBUG=1.
if os.environ.get("MT_DEBUG_CHECKS") == "1":
    EXTENSIONS.append(CUDAExtension(
        name="meshtrain_b200.ops._C_debug",
        sources=SOURCES,
        include_dirs=[os.path.join(HERE, CSRC)],
        extra_compile_args={"cxx": ["-O3", "-std=c++17", "-DMT_DEBUG_CHECKS"],
                            "nvcc": NVCC_FLAGS + ["-DMT_DEBUG_CHECKS"]},
    ))

setup(
    name="meshtrain_b200",
    version="0.1.0",
    packages=find_packages(include=["meshtrain_b200", "meshtrain_b200.*"]),
    package_data={"meshtrain_b200": ["dashboard.html"]},
    ext_modules=EXTENSIONS,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": ["meshtrain-b200=meshtrain_b200.cli:main"]},
    python_requires=">=3.10",
)
