"""Builds the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

Produces ``priml_b200/ops/_C*.so`` (CUDA kernels) and ``priml_b200/data/_native*.so``
(host-side tokenizer and packer). Every CUDA source is compiled for
``compute_100a`` / ``sm_100a`` only (no PTX for other targets).
"""

from pathlib import Path

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "priml_b200" / "ops" / "csrc"

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-diag-suppress=177",
]

ext = CUDAExtension(
    name="priml_b200.ops._C",
    sources=sorted(str(p.relative_to(ROOT)) for p in CSRC.glob("*.cu")) + [str((CSRC / "bindings.cpp").relative_to(ROOT))],
    include_dirs=[str(CSRC)],
    extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
)

# Host-side data runtime (byte-level BPE, row packer): plain C++, no CUDA.
data_ext = CppExtension(
    name="priml_b200.data._native",
    sources=["priml_b200/data/csrc/bpe.cpp"],
    extra_compile_args=["-O3", "-std=c++17", "-pthread"],
    extra_link_args=["-pthread"],
)

setup(
    name="priml_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[ext, data_ext],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
