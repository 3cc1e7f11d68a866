"""Build the two in-tree native extensions of the package.

* ``_cpu``: host-only C++ runtime (CPU mailbox allreduce engine, FD exchange).
* ``_C``:   CUDA for sm_100a only (symmetric memory, allreduce kernels,
            tcgen05 GEMM, attention, elementwise ops, AWQ int4 GEMV/dequant).

Usage: ``python setup.py build_ext --inplace`` (``__graft_entry__.build`` does
this). The arch is passed explicitly as ``-gencode arch=compute_100a,
code=sm_100a``, which also stops torch from adding its own arch list.
"""
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

PKG = "3080_mod_p2p_sglang_patch_b200"
ROOT = os.path.dirname(os.path.abspath(__file__))


def src(*parts):
    return os.path.join("csrc", *parts)


NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
    "-Xptxas", "-warn-spills",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG"]

ext_modules = [
    CppExtension(
        name=f"{PKG}._cpu",
        sources=[src("cpu", "mailbox_cpu.cpp"), src("cpu", "fdx.cpp"), src("cpu", "bindings_cpu.cpp")],
        extra_compile_args={"cxx": CXX_FLAGS},
    ),
    CUDAExtension(
        name=f"{PKG}._C",
        sources=[
            src("bindings.cpp"),
            src("symm", "symm.cpp"),
            src("ar", "allreduce.cu"),
            src("ops", "elementwise.cu"),
            src("gemm", "gemm.cu"),
            src("gemm", "gemv.cu"),
            src("attn", "attention.cu"),
            src("attn", "decode_noalloc.cu"),
            src("attn", "fmha_tc.cu"),
            src("quant", "awq.cu"),
        ],
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    ),
]

setup(
    name="mailbox-ar-b200",
    version="0.1.0",
    packages=find_packages(include=[PKG, PKG + ".*", "mailbox_ar_b200"]),
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
