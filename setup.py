"""Build the sm_100a (B200) CUDA extension of kvserve_b200 in-tree.

    python setup.py build_ext --inplace

produces ``kvserve_b200/_C.*.so``.  Every kernel is compiled for
``sm_100a`` only (tcgen05 / TMA / TMEM need the arch-specific target).
"""
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")

SOURCES = [
    "bindings.cpp",
    "kv_codec.cu",
    "bitpack.cu",
    "codebook.cu",
    "lossless.cu",
    "engine_ops.cu",
    "gemm_sm100.cu",
    "gemv.cu",
    "decode_fused.cu",
    "attention_prefill_sm100.cu",
    "attention_decode.cu",
    "paged_decode_noalloc.cu",
    "p2p.cu",
]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("KVS_PTXAS_VERBOSE") else "-O3",
    "-DNDEBUG",
]
if os.environ.get("KVS_CHECK"):
    NVCC_FLAGS.append("-DKVS_CHECK=1")

setup(
    name="kvserve_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="kvserve_b200._C",
            sources=[os.path.join("csrc", s) for s in SOURCES],
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
