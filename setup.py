"""Build the sm_100a CUDA extension of complexity_framework_b200 in place.

    python setup.py build_ext --inplace

Only Blackwell (sm_100a) code is generated; there is no other target.
"""
import os
from setuptools import setup, find_packages
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("complexity_framework_b200", "csrc")

SOURCES = [
    "bindings.cpp",
    "bind_elementwise.cpp",
    "gemm_tc.cu",
    "elementwise.cu",
    "flash_fwd.cu",
    "flash_bwd.cu",
    "paged_attn.cu",
    "dist_fused.cu",
    "noalloc.cu",
    "tp_fused.cu",
    "ep_fused.cu",
    "pack.cu",
    "moe_grouped.cu",
    "tp_decode.cu",
    "fsdp.cu",
]

# Link the shared system libstdc++ (the one libtorch uses).  The compiler wrapper
# in this image cannot open its own libstdc++.so and would silently fall back to
# libstdc++.a: a private static copy whose stream/locale state is never set up,
# so formatting any error message inside the extension would crash.
LINK_ARGS = ["-L/usr/lib/x86_64-linux-gnu", "-l:libstdc++.so.6"]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]

ext = CUDAExtension(
    name="complexity_framework_b200._C",
    sources=[os.path.join(CSRC, s) for s in SOURCES],
    include_dirs=[os.path.join(HERE, CSRC)],
    extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    libraries=["cuda"],
    extra_link_args=LINK_ARGS,
)

# host-side data IO (memory-mapped token shards, batch gather, packing)
io_ext = CppExtension(
    name="complexity_framework_b200._io",
    sources=[os.path.join(CSRC, "io", "token_io.cpp")],
    extra_compile_args={"cxx": ["-O3", "-std=c++17"]},
    extra_link_args=LINK_ARGS,
)

setup(
    name="complexity_framework_b200",
    version="0.1.0",
    packages=find_packages(include=["complexity_framework_b200*"]),
    ext_modules=[ext, io_ext],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": [
        "cfb=complexity_framework_b200.cli.app:main",
        "cf-plan-cluster=complexity_framework_b200.training.cluster_plan:main",
    ]},
)
