"""Builds the two native extensions in-tree:

  rusteeze_b200._host  C++ host runtime (block manager, batch builder,
                       staging pool, shared-memory ring, NUMA helpers)
  rusteeze_b200._C     sm_100a CUDA kernels + their torch bindings

    python setup.py build_ext --inplace

The CUDA extension is compiled for sm_100a only (`-gencode
arch=compute_100a,code=sm_100a`); nvcc cross-compiles it without a GPU.
"""
import glob
import os
import sys

from setuptools import setup, Extension

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "rusteeze_b200")


def host_ext():
    import pybind11
    srcs = sorted(glob.glob(os.path.join(PKG, "csrc", "host", "*.cpp")))
    return Extension(
        "rusteeze_b200._host",
        [os.path.relpath(s, ROOT) for s in srcs],
        include_dirs=[pybind11.get_include()],
        language="c++",
        extra_compile_args=["-O3", "-std=c++17", "-fvisibility=hidden", "-Wall", "-Wno-sign-compare"],
    )


NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr", "--expt-extended-lambda",
    "-Xptxas", "-v",
    "-DNDEBUG",
]


def cuda_ext():
    from torch.utils.cpp_extension import CUDAExtension
    srcs = sorted(glob.glob(os.path.join(PKG, "csrc", "kernels", "*.cu")))
    srcs += sorted(glob.glob(os.path.join(PKG, "csrc", "kernels", "*.cpp")))
    return CUDAExtension(
        "rusteeze_b200._C",
        [os.path.relpath(s, ROOT) for s in srcs],
        include_dirs=[os.path.join(PKG, "csrc", "kernels")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        libraries=["cuda"],
        library_dirs=["/usr/local/cuda/lib64/stubs"],
    )


def main():
    exts = [host_ext()]
    cmdclass = {}
    if os.environ.get("RUSTEEZE_SKIP_CUDA", "0") != "1":
        from torch.utils.cpp_extension import BuildExtension
        exts.append(cuda_ext())
        cmdclass["build_ext"] = BuildExtension.with_options(use_ninja=True)
    setup(
        name="rusteeze_b200",
        version="0.1.0",
        packages=["rusteeze_b200"],
        ext_modules=exts,
        cmdclass=cmdclass,
        entry_points={"console_scripts": ["rusteeze=rusteeze_b200.cli.main:main"]},
    )


if __name__ == "__main__":
    main()
