"""Build script for the native parts of kapsl_sdk_b200.

Extensions (all built in-tree with ``python setup.py build_ext --inplace``):

* ``kapsl_sdk_b200._cuda``   sm_100a CUDA kernels (tcgen05 GEMM, paged attention,
  fused norm/RoPE/SwiGLU, sampler) with torch bindings.
* ``kapsl_sdk_b200._native`` C++ runtime: bincode wire codec, framing, block
  allocator / radix prefix index, SHM ring + allocators, UDS/TCP servers.
* ``kapsl_sdk.kapsl_sdk``     C++ client SDK (KapslClient, KapslShmClient,
  KapslHybridClient) sharing the wire codec with the server.

Only sm_100a code is generated (``-gencode arch=compute_100a,code=sm_100a``).
"""
import glob
import os

from setuptools import setup

ROOT = os.path.dirname(os.path.abspath(__file__))

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-gencode=arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("KAPSL_PTXAS_VERBOSE") else "-Xptxas=-O3",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-fvisibility=hidden"]


def _rel(paths):
    return sorted(os.path.relpath(p, ROOT) for p in paths)


def cuda_extension():
    from torch.utils.cpp_extension import CUDAExtension

    sources = _rel(glob.glob(os.path.join(ROOT, "csrc", "cuda", "*.cu")) +
                   glob.glob(os.path.join(ROOT, "csrc", "cuda", "*.cpp")))
    return CUDAExtension(
        name="kapsl_sdk_b200._cuda",
        sources=sources,
        include_dirs=[os.path.join(ROOT, "csrc", "cuda")],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    )


def native_extensions():
    from pybind11.setup_helpers import Pybind11Extension

    exts = []
    # selftest.cpp is a standalone program (sanitizer builds), not part of the module
    native_src = [s for s in _rel(glob.glob(os.path.join(ROOT, "csrc", "native", "*.cpp")))
                  if os.path.basename(s) != "selftest.cpp"]
    if native_src:
        # The CPU kernels use OpenMP from PyTorch's own libgomp, so one worker team serves
        # both torch's GEMMs and these kernels (a second thread pool would compete for the
        # cores and make libgomp throttle its spinning).
        import torch

        torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
        exts.append(Pybind11Extension(
            "kapsl_sdk_b200._native",
            native_src,
            include_dirs=[os.path.join(ROOT, "csrc", "native")],
            extra_compile_args=CXX_FLAGS + ["-pthread", "-fopenmp", "-mavx2", "-mfma"],
            extra_link_args=["-pthread", "-lrt", f"-L{torch_lib}", "-l:libgomp.so.1", f"-Wl,-rpath,{torch_lib}"],
            cxx_std=17,
        ))
    sdk_src = _rel(glob.glob(os.path.join(ROOT, "csrc", "sdk", "*.cpp")))
    if sdk_src:
        wire = [s for s in native_src if os.path.basename(s) in ("wire.cpp", "shm.cpp")]  # the SDK needs no CPU kernels
        exts.append(Pybind11Extension(
            "kapsl_sdk.kapsl_sdk",
            sdk_src + wire,
            include_dirs=[os.path.join(ROOT, "csrc", "native"), os.path.join(ROOT, "csrc", "sdk")],
            extra_compile_args=CXX_FLAGS + ["-pthread"],
            extra_link_args=["-pthread", "-lrt"],
            cxx_std=17,
        ))
    return exts


def main():
    from torch.utils.cpp_extension import BuildExtension

    which = os.environ.get("KAPSL_BUILD", "all")
    ext_modules = []
    if which in ("all", "cuda"):
        ext_modules.append(cuda_extension())
    if which in ("all", "native"):
        ext_modules.extend(native_extensions())
    setup(
        name="kapsl_sdk_b200",
        version="0.1.0",
        packages=["kapsl_sdk_b200", "kapsl_sdk"],
        ext_modules=ext_modules,
        cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    )


if __name__ == "__main__":
    main()
