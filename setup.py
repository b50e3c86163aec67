"""Build the appcorr_b200 native extension in-tree for sm_100a.

    python setup.py build_ext --inplace

produces appcorr_b200/_C*.so (CUDA kernels + pybind11 bindings) and, from csrc/runtime/,
appcorr_b200/_runtime*.so (host-side C++ runtime).
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension, CppExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CUDA_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-gencode=arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("APPCORR_PTXAS_VERBOSE") else "-Xptxas=-O3",
]
CXX_FLAGS = ["-O3", "-std=c++17"]

cuda_sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + ["csrc/bindings.cpp"]
runtime_sources = sorted(glob.glob(os.path.join("csrc", "runtime", "*.cpp")))

ext_modules = [
    CUDAExtension(
        name="appcorr_b200._C",
        sources=cuda_sources,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": CUDA_FLAGS},
        libraries=["cuda"],
        library_dirs=["/usr/local/cuda/lib64/stubs"],
    ),
]
if runtime_sources:
    # host-only runtime: plain pybind11, no torch libraries (importable without torch)
    import pybind11
    from setuptools import Extension

    ext_modules.append(
        Extension(
            name="appcorr_b200._runtime",
            sources=runtime_sources,
            include_dirs=[os.path.join(ROOT, "csrc", "runtime"), pybind11.get_include()],
            language="c++",
            extra_compile_args=CXX_FLAGS + ["-fvisibility=hidden"],
            extra_link_args=["-lrt"],
        )
    )

setup(
    name="appcorr_b200",
    version="0.1.0",
    packages=["appcorr_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
