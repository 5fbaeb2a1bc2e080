"""Build the LunaFlux native extensions in-tree.

    python setup.py build_ext --inplace

* ``lunaflux_b200._C``    hand-written sm_100a CUDA kernels (tcgen05/TMA/mma).
* ``lunaflux_b200._host`` C++ host runtime: page allocator, block tables,
  radix prefix tree, BPE encoder, process channel, approved filesystem.

Only sm_100a (B200) code is generated.
"""
import os

from setuptools import setup

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")

cuda_sources = [
    "csrc/bindings.cpp",
    "csrc/kernels/runtime.cu",
    "csrc/kernels/gemm_bf16.cu",
    "csrc/kernels/elementwise.cu",
    "csrc/kernels/attention.cu",
]
cuda_sources += [os.path.join("csrc/kernels", f) for f in sorted(os.listdir(os.path.join(CSRC, "kernels")))
                 if f.endswith(".cu") and os.path.join("csrc/kernels", f) not in cuda_sources]
cuda_sources += [os.path.join("csrc/runtime", f) for f in sorted(os.listdir(os.path.join(CSRC, "runtime")))
                 if f.endswith(".cpp")] if os.path.isdir(os.path.join(CSRC, "runtime")) else []

_host_dir = os.path.join(CSRC, "host")
host_sources = sorted(os.path.join("csrc/host", f) for f in os.listdir(_host_dir)
                      if f.endswith(".cpp")) if os.path.isdir(_host_dir) else []

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("LF_PTXAS_VERBOSE") else "-O3",
]

ext_modules = [
    CUDAExtension(
        name="lunaflux_b200._C",
        sources=cuda_sources,
        include_dirs=[CSRC],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    ),
]
if host_sources:
    import pybind11
    from setuptools import Extension
    # plain pybind11 module: no torch linkage, importable on any host
    ext_modules.append(
        Extension(
            name="lunaflux_b200._host",
            sources=host_sources,
            include_dirs=[CSRC, pybind11.get_include()],
            extra_compile_args=["-O3", "-std=c++20", "-fvisibility=hidden"],
            language="c++",
        ))

setup(
    name="lunaflux_b200",
    version="0.1.0",
    packages=["lunaflux_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
