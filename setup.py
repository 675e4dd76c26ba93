"""Build the native parts of nexar_b200 in-tree.

    python setup.py build_ext --inplace

Three extension modules:
  * nexar_b200._host  - C++17 host runtime (control plane, CPU collectives,
                        compression, cluster management). No CUDA, no torch.
  * nexar_b200._cuda  - CUDA runtime for sm_100a (symmetric heap, peer-memory
                        collectives, fused GEMM+collective kernels, model ops).
  * nexar_b200._nccl  - NCCL communicator (libnccl resolved at run time) for
                        device point-to-point and the NCCL comparator.

Device code is compiled for sm_100a only.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 8))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "--use_fast_math",
    "--expt-relaxed-constexpr", "-Xptxas", "-v", "-DNDEBUG",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG", "-fvisibility=hidden"]


def rel(paths):
    return sorted(os.path.relpath(p, ROOT) for p in paths)


# csrc/host/tests/ holds native test drivers (their own main): not part of the extension.
host_sources = rel(glob.glob(os.path.join(ROOT, "csrc", "host", "*.cc")))
cuda_sources = rel(glob.glob(os.path.join(ROOT, "csrc", "cuda", "*.cu"))
                   + glob.glob(os.path.join(ROOT, "csrc", "cuda", "*.cpp")))

ext_modules = []
if host_sources:
    ext_modules.append(CppExtension(
        "nexar_b200._host",
        host_sources,
        include_dirs=[os.path.join(ROOT, "csrc", "host")],
        extra_compile_args={"cxx": CXX_FLAGS + ["-pthread"]},
        extra_link_args=["-pthread"],
        libraries=["ssl", "crypto"],  # TLS 1.3 for host links (csrc/host/tls.cc)
    ))
ext_modules.append(CUDAExtension(
    "nexar_b200._cuda",
    cuda_sources,
    include_dirs=[os.path.join(ROOT, "csrc", "cuda")],
    extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
))

ext_modules.append(CUDAExtension(
    "nexar_b200._nccl",
    rel(glob.glob(os.path.join(ROOT, "csrc", "nccl", "*.cpp"))),
    extra_compile_args={"cxx": CXX_FLAGS},
    libraries=["dl"],
))

setup(
    name="nexar_b200",
    version="0.1.0",
    packages=["nexar_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
