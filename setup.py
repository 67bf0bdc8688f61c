"""Build script of the nano_train_b200 CUDA extension (sm_100a only).

    python setup.py build_ext --inplace

puts ``nano_train_b200/_C*.so`` next to the Python sources, so the built
library travels with the source tree.
"""
import glob
import os

# Use the system toolchain: a compiler wrapper whose private libstdc++.so
# symlink does not resolve makes the linker fall back to the static archive,
# and a second (static) libstdc++ inside the extension breaks iostreams.
for _var, _path in (("CC", "/usr/bin/gcc"), ("CXX", "/usr/bin/g++")):
    if os.path.exists(_path):
        os.environ[_var] = _path
os.environ.setdefault("CUDAHOSTCXX", os.environ.get("CXX", "g++"))

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode=arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
if os.environ.get("NTB_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")

sources = sorted(glob.glob(os.path.join("csrc", "*.cu")) + glob.glob(os.path.join("csrc", "*.cpp")))

setup(
    name="nano_train_b200",
    version="0.1.0",
    packages=find_packages(include=["nano_train_b200", "nano_train_b200.*", "src", "src.*"]),
    ext_modules=[
        CUDAExtension(
            name="nano_train_b200._C",
            sources=sources,
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
