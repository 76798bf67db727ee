"""setuptools recipe for the torch extension decode_kernel._cuda only.

Invoked by build.py (``python setup.py build_ext --inplace``) after nvcc has
produced decode_kernel/libdk_b200.so; the extension is a thin C++ layer over
that library's C ABI and compiles no CUDA itself.
"""

from pathlib import Path

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = Path(__file__).resolve().parent
INCLUDE = HERE.parent / "include"

setup(
    name="decode_kernel_b200_ext",
    ext_modules=[
        CUDAExtension(
            name="decode_kernel._cuda",
            sources=["csrc/bindings.cpp"],
            include_dirs=[str(INCLUDE)],
            library_dirs=[str(HERE / "decode_kernel")],
            libraries=["dk_b200"],
            extra_compile_args={"cxx": ["-O2", "-g0"]},
            extra_link_args=["-Wl,-rpath,$ORIGIN"],
        )
    ],
    cmdclass={"build_ext": BuildExtension},
    packages=[],
)
