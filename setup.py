"""Builds the native library vllm_moet_b200/_C (sm_100a CUDA kernels + C++ runtime).

    python setup.py build_ext --inplace

Every .cu file is compiled for sm_100a only (tcgen05 / TMA need the 'a'
target); nvcc cross-compiles without a GPU.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))


def _fingerprint():
    import importlib.util
    spec = importlib.util.spec_from_file_location("fp", os.path.join(ROOT, "vllm_moet_b200", "ops", "fingerprint.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m.source_fingerprint(ROOT)


FP = _fingerprint()
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

sources = sorted(glob.glob(os.path.join("csrc", "*.cpp")) + glob.glob(os.path.join("csrc", "kernels", "*.cu"))
                 + glob.glob(os.path.join("csrc", "runtime", "*.cpp")))

setup(
    name="vllm_moet_b200",
    version="0.1.0",
    packages=["vllm_moet_b200"],
    ext_modules=[
        CUDAExtension(
            name="vllm_moet_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, "csrc"), os.path.join(ROOT, "csrc", "kernels")],
            extra_compile_args={
                "cxx": ["-O3", "-std=c++17", f'-DMOET_SOURCE_FINGERPRINT="{FP}"'],
                "nvcc": ARCH + ["-O3", "-std=c++17", "-lineinfo", "--use_fast_math",
                                "-Xptxas", "-warn-spills",
                                "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__"],
            },
            libraries=["cuda"],
        ),
        # test-only kernels (tests/csrc), a separate module the product never loads
        CUDAExtension(
            name="tests.moet_testkit",
            sources=sorted(glob.glob(os.path.join("tests", "csrc", "*.cpp")) +
                           glob.glob(os.path.join("tests", "csrc", "*.cu"))),
            include_dirs=[os.path.join(ROOT, "csrc"), os.path.join(ROOT, "csrc", "kernels")],
            extra_compile_args={
                "cxx": ["-O3", "-std=c++17"],
                "nvcc": ARCH + ["-O3", "-std=c++17", "-lineinfo",
                                "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__"],
            },
            libraries=["cuda"],
        ),
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
