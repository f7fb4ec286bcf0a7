"""Build the two in-tree native extensions.

* ``vllm_suffix_hybrid_b200._native`` -- the C++ proposer core (CPU only).
* ``vllm_suffix_hybrid_b200._C``      -- the sm_100a CUDA kernels and the
  comm runtime, compiled for Blackwell data-center GPUs only.

``python setup.py build_ext --inplace`` builds both next to the sources so the
shared objects travel with the source tree.  ``SKIP_CUDA=1`` builds only the
proposer core.
"""
import glob
import os

from setuptools import setup

ROOT = os.path.dirname(os.path.abspath(__file__))


def native_ext():
    from pybind11.setup_helpers import Pybind11Extension

    srcs = sorted(glob.glob(os.path.join("csrc", "proposer", "*.cc")))
    return Pybind11Extension(
        "vllm_suffix_hybrid_b200._native",
        srcs,
        cxx_std=20,
        extra_compile_args=["-O3", "-fno-plt", "-Wall", "-Wno-sign-compare"],
    )


def cuda_ext():
    from torch.utils.cpp_extension import CUDAExtension

    srcs = sorted(glob.glob(os.path.join("csrc", "kernels", "*.cu"))) + sorted(
        glob.glob(os.path.join("csrc", "kernels", "*.cpp"))
    )
    nvcc = [
        "-O3",
        "-std=c++17",
        "-gencode",
        "arch=compute_100a,code=sm_100a",
        "-lineinfo",
        "--expt-relaxed-constexpr",
        "--use_fast_math",
        "-DNDEBUG",
        "-U__CUDA_NO_HALF_OPERATORS__",
        "-U__CUDA_NO_HALF_CONVERSIONS__",
        "-U__CUDA_NO_BFLOAT16_OPERATORS__",
        "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
        "-U__CUDA_NO_BFLOAT162_OPERATORS__",
        "-U__CUDA_NO_BFLOAT162_CONVERSIONS__",
        "-Xptxas=-warn-spills",
    ]
    return CUDAExtension(
        "vllm_suffix_hybrid_b200._C",
        srcs,
        include_dirs=[os.path.join(ROOT, "csrc", "kernels")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc},
        # No -lcuda: driver entry points are fetched through the runtime
        # (cudaGetDriverEntryPointByVersion), so the module imports on a
        # machine without a GPU driver (the build check).
    )


def use_system_compiler():
    """Compile with the system GCC when the environment points CC/CXX at a wrapper toolchain.

    The /opt/gcc wrapper of this image (a relocated copy of GCC 13 with its own
    assembler) produces objects in which a C++ exception carrying a formatted
    message (TORCH_CHECK(cond, "...", value)) crashes during unwinding; the
    system GCC 13 (/usr/bin) does not.  Set SH_KEEP_CXX=1 to keep CC/CXX.
    """
    if os.environ.get("SH_KEEP_CXX") == "1":
        return
    for var, path in (("CC", "/usr/bin/gcc"), ("CXX", "/usr/bin/g++")):
        if os.path.exists(path) and os.environ.get(var, "").startswith("/opt/gcc"):
            os.environ[var] = path


def main():
    use_system_compiler()
    exts = [native_ext()]
    cmdclass = {}
    if os.environ.get("SKIP_CUDA", "0") != "1":
        from torch.utils.cpp_extension import BuildExtension

        exts.append(cuda_ext())
        cmdclass["build_ext"] = BuildExtension.with_options(use_ninja=True)
    setup(
        name="vllm_suffix_hybrid_b200",
        version="0.3.0",
        packages=["vllm_suffix_hybrid_b200"],
        ext_modules=exts,
        cmdclass=cmdclass,
    )


if __name__ == "__main__":
    main()
