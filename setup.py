"""Build the native core of turbol_b200 in-tree.

    python setup.py build_ext --inplace
    TURBOL_CPU_ONLY=1 python setup.py build_ext --build-lib <dir>   # host core only

CPU-only build (TURBOL_CPU_ONLY=1): the host runtime (Tensor/Config/engines on
CPU tensors/profiler/writers/tokenizer/dataset/store/schedules/KV allocator and
the pybind11 module) compiled with the C++ compiler alone against torch's CPU
headers: no nvcc, no CUDA runtime, no kernels (the ``ops`` submodule is absent
and ``built_for()`` returns "cpu").  It is for machines without a GPU and for
CI; write it to its own --build-lib so it does not replace the CUDA build.

One extension, ``turbol_b200.turbol_core``, holds both the C++ host runtime
(Tensor/Config/engines/profiler/writers/bootstrap store/pybind11 bindings) and
the hand-written CUDA kernels.  Every ``.cu`` file is compiled for sm_100a only:
the ``-gencode`` flag below makes ``torch.utils.cpp_extension`` skip its own
arch list.  Kernel sources include no torch headers, so they compile in seconds;
only the binding/engine ``.cpp`` files pay for the torch headers.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs():
    """Headers and library of the NCCL that torch loads (the nvidia-nccl wheel
    next to torch), so the C++ communicators share torch's libnccl.so.2."""
    try:
        import nvidia.nccl  # namespace package: no __file__

        base = list(nvidia.nccl.__path__)[0]
    except ImportError:
        return None, None
    inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
    if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
        return inc, lib
    return None, None


NCCL_INC, NCCL_LIB = nccl_dirs()


def sources():
    pats = ["csrc/core/*.cpp", "csrc/engines/*.cpp", "csrc/bindings/*.cpp", "csrc/kernels/*.cu"]
    out = []
    for p in pats:
        out += sorted(glob.glob(os.path.join(ROOT, p)))
    return [os.path.relpath(s, ROOT) for s in out]


nvcc_flags = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("TURBOL_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DTURBOL_CUDA=1",
]
# -ffp-contract=off: host arithmetic that restates a device kernel (the linear
# environment, the Philox draws) rounds every product and sum like it.
# -fno-math-errno: no host code reads errno, and with it a square root in a
# loop keeps a scalar errno path that stops the loop from vectorizing (host
# Adam); results are unchanged.
cxx_flags = ["-O3", "-std=c++17", "-ffp-contract=off", "-fno-math-errno", "-DTURBOL_CUDA=1", "-Wno-unused-function"]

CPU_ONLY = os.environ.get("TURBOL_CPU_ONLY", "") not in ("", "0")


def cpu_sources():
    pats = ["csrc/core/*.cpp", "csrc/engines/*.cpp", "csrc/bindings/bindings.cpp", "csrc/cpu_only/*.cpp"]
    out = []
    for p in pats:
        out += sorted(glob.glob(os.path.join(ROOT, p)))
    # NVLink peer memory and the NCCL communicators: CUDA build only
    out = [s for s in out if os.path.basename(s) not in ("peer.cpp", "distributed.cpp")]
    return [os.path.relpath(s, ROOT) for s in out]


cpu_ext = CppExtension(
    name="turbol_b200.turbol_core",
    sources=cpu_sources(),
    include_dirs=[os.path.join(ROOT, "csrc/include"), os.path.join(ROOT, "csrc/kernels")],
    extra_compile_args=["-O3", "-std=c++17", "-ffp-contract=off", "-fno-math-errno", "-DTURBOL_CUDA=0",
                        "-Wno-unused-function",
                        "-Wno-unused-parameter"],
    extra_link_args=["-l:libstdc++.so.6"],
)

ext = cpu_ext if CPU_ONLY else CUDAExtension(
    name="turbol_b200.turbol_core",
    sources=sources(),
    include_dirs=[os.path.join(ROOT, "csrc/include"), os.path.join(ROOT, "csrc/kernels")] + ([NCCL_INC] if NCCL_INC else []),
    extra_compile_args={"cxx": cxx_flags, "nvcc": nvcc_flags},
    # Link the C++ runtime dynamically: a toolchain whose libstdc++.so link is
    # missing falls back to libstdc++.a, and a private static copy of the
    # iostream/locale machinery inside this library crashes on the first
    # number it formats (its facet ids differ from the process's libstdc++).
    # (an RPATH, not a RUNPATH, for NCCL's directory: a RUNPATH here would stop a
    # native program that links this library from resolving torch's libraries
    # through its own RPATH)
    extra_link_args=["-l:libstdc++.so.6"] + ([f"-L{NCCL_LIB}", "-l:libnccl.so.2", "-Wl,--disable-new-dtags",
                                              f"-Wl,-rpath,{NCCL_LIB}"] if NCCL_LIB else ["-lnccl"]),
)

setup(
    name="turbol_b200",
    version="0.1.0",
    packages=["turbol_b200", "turbol"],
    ext_modules=[ext],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
