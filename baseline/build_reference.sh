#!/usr/bin/env bash
# Builds the unmodified reference (DeRuiChen258/Turbol, turbol_vllm tree) with
# its own CMake for sm_100 and installs its Python package + benchmark binaries
# into baseline/_ref (git-ignored).  The reference ships no setup.py or
# pyproject.toml at its root, so a plain `pip install` of it cannot work;
# this runs the build the reference's own CMakeLists.txt defines, from a copy
# (the source tree is read-only).  Tests are off (GoogleTest is not installed)
# and NCCL is off (its NCCL build calls a function NCCL does not have).
# Its CMakeLists.txt pins libtorch's arch list to 12.0 (sm_120 only), so an
# sm_100 -gencode is added through CMAKE_CUDA_FLAGS (appended to, not replaced).
#
#   REF=<path to the reference checkout> baseline/build_reference.sh
set -euo pipefail
if [ -z "${REF:-}" ] || [ ! -d "$REF/turbol_vllm" ]; then
  echo "set REF to the reference checkout (the directory holding turbol_vllm/)" >&2
  exit 2
fi
HERE=$(cd "$(dirname "$0")" && pwd)
SRC=$(mktemp -d /tmp/ref_src.XXXX)
BLD=$(mktemp -d /tmp/ref_build.XXXX)
cp -r "$REF"/. "$SRC"/
chmod -R u+w "$SRC"
TORCH_DIR=$(python -c 'import torch,os;print(os.path.join(os.path.dirname(torch.__file__),"share/cmake/Torch"))')
PYBIND_DIR=$(python -c 'import pybind11;print(pybind11.get_cmake_dir())')
cmake -S "$SRC/turbol_vllm" -B "$BLD" -G Ninja -DCMAKE_BUILD_TYPE=Release -DCMAKE_CUDA_ARCHITECTURES=100 \
  -DTURBORL_ENABLE_TESTS=OFF -DTURBORL_ENABLE_PYTHON=ON -DTURBORL_USE_NCCL=OFF \
  -DCMAKE_CUDA_FLAGS="-gencode arch=compute_100,code=sm_100" \
  -DTorch_DIR="$TORCH_DIR" -Dpybind11_DIR="$PYBIND_DIR" -DPython_EXECUTABLE="$(which python)"
cmake --build "$BLD" -j "$(nproc)"
mkdir -p "$HERE/_ref/bin"
rm -rf "$HERE/_ref/turbol" "$HERE/_ref/examples"
cp -r "$SRC/turbol_vllm/python/turbol" "$HERE/_ref/"
cp -r "$SRC/turbol_vllm/examples" "$HERE/_ref/examples"
cp "$BLD"/benchmark_components "$BLD"/benchmark_tensor "$BLD"/benchmark_attention "$BLD"/turbol_example "$HERE/_ref/bin/"
# The reference's attention kernel is compiled into its library, but nothing it
# builds calls it (its benchmark_attention only prints sizes).  Its extern "C"
# launcher flash_attention_forward goes into a shared library of its own, from
# the unmodified source, so benchmarks/benchmark_attention.py can time it.
mkdir -p "$HERE/_ref/lib"
nvcc -O3 -std=c++17 -gencode arch=compute_100,code=sm_100 -shared -Xcompiler -fPIC \
  "$SRC/turbol_vllm/src/cuda/attention.cu" -o "$HERE/_ref/lib/libref_attention.so"
echo "reference installed in $HERE/_ref"
