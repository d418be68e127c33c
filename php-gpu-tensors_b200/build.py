"""In-tree build of libgemm_sm100.so (sm_100a) and of the CPU oracle.

    python php-gpu-tensors_b200/build.py            # library + oracle
    python php-gpu-tensors_b200/build.py --force    # rebuild everything

The library is the CUDA translation units csrc/gemm_sm100.cu (kernels and the
launcher ABI) and csrc/mgpu.cu (multi-GPU entry points, NCCL loaded at run
time) plus the C++ host layer host/tensor_matmul.cpp, compiled by
nvcc for compute_100a/sm_100a only, linked with the static CUDA runtime and an export
map so that only the C ABI of include/gemm_sm100.h is visible.  nvcc
cross-compiles without a GPU.  The oracle (test infrastructure) is built by
oracle/Makefile.
"""
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libgemm_sm100.so")
HOST = os.path.join(PKG, "host")
SOURCES = [os.path.join(CSRC, "gemm_sm100.cu"), os.path.join(CSRC, "mgpu.cu"),
           os.path.join(HOST, "tensor_matmul.cpp")]
EXPORTS = os.path.join(CSRC, "exports.map")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-Xptxas", "-v" if os.environ.get("PTG_PTXAS_VERBOSE") else "-O3",
]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _sources():
    return (glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
            glob.glob(os.path.join(CSRC, "*.h")) +
            glob.glob(os.path.join(HOST, "*.cpp")) +
            glob.glob(os.path.join(INCLUDE, "*.h")) + [EXPORTS, os.path.abspath(__file__)])


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_library(force=False, verbose=False):
    if not force and not _stale(LIB, _sources()):
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc_path()] + NVCC_FLAGS + [
        "-shared", "-I", INCLUDE, "-I", CSRC,
        "-Xlinker", "--version-script=" + EXPORTS,
        "-o", tmp,
    ] + SOURCES + ["-ldl"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def reference_src():
    """src/ of the reference tree used to build oracle/_ref: PTG_REFERENCE_ROOT
    when set, else a `reference` directory beside the repository; None when
    neither exists (e.g. on a GPU box, which uses the prebuilt files)."""
    root = os.environ.get("PTG_REFERENCE_ROOT") or os.path.join(os.path.dirname(ROOT),
                                                                "reference")
    src = os.path.join(root, "src")
    return src if os.path.isdir(src) else None


def build_oracle(verbose=False):
    cmd = ["make", "-s", "-C", os.path.join(ROOT, "oracle"), "all"]
    src = reference_src()
    if src:
        cmd.append("REF_SRC=" + src)
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force=False, verbose=False):
    build_library(force=force, verbose=verbose)
    build_oracle(verbose=verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
