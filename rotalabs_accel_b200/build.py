"""Build the sm_100a W8A16 library in-tree.

    python -m rotalabs_accel_b200.build        (or __graft_entry__.build())

Compiles ``csrc/rla_lib.cu`` (one translation unit holding every kernel and
the C ABI of ``include/rla_w8a16.h``) with nvcc for ``sm_100a`` into
``rotalabs_accel_b200/librla_w8a16.so``.  The CUDA runtime is linked
statically; the driver's tensor-map encoder is reached through
``cudaGetDriverEntryPoint`` so nothing links ``libcuda`` directly.

Then compiles ``csrc/rla_pyfast.c``, the CPython fast-call bindings of the
hot entry points, with the host C compiler into ``_rla_fast<EXT_SUFFIX>``
next to the library, linked to it by soname with an ``$ORIGIN`` rpath; and
``csrc/rla_torch_op.cpp``, the ``torch.library`` registration of
``rla::w8a16_gemm`` over the same C ABI, against the installed torch's
headers and libraries into ``_rla_torch_ops.so``, which is also a Python
extension module: importing it registers the op and gives its CUDA kernel
function as ``_rla_torch_ops.w8a16_gemm`` (called without the dispatcher on
the per-token path).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_NAME = "librla_w8a16.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
FAST_PATH = os.path.join(HERE, "_rla_fast" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
TORCH_OP_PATH = os.path.join(HERE, "_rla_torch_ops.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-shared", "-cudart", "static",
    "--expt-relaxed-constexpr",
    "-Xlinker", "-soname=" + LIB_NAME,
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _cc() -> str:
    for cand in (os.environ.get("CC"), shutil.which("gcc"), shutil.which("cc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("no host C compiler found for the fast-call bindings")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)
                  if f.endswith((".cu", ".cuh", ".h"))) + \
        [os.path.join(os.path.dirname(HERE), "include", "rla_w8a16.h")]


def needs_build() -> bool:
    outs = (LIB_PATH, FAST_PATH, TORCH_OP_PATH)
    if not all(os.path.exists(o) for o in outs):
        return True
    t = min(os.path.getmtime(o) for o in outs)
    extra = [os.path.join(CSRC, "rla_pyfast.c"), os.path.join(CSRC, "rla_torch_op.cpp")]
    return any(os.path.getmtime(s) > t for s in _sources() + extra)


def build_torch_op(verbose: bool = False) -> str:
    """Compile the torch.library registration (rla::w8a16_gemm) against the
    installed torch and the built library."""
    import torch
    from torch.utils import cpp_extension
    cxx = shutil.which("g++") or shutil.which("c++")
    if not cxx:
        raise RuntimeError("no host C++ compiler found for the torch op registration")
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(_nvcc())), "include")
    tlib = cpp_extension.library_paths()[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_OP_PATH + ".tmp"
    cmd = [cxx, "-O2", "-shared", "-fPIC", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_rla_torch_ops", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{p}" for p in cpp_extension.include_paths()], f"-I{cuda_inc}",
           "-I" + sysconfig.get_paths()["include"],
           os.path.join(CSRC, "rla_torch_op.cpp"), "-L" + HERE, "-l:" + LIB_NAME, f"-L{tlib}",
           "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch", "-ltorch_python",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{tlib}", "-o", tmp]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building the torch op registration failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, TORCH_OP_PATH)
    return TORCH_OP_PATH


def build_fast(verbose: bool = False) -> str:
    """Compile the CPython fast-call module against the built library."""
    tmp = FAST_PATH + ".tmp"
    cmd = [_cc(), "-O2", "-shared", "-fPIC", "-std=c11", "-I" + sysconfig.get_paths()["include"],
           os.path.join(CSRC, "rla_pyfast.c"), "-L" + HERE, "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN", "-o", tmp]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building the fast-call bindings failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, FAST_PATH)
    return FAST_PATH


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    """Compile the library if a source is newer than it; return its path."""
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, *(extra_flags or []), os.path.join(CSRC, "rla_lib.cu"), "-o", tmp]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout, r.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    build_fast(verbose)
    build_torch_op(verbose)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
