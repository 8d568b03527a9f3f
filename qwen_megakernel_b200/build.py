"""In-tree build of the native libraries (sm_100a only, no JIT cache).

Outputs, next to this file:
  libqwen_megakernel.so   the C-ABI library (kernels + launchers), nvcc, static
                          cudart; no vendor GEMM library
  qwen_megakernel_C.so    the torch operator library (TORCH_LIBRARY qwen_megakernel_C)

Mirrors the role of the reference's qwen_megakernel/build.py (JIT
torch.utils.cpp_extension.load with -arch=sm_120a and -D tuning macros), but
builds ahead of time, in-tree, for sm_100a only.

    python -m qwen_megakernel_b200.build [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
import sysconfig

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")

LIB_PATH = os.path.join(PKG_DIR, "libqwen_megakernel.so")
OPS_PATH = os.path.join(PKG_DIR, "qwen_megakernel_C.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]

NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-shared",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]

KERNEL_SOURCES = [
    os.path.join(CSRC, "megakernel.cu"),
    os.path.join(CSRC, "batch.cu"),
    os.path.join(CSRC, "gemm_tc.cu"),
]
KERNEL_DEPS = KERNEL_SOURCES + [
    os.path.join(CSRC, "qmk_device.cuh"),
    os.path.join(CSRC, "qmk_schedule.h"),
    os.path.join(INCLUDE, "qwen_megakernel.h"),
]
OPS_SOURCES = [os.path.join(CSRC, "torch_bindings.cpp")]
OPS_DEPS = OPS_SOURCES + [os.path.join(INCLUDE, "qwen_megakernel.h")]


def _cuda_home() -> str:
    home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if home:
        return home
    nvcc = shutil.which("nvcc")
    if nvcc:
        return os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))
    return "/usr/local/cuda"


def _nvcc() -> str:
    return os.path.join(_cuda_home(), "bin", "nvcc")


def _digest(deps: list[str], extra: list[str]) -> str:
    h = hashlib.sha256()
    for d in deps:
        with open(d, "rb") as f:
            h.update(f.read())
    for e in extra:
        if not e.startswith("-I"):  # paths differ between checkouts; contents matter
            h.update(e.encode())
    return h.hexdigest()


def _stale(output: str, deps: list[str], extra: list[str]) -> bool:
    """An output is stale when it is missing or was built from other source
    contents or flags (content hash, so copying the tree keeps it fresh)."""
    stamp = output + ".sha256"
    if not (os.path.exists(output) and os.path.exists(stamp)):
        return True
    with open(stamp) as f:
        return f.read().strip() != _digest(deps, extra)


def _stamp(output: str, deps: list[str], extra: list[str]) -> None:
    with open(output + ".sha256", "w") as f:
        f.write(_digest(deps, extra) + "\n")


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        msg = (res.stderr or "") + (res.stdout or "")
        raise RuntimeError(f"build command failed ({res.returncode}): {' '.join(cmd)}\n{msg}")


def _link_flags() -> list[str]:
    """Static cudart only: every kernel is this library's own (the GEMMs of
    the token-parallel path included); the driver's tensor-map encoder is
    reached through cudaGetDriverEntryPoint, so no libcuda link either."""
    return []


def build_kernel_library(force: bool = False, verbose: bool = False) -> str:
    if force or _stale(LIB_PATH, KERNEL_DEPS, NVCC_FLAGS + _link_flags()):
        tmp = LIB_PATH + ".tmp"
        _run([_nvcc()] + NVCC_FLAGS + KERNEL_SOURCES + ["-o", tmp] + _link_flags(), verbose)
        os.replace(tmp, LIB_PATH)
        _stamp(LIB_PATH, KERNEL_DEPS, NVCC_FLAGS + _link_flags())
    return LIB_PATH


def _torch_paths():
    import torch
    from torch.utils import cpp_extension

    incs = cpp_extension.include_paths()
    libs = cpp_extension.library_paths()
    site = os.path.dirname(os.path.dirname(torch.__file__))
    cudart_dir = os.path.join(site, "nvidia", "cuda_runtime", "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return incs, libs, cudart_dir, abi


def build_ops_library(force: bool = False, verbose: bool = False) -> str:
    if not (force or _stale(OPS_PATH, OPS_DEPS, [])):
        return OPS_PATH
    incs, libs, cudart_dir, abi = _torch_paths()
    py_inc = sysconfig.get_paths()["include"]
    cmd = [
        os.environ.get("CXX", "g++"),
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_EXTENSION_NAME=qwen_megakernel_C",
        f"-I{INCLUDE}",
        f"-I{py_inc}",
        f"-I{os.path.join(_cuda_home(), 'include')}",
    ]
    cmd += [f"-I{p}" for p in incs]
    cmd += OPS_SOURCES
    cmd += ["-o", OPS_PATH + ".tmp", f"-L{PKG_DIR}", "-lqwen_megakernel"]
    for p in libs:
        cmd += [f"-L{p}", f"-Wl,-rpath,{p}"]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda"]
    if os.path.isdir(cudart_dir):
        cmd += [f"-L{cudart_dir}", f"-Wl,-rpath,{cudart_dir}", "-l:libcudart.so.12"]
    else:
        cmd += [f"-L{os.path.join(_cuda_home(), 'lib64')}", "-lcudart"]
    cmd += ["-Wl,-rpath,$ORIGIN"]
    _run(cmd, verbose)
    os.replace(OPS_PATH + ".tmp", OPS_PATH)
    _stamp(OPS_PATH, OPS_DEPS, [])
    return OPS_PATH


def build(force: bool = False, verbose: bool = False) -> tuple[str, str]:
    """Compile both libraries unless their source contents are unchanged."""
    lib = build_kernel_library(force, verbose)
    ops = build_ops_library(force, verbose)
    return lib, ops


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    lib, ops = build(force=args.force, verbose=args.verbose)
    print(lib)
    print(ops)
    return 0


if __name__ == "__main__":
    sys.exit(main())
