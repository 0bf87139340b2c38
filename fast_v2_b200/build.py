"""Build the two in-tree shared libraries of the package.

* ``libfdl_b200.so``  -- the C ABI of ``include/fdl_kvcache.h`` (all CUDA
  kernels), compiled by nvcc for sm_100a only.  Depends on the CUDA runtime
  alone; no torch types cross this boundary.
* ``libfdl_torch.so`` -- ``torch.library`` registration of the ``fdl`` ops on
  top of that ABI (host C++ only), linked against ``libfdl_b200.so`` with an
  ``$ORIGIN`` rpath.

Both land next to this file so they travel with the source tree.  Run as
``python -m fast_v2_b200.build`` or call :func:`build`.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB_ABI = PKG / "libfdl_b200.so"
LIB_TORCH = PKG / "libfdl_torch.so"

NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else (shutil.which("nvcc") or "nvcc")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed ({r.returncode}): {cmd[0]} ... {cmd[-1]}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)


def build_abi(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    deps = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "fdl_kvcache.h"]
    if not force and not _stale(LIB_ABI, deps):
        return LIB_ABI
    cmd = [_nvcc(), *NVCC_ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "--expt-relaxed-constexpr", str(CSRC / "fdl_b200.cu"), "-o", str(LIB_ABI) + ".tmp"]
    if ptxas_verbose:
        cmd.insert(1, "-Xptxas=-v")
    _run(cmd, verbose)
    os.replace(str(LIB_ABI) + ".tmp", LIB_ABI)
    return LIB_ABI


def build_torch(force: bool = False, verbose: bool = False) -> Path:
    deps = [CSRC / "torch_ops.cpp", INCLUDE / "fdl_kvcache.h", LIB_ABI]
    if not force and not _stale(LIB_TORCH, deps):
        return LIB_TORCH
    import torch
    from torch.utils import cpp_extension as ce

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = ce.include_paths(device_type="cuda")
    libdirs = ce.library_paths(device_type="cuda")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", str(CSRC / "torch_ops.cpp"), "-o", str(LIB_TORCH) + ".tmp"]
    cmd += [f"-I{d}" for d in incs]
    cmd += [f"-L{d}" for d in libdirs]
    cmd += [f"-L{PKG}", "-lfdl_b200", "-Wl,-rpath,$ORIGIN", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
            "-ltorch_cuda", "-lcudart"]
    _run(cmd, verbose)
    os.replace(str(LIB_TORCH) + ".tmp", LIB_TORCH)
    return LIB_TORCH


def build(force: bool = False, verbose: bool = False) -> tuple[Path, Path]:
    return build_abi(force, verbose), build_torch(force, verbose)


if __name__ == "__main__":
    force = "--force" in sys.argv
    a, t = build(force=force, verbose="-v" in sys.argv)
    print(a)
    print(t)
