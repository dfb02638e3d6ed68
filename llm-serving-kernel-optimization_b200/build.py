"""Build the sm_100a kernel library and the torch custom-op shim in-tree.

    python llm-serving-kernel-optimization_b200/build.py [--force] [--jobs N]

Outputs (git-ignored, shipped with the source tree):
    lightning_router/_lib/liblr_kernels.so     C ABI (include/lightning_router.h),
                                               kernels for sm_100a only
    lightning_router/_lib/_lr_torch_ops.so     torch.ops.lightning_router.*

nvcc cross-compiles without a GPU; the build is incremental on file mtimes.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB_DIR = HERE / "lightning_router" / "_lib"
OBJ_DIR = HERE / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")

CU_SOURCES = ["lr_capi.cu", "lr_routing.cu", "lr_w4a16_gemm.cu", "lr_w4a16_i8.cu",
              "lr_w4a16_skinny.cu", "lr_w4a16_generic.cu", "lr_ep.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr", "-I", str(INCLUDE),
]
KERNEL_LIB = LIB_DIR / "liblr_kernels.so"
OPS_LIB = LIB_DIR / "_lr_torch_ops.so"


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def build_kernels(force: bool = False, jobs: int = 4) -> Path:
    OBJ_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    objs = []
    todo = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = OBJ_DIR / (s.stem + ".o")
        objs.append(o)
        if force or _stale(o, [s] + _headers()):
            todo.append([NVCC, *NVCC_FLAGS, "-c", str(s), "-o", str(o)])
    with ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        list(ex.map(_run, todo))
    if force or _stale(KERNEL_LIB, objs):
        _run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
              "-o", str(KERNEL_LIB), *map(str, objs)])
    return KERNEL_LIB


def build_torch_ops(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "lr_torch_ops.cpp"
    if not (force or _stale(OPS_LIB, [src, KERNEL_LIB] + _headers())):
        return OPS_LIB
    inc = cpp_extension.include_paths() + [str(CUDA_HOME / "include"), str(INCLUDE),
                                           sysconfig.get_paths()["include"]]
    libdirs = cpp_extension.library_paths()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_lr_torch_ops", str(src), "-o", str(OPS_LIB)]
    for i in inc:
        cmd += ["-I", i]
    for d in libdirs:
        cmd += ["-L", d, f"-Wl,-rpath,{d}"]
    cmd += ["-L", str(LIB_DIR), "-l:liblr_kernels.so", "-Wl,-rpath,$ORIGIN",
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda"]
    _run(cmd)
    return OPS_LIB


def build(force: bool = False, jobs: int = 4) -> None:
    build_kernels(force, jobs)
    build_torch_ops(force)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=4)
    a = ap.parse_args()
    build(a.force, a.jobs)
    sys.exit(0)
