"""Builds libomni_b200.so (sm_100a) in-tree with nvcc.

Each csrc/*.cu (and host-only csrc/*.cpp) compiles to an object under sglang-omni_b200/_build/ (in
parallel, skipped when newer than its sources), then one shared library is
linked into sglang-omni_b200/omni_b200/.  No torch dependency: the library
links the static CUDA runtime and resolves driver entry points at run time.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
BUILD = ROOT / "_build"
INCLUDE = ROOT.parent / "include"
LIB = ROOT / "omni_b200" / "libomni_b200.so"
TORCH_OPS_SRC = ROOT / "torch_ext" / "omni_torch_ops.cpp"
TORCH_OPS_LIB = ROOT / "omni_b200" / "libomni_torch_ops.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-diag-suppress",
    "177",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the omni_b200 CUDA library cannot be built")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    if _stale(obj, [src, *_headers()]):
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stderr[-6000:]}")
    return obj


def build(verbose: bool = False, extra: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    workers = max(1, min(len(sources), os.cpu_count() or 4))
    with concurrent.futures.ThreadPoolExecutor(workers) as pool:
        objs = list(pool.map(lambda s: _compile(s, extra or []), sources))
    if _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stderr[-4000:]}")
    if verbose:
        print(f"built {LIB}")
    return LIB


def build_torch_ops(verbose: bool = False) -> Path:
    """The torch operator registration (torch_ext/omni_torch_ops.cpp, TORCH_LIBRARY): a
    host-only C++ library over libomni_b200.so's C ABI, compiled against the installed
    torch's headers and linked with an $ORIGIN rpath, next to libomni_b200.so."""
    import torch
    from torch.utils import cpp_extension as ce

    if not _stale(TORCH_OPS_LIB, [TORCH_OPS_SRC, LIB, *sorted(INCLUDE.glob("*.h"))]):
        return TORCH_OPS_LIB
    cuda_home = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    incs = ce.include_paths() + [str(cuda_home / "include"), str(INCLUDE)]
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=omni_torch_ops", *[f"-I{i}" for i in incs], str(TORCH_OPS_SRC),
           f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", f"-Wl,-rpath,{torch_lib}",
           f"-L{LIB.parent}", "-l:libomni_b200.so", "-Wl,-rpath,$ORIGIN", "-o", str(TORCH_OPS_LIB)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"torch ops build failed:\n{proc.stderr[-6000:]}")
    if verbose:
        print(f"built {TORCH_OPS_LIB}")
    return TORCH_OPS_LIB


if __name__ == "__main__":
    build(verbose=True, extra=sys.argv[1:])
    build_torch_ops(verbose=True)
