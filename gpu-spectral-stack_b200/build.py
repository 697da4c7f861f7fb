"""Builds the library in-tree, for sm_100a only.

    python gpu-spectral-stack_b200/build.py            # or __graft_entry__.build()

Produces, next to the Python package (gpu-spectral-stack_b200/spectral/):

- libspectral_b200.so  the C ABI of include/spectral_b200.h: every CUDA kernel, the registry,
                       the drivers. CUDA runtime linked statically; no torch.
- _C<ext-suffix>.so    the torch.ops.spectral operators, a thin shim over the C ABI, linked to
                       libspectral_b200.so through an $ORIGIN rpath.

Each .cu file compiles to its own object in parallel (the four engine variants are the long
ones). A target is rebuilt only when a source or header is newer than it. Objects go to _build/
at the repository root.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
OUT_DIR = PKG_ROOT / "spectral"
BUILD = REPO / "_build"
INCLUDE = REPO / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]

LIB_NAME = "libspectral_b200.so"


def cuda_home() -> Path:
    home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if home:
        return Path(home)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    return Path("/usr/local/cuda")


def nvcc() -> str:
    return str(cuda_home() / "bin" / "nvcc")


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + sorted(INCLUDE.glob("*.h"))


def newest(paths: list[Path]) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def stale(target: Path, deps: list[Path]) -> bool:
    return not target.exists() or target.stat().st_mtime < newest(deps)


def run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stderr}")


def compile_cu(src: Path, hdrs: list[Path]) -> Path:
    obj = BUILD / (src.stem + ".o")
    if stale(obj, [src, *hdrs]):
        run([nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    return obj


def build_library(jobs: int) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdrs = headers()
    sources = sorted(CSRC.glob("*.cu"))
    # The long-compiling engine variants first, so they overlap with everything else.
    sources.sort(key=lambda p: (not p.name.startswith("variant_"), p.name))
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as pool:
        objs = list(pool.map(lambda s: compile_cu(s, hdrs), sources))
    lib = OUT_DIR / LIB_NAME
    if stale(lib, objs):
        # Only the C ABI is exported: the objects are built with hidden visibility and the
        # header's declarations carry default visibility (SPECTRAL_API).
        run([nvcc(), *ARCH, "-shared", "-o", str(lib), *map(str, objs)])
    return lib


def torch_paths() -> tuple[list[str], list[str], bool]:
    import torch
    from torch.utils import cpp_extension

    includes = cpp_extension.include_paths()
    libs = cpp_extension.library_paths()
    return includes, libs, bool(torch._C._GLIBCXX_USE_CXX11_ABI)


def host_cxx() -> str:
    """The host C++ compiler for the torch shim: SPECTRAL_CXX if set, else the g++ on PATH (the
    one nvcc uses for host code). CXX is deliberately not used: a toolchain wrapper there may link
    libstdc++ statically, and a shim with a private libstdc++ inside a process that already has the
    shared one breaks iostream formatting (c10::str of an integer) once both are initialised."""
    return os.environ.get("SPECTRAL_CXX") or shutil.which("g++") or "g++"


def check_shared_libstdcxx(path: Path) -> None:
    """Fails the build unless `path` links libstdc++ dynamically."""
    out = subprocess.run(["readelf", "-d", str(path)], capture_output=True, text=True).stdout
    if "libstdc++.so" not in out:
        raise RuntimeError(
            f"{path.name} does not link libstdc++.so dynamically; set SPECTRAL_CXX to a g++ that "
            "links the shared libstdc++"
        )


def build_torch_shim(lib: Path) -> Path:
    src = CSRC / "torch_ops.cpp"
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    out = OUT_DIR / ("_C" + suffix)
    if not stale(out, [src, lib, *headers()]):
        return out
    includes, libdirs, cxx11 = torch_paths()
    py_inc = sysconfig.get_paths()["include"]
    cmd = [
        host_cxx(),
        "-shared",
        "-fPIC",
        "-O2",
        "-std=c++17",
        f"-D_GLIBCXX_USE_CXX11_ABI={int(cxx11)}",
        "-DTORCH_EXTENSION_NAME=_C",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        f"-I{py_inc}",
        f"-I{cuda_home() / 'include'}",
        *[f"-I{p}" for p in includes],
        str(src),
        "-o",
        str(out),
        f"-L{OUT_DIR}",
        "-l:" + LIB_NAME,
        *[f"-L{p}" for p in libdirs],
        "-lc10",
        "-lc10_cuda",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_cuda",
        "-ltorch_python",
        "-Wl,-rpath,$ORIGIN",
        *[f"-Wl,-rpath,{p}" for p in libdirs],
    ]
    run(cmd)
    check_shared_libstdcxx(out)
    return out


def build(jobs: int | None = None) -> tuple[Path, Path]:
    jobs = jobs or max(1, min(8, os.cpu_count() or 1))
    lib = build_library(jobs)
    shim = build_torch_shim(lib)
    return lib, shim


if __name__ == "__main__":
    lib, shim = build()
    print(lib)
    print(shim)
    sys.exit(0)
