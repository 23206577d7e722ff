"""Builds the native parts of kvflux_b200 in-tree.

Outputs (next to this file, git-ignored, shipped with the tree):
  libkvflux_b200.so  - CUDA kernels for sm_100a + C ABI (include/kvfx.h)
                       + the C++17 v2 API (include/kvflux/...)
  _C.<abi>.so        - pybind11 binding of the C++ API

Usage: python kvflux_b200/build.py [--force] [-j N]
Recompiles a source only when it, or any header of the tree, is newer than
its object file. nvcc cross-compiles for sm_100a without a GPU.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build" / "kvflux_b200"
LIB = PKG / "libkvflux_b200.so"
EXT_SUFFIX = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
PYMOD = PKG / f"_C{EXT_SUFFIX}"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", f"-I{INCLUDE}", f"-I{CSRC}", f"-I{CUDA_HOME / 'include'}"]


def _sources() -> list[Path]:
    files = sorted(CSRC.glob("control/*.cpp")) + sorted(CSRC.glob("data/*.cpp"))
    files += sorted(CSRC.glob("kernels/*.cu")) + [CSRC / "capi.cu"]
    return files


def _headers() -> list[Path]:
    return sorted(INCLUDE.rglob("*.h")) + sorted(CSRC.rglob("*.h")) + sorted(CSRC.rglob("*.cuh"))


def _newest(paths) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def _compile(src: Path, force: bool, header_time: float) -> Path:
    obj = BUILD / (src.relative_to(CSRC).as_posix().replace("/", "__") + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, header_time):
        return obj
    obj.parent.mkdir(parents=True, exist_ok=True)
    if src.suffix == ".cu":
        cmd = [NVCC, *ARCH, *COMMON, "-lineinfo", "-Xcompiler", "-fPIC,-Wall", "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++", *COMMON, "-fPIC", "-Wall", "-Wextra", "-c", str(src), "-o", str(obj)]
    _run(cmd)
    return obj


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> None:
    header_time = _newest(_headers())
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, header_time), srcs))
    if force or not LIB.exists() or LIB.stat().st_mtime < _newest(objs):
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-Xcompiler", "-fPIC", *map(str, objs),
              "-o", str(LIB), "-Xlinker", "-soname=libkvflux_b200.so", "-lpthread", "-ldl", "-lrt"])
        if verbose:
            print(f"linked {LIB}")
    pybind_src = CSRC / "pybind.cpp"
    if force or not PYMOD.exists() or PYMOD.stat().st_mtime < max(LIB.stat().st_mtime, pybind_src.stat().st_mtime,
                                                                   header_time):
        import pybind11

        py_inc = sysconfig.get_paths()["include"]
        _run(["g++", "-std=c++17", "-O2", "-shared", "-fPIC", "-fvisibility=hidden", f"-I{INCLUDE}",
              f"-I{CSRC}", f"-I{CUDA_HOME / 'include'}", f"-I{pybind11.get_include()}", f"-I{py_inc}",
              str(pybind_src), "-o", str(PYMOD), f"-L{PKG}", "-lkvflux_b200", "-Wl,-rpath,$ORIGIN"])
        if verbose:
            print(f"linked {PYMOD}")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=os.cpu_count() or 4)
    args = ap.parse_args(argv)
    build(force=args.force, jobs=args.jobs, verbose=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
