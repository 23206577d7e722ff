"""Builds the test oracles (TEST INFRASTRUCTURE ONLY).

  oracle/libkvoracle.so        - kvoracle.c, the CPU restatement of the path
  oracle/_ref/libkvflux_ref.so - the reference's own CPU sources (control plane
                                 and reference_attention) + ref_shim.cpp, built
                                 from a KVFlux checkout when one is found
                                 (--reference PATH, else $KVFLUX_REFERENCE, else a
                                 directory named "reference" beside this
                                 repository's own directory).
                                 The built file travels with the tree; the
                                 sources are never copied into it.
  oracle/_ref/libkvflux_ref_gpu.so - the reference's own GPU path (its CPU
                                 control plane, v1 GpuMemoryPool, v2 storage and
                                 its CUDA write/read/attention files) compiled
                                 with nvcc for sm_100a + ref_gpu_shim.cpp: the
                                 GPU-side baseline and an independent parity check.

Usage: python oracle/build.py [--force] [--reference PATH]
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "libkvoracle.so"
REF_DIR = HERE / "_ref"
REF_LIB = REF_DIR / "libkvflux_ref.so"
REF_GPU_LIB = REF_DIR / "libkvflux_ref_gpu.so"
# The reference's GPU path on top of REF_SOURCES (its CMake target builds the
# same files; src/v2/*.cu are its kernels).
REF_GPU_EXTRA = [
    "src/kv_layout.cpp",
    "src/gpu_memory_pool.cpp",
    "src/v2/paged_kv_storage.cpp",
    "src/v2/copy_on_write.cpp",
    "src/v2/paged_kv_write.cu",
    "src/v2/paged_kv_read.cu",
    "src/v2/paged_attention.cu",
]
REF_SOURCES = [
    "src/block_manager.cpp",
    "src/physical_block_pool.cpp",
    "src/v2/block_table.cpp",
    "src/v2/sequence_state.cpp",
    "src/v2/batch_block_table.cpp",
    "src/v2/slot_mapping.cpp",
    "src/v2/paged_kv_layout.cpp",
    "src/v2/reference_attention.cpp",
    "src/v2/prefix_cache.cpp",
    "src/v2/paged_kv_read_table.cpp",
]


_REFERENCE_OVERRIDE: Path | None = None


def reference_root() -> Path:
    """The KVFlux checkout whose sources the reference builds use: the
    --reference argument, else $KVFLUX_REFERENCE, else a sibling directory
    named "reference" next to this repository. It need not exist: without it
    only the C restatement is built."""
    if _REFERENCE_OVERRIDE is not None:
        return _REFERENCE_OVERRIDE
    env = os.environ.get("KVFLUX_REFERENCE")
    if env:
        return Path(env)
    return HERE.parent.parent / "reference"


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def _stale(out: Path, inputs: list[Path]) -> bool:
    return not out.exists() or out.stat().st_mtime < max(p.stat().st_mtime for p in inputs)


def build(force: bool = False) -> dict:
    built = {}
    srcs = [HERE / "kvoracle.c", HERE / "kvoracle.h"]
    if force or _stale(ORACLE_LIB, srcs):
        _run(["gcc", "-std=c11", "-O2", "-fPIC", "-shared", "-pthread", "-Wall", str(HERE / "kvoracle.c"),
              "-o", str(ORACLE_LIB), "-lm"])
    built["oracle"] = str(ORACLE_LIB)
    ref = reference_root()
    if (ref / "src" / "v2" / "reference_attention.cpp").exists():
        inputs = [ref / s for s in REF_SOURCES] + [HERE / "ref_shim.cpp"]
        if force or _stale(REF_LIB, inputs):
            REF_DIR.mkdir(exist_ok=True)
            _run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-fvisibility=hidden", "-pthread",
                  f"-I{ref / 'include'}", *map(str, inputs), "-o", str(REF_LIB)])
        built["reference"] = str(REF_LIB)
        gpu_inputs = [ref / s for s in REF_SOURCES + REF_GPU_EXTRA] + [HERE / "ref_gpu_shim.cpp"]
        if force or _stale(REF_GPU_LIB, gpu_inputs):
            nvcc = str(Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc")
            _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O2", "-shared",
                  "-Xcompiler", "-fPIC,-fvisibility=hidden", "-cudart", "static", f"-I{ref / 'include'}",
                  *map(str, gpu_inputs), "-o", str(REF_GPU_LIB)])
        built["reference_gpu"] = str(REF_GPU_LIB)
    elif REF_LIB.exists():
        built["reference"] = str(REF_LIB)  # prebuilt elsewhere, shipped with the tree
        if REF_GPU_LIB.exists():
            built["reference_gpu"] = str(REF_GPU_LIB)
    return built


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--reference", type=Path, default=None, help="KVFlux checkout to build the reference from")
    args = ap.parse_args(argv)
    global _REFERENCE_OVERRIDE
    if args.reference is not None:
        _REFERENCE_OVERRIDE = args.reference.resolve()
    for k, v in build(force=args.force).items():
        print(f"{k}: {v}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
