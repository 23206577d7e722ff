"""Builds KVFlux's own v2 test programs, unchanged, against this repository's
headers (include/) and library (kvflux_b200/libkvflux_b200.so): the proof that
a KVFlux translation unit compiles and passes against this implementation of
the API with no source change.

The test sources are read from a KVFlux checkout (--reference PATH, else
$KVFLUX_REFERENCE, else a directory named "reference" beside this
repository's own directory) and compiled where they lie; nothing is copied
into this tree. The programs are written to tests/reference_suite/bin/
(git-ignored; they travel with the working tree to a GPU machine, which has no
checkout). Each program links libkvflux_b200.so through an $ORIGIN-relative
rpath and the CUDA runtime statically, as KVFlux's CMake target
(tests/CMakeLists.txt:1-136) links its own library.

Programs (KVFlux tests/CMakeLists.txt target names in brackets):
  host only  block_manager [kvflux_tests], physical_block_pool, block_table,
             batch_block_table, sequence_state, copy_on_write, prefix_cache,
             fragmentation, oom, slot_mapping, paged_kv_layout,
             paged_kv_read_table, reference_attention
  GPU        paged_kv_write, paged_kv_read, paged_kv_gather, paged_kv_storage,
             paged_attention (.cu), paged_attention_batch (.cu),
             copy_on_write_gpu, sequence_lifecycle
Not built: kv_layout_test, gpu_memory_pool_test, async_transfer_test,
tiered_block_manager_test and the v3_* tests, which test the v0/v1 layout,
host<->GPU block copies and offload tiers that this library does not
implement.

Usage: python tests/reference_suite/build.py [--force] [--reference PATH]
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
BIN = HERE / "bin"
LIB_DIR = ROOT / "kvflux_b200"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

HOST_TESTS = [
    "block_manager_test", "physical_block_pool_test", "block_table_test", "batch_block_table_test",
    "sequence_state_test", "copy_on_write_test", "prefix_cache_test", "fragmentation_test", "oom_test",
    "slot_mapping_test", "paged_kv_layout_test", "paged_kv_read_table_test", "reference_attention_test",
]
GPU_TESTS = [
    "paged_kv_write_test", "paged_kv_read_test", "paged_kv_gather_test", "paged_kv_storage_test",
    "paged_attention_test", "paged_attention_batch_test", "copy_on_write_gpu_test", "sequence_lifecycle_test",
]


def reference_root(arg: Path | None = None) -> Path:
    if arg is not None:
        return arg
    env = os.environ.get("KVFLUX_REFERENCE")
    if env:
        return Path(env)
    return ROOT.parent / "reference"


def _source(ref: Path, name: str) -> Path:
    cu = ref / "tests" / f"{name}.cu"
    return cu if cu.exists() else ref / "tests" / f"{name}.cpp"


def _link_flags() -> list[str]:
    return [f"-L{LIB_DIR}", "-lkvflux_b200", f"-L{CUDA_HOME / 'lib64'}", "-lcudart_static", "-ldl", "-lrt",
            "-lpthread"]


def _build_one(ref: Path, name: str, force: bool) -> str:
    src = _source(ref, name)
    out = BIN / name
    lib = LIB_DIR / "libkvflux_b200.so"
    headers = list((ROOT / "include").rglob("*.h"))
    newest = max([src.stat().st_mtime, lib.stat().st_mtime] + [h.stat().st_mtime for h in headers])
    if not force and out.exists() and out.stat().st_mtime >= newest:
        return name
    inc = [f"-I{ROOT / 'include'}", f"-I{CUDA_HOME / 'include'}"]
    if src.suffix == ".cu":
        cmd = [str(CUDA_HOME / "bin" / "nvcc"), "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a",
               *inc, str(src), "-o", str(out), "-Xlinker", "-rpath,$ORIGIN/../../../kvflux_b200", *_link_flags()]
    else:
        cmd = ["g++", "-std=c++17", "-O2", *inc, str(src), "-o", str(out), "-Wl,-rpath,$ORIGIN/../../../kvflux_b200",
               *_link_flags()]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"building {name} failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    return name


def build(force: bool = False, reference: Path | None = None) -> list[str]:
    """Builds every program whose source is found; returns their names
    (empty when no checkout is found). Needs libkvflux_b200.so built first."""
    ref = reference_root(reference)
    if not (ref / "tests" / "paged_kv_write_test.cpp").exists():
        return []
    if not (LIB_DIR / "libkvflux_b200.so").exists():
        raise RuntimeError("build libkvflux_b200.so first (python kvflux_b200/build.py)")
    BIN.mkdir(parents=True, exist_ok=True)
    names = HOST_TESTS + GPU_TESTS
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        return list(ex.map(lambda n: _build_one(ref, n, force), names))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--reference", type=Path, default=None)
    args = ap.parse_args(argv)
    built = build(force=args.force, reference=args.reference)
    print(f"built {len(built)} programs into {BIN}" if built else "no KVFlux checkout found: nothing built")
    return 0


if __name__ == "__main__":
    sys.exit(main())
