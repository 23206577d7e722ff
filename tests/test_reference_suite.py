"""KVFlux's own v2 test programs, compiled unchanged against this repository's
include/ and linked with libkvflux_b200.so (tests/reference_suite/build.py),
must exit 0: the host-only programs here on the CPU, the GPU programs on a
B200. Their sources (KVFlux tests/*.cpp, tests/*.cu) are never copied into
this tree; the programs are built from a KVFlux checkout and carried as
binaries, so a machine without the checkout runs what was built."""
import subprocess
from pathlib import Path

import pytest

import kvflux_b200  # noqa: F401  (the library the programs link must be built)

HERE = Path(__file__).resolve().parent
BIN = HERE / "reference_suite" / "bin"

import importlib.util  # noqa: E402

_spec = importlib.util.spec_from_file_location("reference_suite_build", HERE / "reference_suite" / "build.py")
_suite = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_suite)
# Where a KVFlux checkout is found, bring the programs up to date with the
# current headers and library first (incremental); elsewhere run what was built.
_suite.build()


def _run(name: str, timeout: int = 300) -> None:
    exe = BIN / name
    if not exe.exists():
        pytest.skip(f"{name} not built (tests/reference_suite/build.py needs a KVFlux checkout)")
    proc = subprocess.run([str(exe)], capture_output=True, text=True, timeout=timeout)
    assert proc.returncode == 0, f"{name} exited {proc.returncode}\n{proc.stdout[-2000:]}\n{proc.stderr[-2000:]}"


@pytest.mark.parametrize("name", _suite.HOST_TESTS)
def test_reference_host_program(name):
    _run(name)


@pytest.mark.gpu
@pytest.mark.parametrize("name", _suite.GPU_TESTS)
def test_reference_gpu_program(name, cuda):
    _run(name)
