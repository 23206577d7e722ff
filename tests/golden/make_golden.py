"""Regenerates the golden fixtures in this directory from the reference's own
compiled CPU code (oracle/_ref/libkvflux_ref.so, built by oracle/build.py from
a KVFlux checkout). Run from the repository root:

    python tests/golden/make_golden.py

reference_attention.json : seeded inputs (regenerated from the seed by
    kvflux_b200.workloads.normal) and the reference's FP32 outputs as bit
    patterns.
control_plane.json : page ids / slots / tables of tests/scenarios.py run on
    the reference's control plane.
"""
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import oracle  # noqa: E402
from oracle import refapi  # noqa: E402
from kvflux_b200 import workloads as w  # noqa: E402
import scenarios  # noqa: E402

SHAPES = [(1, 40, 8, 2, 64), (10, 10, 4, 2, 4), (3, 10, 4, 2, 4), (1, 10, 4, 2, 4), (4, 9, 6, 3, 3),
          (1, 64, 4, 1, 32)]


def main():
    if oracle.ref() is None:
        raise SystemExit("build oracle/_ref first: python oracle/build.py")
    cases = []
    for i, shape in enumerate(SHAPES):
        lq, lkv, hq, hkv, hd = shape
        seed = 0x601D + 97 * i
        q = w.normal(seed, lq * hq * hd)
        k = w.normal(seed + 1, lkv * hkv * hd)
        v = w.normal(seed + 2, lkv * hkv * hd)
        out = oracle.ref_reference_attention(q, k, v, shape)
        cases.append({"shape": list(shape), "seed": seed, "q_head_f32_bits": [int(x) for x in q[:4].view(np.uint32)],
                      "output_f32_bits": [int(x) for x in out.view(np.uint32)]})
    here = Path(__file__).resolve().parent
    (here / "reference_attention.json").write_text(json.dumps({"generator": "reference reference_attention",
                                                               "cases": cases}, indent=0))
    traces = {fn.__name__: fn(refapi) for fn in scenarios.ALL}
    (here / "control_plane.json").write_text(json.dumps(traces, indent=1))
    print("wrote", len(cases), "attention cases and", len(traces), "control-plane traces")


if __name__ == "__main__":
    main()
