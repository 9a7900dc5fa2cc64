"""Golden update-size figures made by running the reference's own size comparison
(bench/compare.py of crukx-sync, imported unchanged) on seeded inputs from tests/cases.py.

    python tests/golden/make_sizes_golden.py /path/to/crukx-sync

compare.py imports ``zstandard`` at module level; it is not installed here, so a stand-in module
is registered first.  The stand-in only serves the import: the two columns that compress with zstd
(nemo, pulse) are not recorded.  raw, sparserl and ctxfree use numpy only and are recorded as the
reference computes them.  Writes sizes.json beside this script: per case the SHA-256 of its
inputs and the three sizes in bytes.
"""

from __future__ import annotations

import json
import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))   # tests/ for cases.py

import cases  # noqa: E402

CASES = ["rl_200k", "multi", "arbitrary", "one_group_wide", "rice_tail", "single", "extreme", "long_unary",
         "no_change", "heavy_10pct", "heavy_100pct", "single_group", "many_small", "toy_decoder"]


def main(ref_root: str):
    stub = types.ModuleType("zstandard")

    class _NoZstd:   # import-time stand-in; its output is never recorded
        def __init__(self, level=1):
            pass

        def compress(self, b):
            return b

    stub.ZstdCompressor = _NoZstd
    sys.modules["zstandard"] = stub
    sys.path.insert(0, os.path.join(ref_root, "bench"))
    import compare   # the reference's bench/compare.py, unchanged

    out = {}
    for name in CASES:
        fn, _ = cases.CASES[name]
        old, new = fn()[0]
        s = compare.sizes(old, new)
        out[name] = {"inputs_sha256": cases.digest_inputs(old, new),
                     "raw": int(s["raw"]), "sparserl": int(s["sparserl"]), "ctxfree": int(s["ctxfree"])}
        print(name, out[name])
    with open(os.path.join(HERE, "sizes.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main(sys.argv[1])
