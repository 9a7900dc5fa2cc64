"""The size-comparison restatement (oracle/sizes.py) against figures the reference's own
bench/compare.py produced (tests/golden/sizes.json), and the product's size formulas
(crukx_sync_b200.sizes.sizes_from_stats) against the restatement, from statistics computed on the
host in the layout crx_size_stats writes."""

import json
import os

import numpy as np
import pytest
import torch

import cases
from crukx_sync_b200 import sizes as psizes
from oracle import sizes as osizes

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "sizes.json")))


def host_stats(old, new):
    """crx_size_stats' words computed with numpy (the layout of include/crukx_b200.h)."""
    st = np.zeros(psizes.STATS_WORDS, dtype=np.uint64)
    for k in old:
        a = old[k].contiguous().view(torch.int16).reshape(-1).numpy()
        b = new[k].contiguous().view(torch.int16).reshape(-1).numpy()
        idx = np.flatnonzero(a != b).astype(np.int64)
        if not idx.size:
            continue
        prev = np.concatenate(([-1], idx[:-1]))
        g = idx - prev - 1
        d = g + 1
        d[0] = idx[0]
        lengths = np.array([int(x).bit_length() for x in g])
        st[0] += idx.size
        st[1] += int((d > 0xFFFF).sum())
        st[2] += int(np.maximum(lengths - 1, 0).sum())
        st[3:3 + 64] += np.bincount(lengths, minlength=64).astype(np.uint64)
        st[psizes._VAL:psizes._VAL + 65536] += np.bincount(b[idx].view(np.uint16), minlength=65536).astype(np.uint64)
        st[psizes._XOR:psizes._XOR + 65536] += np.bincount((a[idx] ^ b[idx]).view(np.uint16),
                                                           minlength=65536).astype(np.uint64)
    return st


@pytest.mark.parametrize("name", sorted(GOLD))
def test_restatement_matches_reference(name):
    fn, _ = cases.CASES[name]
    old, new = fn()[0]
    row = GOLD[name]
    assert cases.digest_inputs(old, new) == row["inputs_sha256"]
    got = osizes.update_sizes(old, new)
    assert got == {k: row[k] for k in ("raw", "sparserl", "ctxfree")}
    assert psizes.sizes_from_stats(host_stats(old, new)) == got

