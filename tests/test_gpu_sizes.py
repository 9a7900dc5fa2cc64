"""crx_size_stats (the CUDA statistics behind the size comparison) against figures the reference's
own bench/compare.py produced and against the numpy restatement, including tile and tensor
boundaries, unaligned views and 2^24-element tensors."""

import json
import os

import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "sizes.json")))


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from crukx_sync_b200 import _ext
    _ext.load()


def cu(d):
    return {k: v.cuda() for k, v in d.items()}


@pytest.mark.parametrize("name", sorted(GOLD))
def test_sizes_match_reference(name):
    from crukx_sync_b200 import sizes
    fn, _ = cases.CASES[name]
    old, new = fn()[0]
    row = GOLD[name]
    assert sizes.update_sizes(cu(old), cu(new)) == {k: row[k] for k in ("raw", "sparserl", "ctxfree")}


def test_statistics_match_host_statistics_at_tile_boundaries():
    from crukx_sync_b200 import sizes
    from test_sizes_cpu import host_stats
    g = torch.Generator().manual_seed(5)
    old, new = {}, {}
    for i, n in enumerate([1, 8191, 8192, 8193, 3 * 8192 + 77, 100_000]):
        a = torch.randint(-32768, 32768, (n + 1,), generator=g, dtype=torch.int32).to(torch.int16)[1:]   # odd start
        b = a.clone()
        pick = torch.rand(n, generator=g) < (0.5 if i % 2 else 0.002)
        b[pick] ^= 1 + torch.randint(0, 7, (int(pick.sum()),), generator=g, dtype=torch.int16)
        old[f"t{i}"], new[f"t{i}"] = a, b
    old["empty"], new["empty"] = torch.zeros(0, dtype=torch.int16), torch.zeros(0, dtype=torch.int16)
    got = sizes.size_stats(cu(old), cu(new))
    assert np.array_equal(got, host_stats(old, new))


@pytest.mark.parametrize("frac", [0.01, 1.0])
def test_sizes_match_restatement_at_16m(frac):
    from crukx_sync_b200 import sizes
    from oracle import sizes as osizes
    a, b = cases.heavy_tail((1 << 24) + 13, frac, seed=31)
    assert sizes.update_sizes({"x": a.cuda()}, {"x": b.cuda()}) == osizes.update_sizes({"x": a}, {"x": b})
