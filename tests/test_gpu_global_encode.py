"""One update encoded by several ranks (crx_encode_global) is byte-identical to the reference's
single encode of all tensors.  Ranks are emulated as threads of one process on one GPU, each with
its own library context and CUDA stream; the collectives are in-process (a barrier)."""

import ctypes
import hashlib
import json
import os
import threading

import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")
MANIFEST = json.load(open(os.path.join(GOLD, "manifest.json")))


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from crukx_sync_b200 import _ext
    _ext.load()


class Collective:
    def __init__(self, world):
        self.world = world
        self.barrier = threading.Barrier(world, timeout=120)
        self.slots = [None] * world

    def sum(self, rank, arr):
        self.slots[rank] = arr.copy()
        self.barrier.wait()
        tot = np.zeros_like(arr)
        for s in self.slots:
            tot += s                      # uint64: wraps like the library expects
        self.barrier.wait()
        arr[:] = tot

    def gather(self, rank, mine):
        self.slots[rank] = mine
        self.barrier.wait()
        out = b"".join(self.slots)
        self.barrier.wait()
        return out


def encode_global(parts, caches=None):
    """parts: per rank (old, new) dicts on the GPU; returns (update bytes, per-rank checksums)."""
    from crukx_sync_b200 import _ext, codec
    from crukx_sync_b200.wire import assemble
    world = len(parts)
    coll = Collective(world)
    L = _ext.load()
    results, errors = [None] * world, []

    def run(r):
        ctx = ctypes.c_void_p()
        err = ctypes.create_string_buffer(256)
        assert L.crx_ctx_create(torch.cuda.current_device(), ctypes.byref(ctx), err, 256) == 0, err.value
        try:
            with torch.cuda.stream(torch.cuda.Stream()):
                old, new = parts[r]
                enc = codec.encode_global(old, new, caches[r] if caches else None, r, world,
                                          lambda a: coll.sum(r, a), lambda m: coll.gather(r, m), ctx=ctx)
                results[r] = (enc.part(), enc.checksums)
                enc.close()
                torch.cuda.current_stream().synchronize()
        except Exception as exc:   # surfaces in the main thread
            errors.append(exc)
            coll.barrier.abort()
        finally:
            L.crx_ctx_destroy(ctx)

    threads = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if errors:
        raise errors[0]
    return assemble([p for p, _ in results]), [c for _, c in results]


def split(old, new, world):
    from crukx_sync_b200.dist import partition_contiguous
    names = list(old)
    ranges = partition_contiguous([old[n].numel() for n in names], world)
    return [({n: old[n].cuda() for n in names[a:b]}, {n: new[n].cuda() for n in names[a:b]}) for a, b in ranges]


CASES = ["multi", "arbitrary", "one_group_wide", "rice_dense", "rice_tail", "single", "extreme", "long_unary",
         "no_change", "empty", "chain5", "heavy_10pct", "heavy_100pct", "single_group", "many_small"]


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("name", CASES)
def test_global_update_is_the_reference_update(name, world):
    fn, chained = cases.CASES[name]
    caches = [{} for _ in range(world)] if chained else None
    for k, (old, new) in enumerate(fn()):
        row = MANIFEST[name]["steps"][k]
        upd, chk = encode_global(split(old, new, world), caches)
        assert (len(upd), hashlib.sha256(upd).hexdigest()) == (row["update_len"], row["update_sha256"]), k
        if chained:
            merged = {}
            for c in caches:
                merged.update(c)
            for r, c in enumerate(chk):
                caches[r].update(c)
                merged.update(c)
            assert {n: str(v) for n, v in merged.items()} == row["sender_checksums"]


def test_global_update_applies_like_the_single_one():
    import crukx_sync_b200 as crx
    old, new = cases.case_multi()[0]
    upd, _ = encode_global(split(old, new, 2))
    assert upd == crx.encode_update({k: v.cuda() for k, v in old.items()}, {k: v.cuda() for k, v in new.items()})
    w = {k: v.cuda() for k, v in old.items()}
    crx.apply_update(w, upd)
    for k in new:
        assert torch.equal(w[k].cpu().view(torch.int16), new[k].view(torch.int16))


def test_rank_without_tensors_and_rank_without_changes():
    import crukx_sync_b200 as crx
    a, b = cases.rl_pair(50_000)
    c, _ = cases.rl_pair(30_000)
    old = {"x": a, "y": c}
    new = {"x": b, "y": c.clone()}       # y does not change: its rank contributes no groups
    single = crx.encode_update({k: v.cuda() for k, v in old.items()}, {k: v.cuda() for k, v in new.items()})
    parts = [({"x": a.cuda()}, {"x": b.cuda()}), ({"y": c.cuda()}, {"y": c.cuda()}), ({}, {})]
    upd, _ = encode_global(parts)
    assert upd == single
