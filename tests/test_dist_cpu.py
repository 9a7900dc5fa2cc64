"""Sharded sync host logic at world size 2 on CPU (gloo): partition, all-gather of the updates,
and a full round trip where every rank encodes its own tensors and applies the others' updates.

Encoding and applying run in the CPU oracle here (this suite has no GPU); the product code under
test is ``crukx_sync_b200.dist`` and the C++ parser (``crukx_sync_b200.wire.parse``).
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from crukx_sync_b200 import dist as cdist


def test_partition_is_deterministic_and_balanced():
    numels = {f"t{i}": (i * 7919) % 1000 + 1 for i in range(50)}
    a = cdist.partition(numels, 4)
    b = cdist.partition(dict(reversed(list(numels.items()))), 4)
    assert a == b
    loads = [sum(n for k, n in numels.items() if a[k] == r) for r in range(4)]
    assert max(loads) - min(loads) <= max(numels.values())
    assert set(a.values()) == {0, 1, 2, 3}
    assert cdist.partition(numels, 1) == {k: 0 for k in numels}
    with pytest.raises(ValueError):
        cdist.partition(numels, 0)


def test_partition_ties_go_to_the_lowest_rank():
    assert cdist.partition({"b": 5, "a": 5, "c": 1}, 2) == {"a": 0, "b": 1, "c": 0}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _states(seed):
    rng = np.random.default_rng(seed)
    shapes = {"embed": 40_000, "layer.0.w": 12_345, "layer.0.b": 77, "layer.1.w": 12_345, "norm": 1, "empty": 0}
    prev, cur = {}, {}
    for k, n in shapes.items():
        w = (rng.standard_normal(n) * 0.02).astype(np.float32)
        a = (w.view(np.uint32) >> 16).astype(np.uint16).view(np.int16)
        step = (rng.standard_normal(n) * 2e-4).astype(np.float32)
        b = ((w + step).view(np.uint32) >> 16).astype(np.uint16).view(np.int16)
        prev[k], cur[k] = torch.from_numpy(a.copy()), torch.from_numpy(b.copy())
    return prev, cur


def _worker(rank, world, port, outdir):
    from oracle import oracle

    from crukx_sync_b200 import wire

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch.distributed as td
    td.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        prev, cur = _states(0)                       # every rank holds the same model
        owner = cdist.partition({k: v.numel() for k, v in prev.items()}, world)
        mine = [k for k in prev if owner[k] == rank]
        upd = oracle.encode_update({k: prev[k] for k in mine}, {k: cur[k] for k in mine}, {})
        got = cdist.allgather_updates(upd, device=torch.device("cpu"))
        assert len(got) == world and got[rank] == upd
        only_next = cdist.allgather_updates(upd, device=torch.device("cpu"), ranks=[(rank + 1) % world])
        assert only_next == [got[(rank + 1) % world]]
        weights = {k: v.clone() for k, v in prev.items()}
        seen = set()
        for r, u in enumerate(got):
            p = wire.parse(u)                         # the product's parser validates every update
            names = [name for name, _, _ in p.tensor_table()]
            assert all(owner[n] == r for n in names)
            seen.update(names)
            oracle.apply_update({n: weights[n] for n in names}, u, {})
        changed = {k for k in prev if not torch.equal(prev[k], cur[k])}
        assert changed <= seen <= set(prev)
        for k in prev:
            assert torch.equal(weights[k], cur[k]), k
        # the device-resident exchange's host logic, on CPU tensors: sizes through a separate gloo
        # group (host_size_group) or through the data group, uneven sizes padded and cut back
        t = torch.frombuffer(bytearray(upd), dtype=torch.uint8)
        sg = cdist.host_size_group()
        for size_group in (sg, None):
            views = cdist.allgather_updates_device(t, size_group=size_group)
            assert [bytes(v.numpy().tobytes()) for v in views] == got
            mine_only = cdist.allgather_updates_device(t, ranks=[rank], size_group=size_group)
            assert bytes(mine_only[0].numpy().tobytes()) == upd
            pg = cdist.allgather_updates_device_async(t, size_group=size_group)   # CPU: completes at once
            pg.wait()
            assert [bytes(v.numpy().tobytes()) for v in pg.views()] == got
        with open(os.path.join(outdir, f"ok{rank}"), "w") as f:
            f.write(str(len(upd)))
    finally:
        td.destroy_process_group()


def test_sharded_round_trip_world2(tmp_path):
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    assert sorted(os.listdir(tmp_path)) == ["ok0", "ok1"]


def test_allgather_single_process_is_identity():
    assert cdist.allgather_updates(b"CRXS\x02abc") == [b"CRXS\x02abc"]
