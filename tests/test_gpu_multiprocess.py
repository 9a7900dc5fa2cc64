"""encode_update_global over real processes, one GPU each, NCCL: every rank returns the
reference's update.  Needs two GPUs (skipped otherwise)."""

import hashlib
import json
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import cases

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, out_dir):
    import datetime

    import torch.distributed as td

    from crukx_sync_b200 import dist as cdist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    td.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                          device_id=torch.device("cuda", rank))
    try:
        fn, chained = cases.CASES[name]
        cache = {} if chained else None
        digests = []
        for old, new in fn():
            names = list(old)
            a, b = cdist.partition_contiguous([old[n].numel() for n in names], world)[rank]
            mine = names[a:b]
            upd = cdist.encode_update_global({n: old[n].cuda() for n in mine}, {n: new[n].cuda() for n in mine}, cache)
            digests.append([len(upd), hashlib.sha256(upd).hexdigest()])
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(digests, f)
    finally:
        td.destroy_process_group()


@pytest.mark.parametrize("name", ["multi", "chain5", "heavy_100pct", "many_small"])
def test_global_update_over_nccl(tmp_path, name):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mp.spawn(_worker, args=(world, _port(), name, str(tmp_path)), nprocs=world, join=True)
    want = [[s["update_len"], s["update_sha256"]] for s in json.load(open(os.path.join(GOLD, "manifest.json")))[name]["steps"]]
    for r in range(world):
        assert json.load(open(os.path.join(tmp_path, f"rank{r}.json"))) == want
