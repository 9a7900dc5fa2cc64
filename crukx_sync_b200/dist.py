"""Sharded weight sync over ``torch.distributed``: one process per GPU.

The reference syncs one model as one update (src/crukx_sync/__init__.py:38-57); it has no
multi-process layer.  On N GPUs the tensors are split between ranks, each rank encodes its own
tensors into an independent, complete update, and the compressed updates cross the job with one
all-gather (NCCL on GPUs, gloo on CPU).  A rank then applies the updates of the tensors it
holds.  Nothing else is exchanged: encode and apply stay local, so the work per rank shrinks as
N grows.

    owner = partition({name: t.numel() for name, t in model.items()}, world)
    mine = {k: v for k, v in model.items() if owner[k] == rank}
    upd = crukx_sync_b200.encode_update(prev_mine, cur_mine, send_chk)
    for u in allgather_updates(upd, ranks=holders):
        crukx_sync_b200.apply_update(weights, u, recv_chk)

With encode_update_device and allgather_updates_device the updates stay in GPU memory end to end.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence

import torch


def partition(numels: Mapping[str, int], world: int) -> dict[str, int]:
    """Owner rank of every tensor: longest-processing-time first on element counts.

    Deterministic on every rank (ties: larger tensor first, then name; then the least-loaded,
    lowest rank), so ranks agree without communicating.
    """
    if world < 1:
        raise ValueError(f"world size must be >= 1, got {world}")
    load = [0] * world
    owner = {}
    for name in sorted(numels, key=lambda k: (-int(numels[k]), k)):
        r = min(range(world), key=lambda i: (load[i], i))
        owner[name] = r
        load[r] += int(numels[name])
    return owner


def allgather_updates(update: bytes, group=None, device: torch.device | None = None,
                      ranks: Sequence[int] | None = None) -> list[bytes]:
    """All-gather every rank's update bytes; returns those of ``ranks`` (default: all), in order.

    Two collectives, taken by every rank in the same order: the sizes, then the payloads padded
    to the largest, into one flat buffer; only the requested slices come back to the host.
    ``device`` is where the collective buffers live: the current CUDA device for NCCL (the
    default), the CPU for gloo.
    """
    import torch.distributed as td

    world = td.get_world_size(group) if td.is_initialized() else 1
    if world == 1:
        return [bytes(update)]
    if device is None:
        nccl = td.get_backend(group) == "nccl"
        device = torch.device("cuda", torch.cuda.current_device()) if nccl else torch.device("cpu")
    n = torch.tensor([len(update)], dtype=torch.int64, device=device)
    sizes_t = [torch.zeros_like(n) for _ in range(world)]
    td.all_gather(sizes_t, n, group=group)
    sizes = [int(s.item()) for s in sizes_t]
    mx = max(max(sizes), 1)
    buf = torch.zeros(mx, dtype=torch.uint8, device=device)
    if update:
        buf[: len(update)].copy_(torch.frombuffer(bytearray(update), dtype=torch.uint8))
    out = torch.empty(world * mx, dtype=torch.uint8, device=device)
    td.all_gather_into_tensor(out, buf, group=group)
    want = range(world) if ranks is None else ranks
    return [out[r * mx: r * mx + sizes[r]].cpu().numpy().tobytes() for r in want]


def allgather_updates_device(update, group=None, ranks: Sequence[int] | None = None) -> list:
    """allgather_updates for device-resident updates (uint8 CUDA tensors from
    encode_update_device): the sizes, then the padded updates, gathered into one device buffer
    over NCCL; returns device views of the requested ranks' updates, ready for apply_update."""
    import torch.distributed as td

    world = td.get_world_size(group) if td.is_initialized() else 1
    if world == 1:
        return [update]
    device = update.device
    n = torch.tensor([update.numel()], dtype=torch.int64, device=device)
    sizes_t = torch.empty(world, dtype=torch.int64, device=device)
    td.all_gather_into_tensor(sizes_t, n, group=group)
    sizes = sizes_t.tolist()
    mx = max(max(sizes), 1)
    buf = torch.zeros(mx, dtype=torch.uint8, device=device)
    buf[: update.numel()].copy_(update)
    out = torch.empty(world * mx, dtype=torch.uint8, device=device)
    td.all_gather_into_tensor(out, buf, group=group)
    want = range(world) if ranks is None else ranks
    return [out[r * mx: r * mx + sizes[r]] for r in want]
