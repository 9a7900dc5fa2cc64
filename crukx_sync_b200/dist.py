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


def host_size_group():
    """A gloo group over the same ranks, for the update sizes: the sizes are known on the host as
    soon as encode_update_device returns, so exchanging them there never waits for the GPU."""
    import torch.distributed as td
    return td.new_group(backend="gloo")


def allgather_updates_device(update, group=None, ranks: Sequence[int] | None = None, size_group=None) -> list:
    """allgather_updates for device-resident updates (uint8 CUDA tensors from
    encode_update_device): every rank's size, then the updates padded to the largest, gathered into
    one device buffer over NCCL; returns device views of the requested ranks' updates, ready for
    apply_update.  With ``size_group`` (a gloo group, see host_size_group) the sizes are exchanged
    between the hosts, so nothing waits for the device; otherwise they take a small NCCL gather
    that the host reads back."""
    import torch.distributed as td

    world = td.get_world_size(group) if td.is_initialized() else 1
    if world == 1:
        return [update]
    device = update.device
    if size_group is not None:
        n = torch.tensor([update.numel()], dtype=torch.int64)
        sizes_t = torch.empty(world, dtype=torch.int64)
        td.all_gather_into_tensor(sizes_t, n, group=size_group)
    else:
        n = torch.tensor([update.numel()], dtype=torch.int64, device=device)
        sizes_t = torch.empty(world, dtype=torch.int64, device=device)
        td.all_gather_into_tensor(sizes_t, n, group=group)
    sizes = sizes_t.tolist()
    mx = max(max(sizes), 1)
    if update.numel() == mx:
        buf = update
    else:
        buf = torch.empty(mx, dtype=torch.uint8, device=device)
        buf[: update.numel()].copy_(update)
        buf[update.numel():].zero_()
    out = torch.empty(world * mx, dtype=torch.uint8, device=device)
    td.all_gather_into_tensor(out, buf, group=group)
    want = range(world) if ranks is None else ranks
    return [out[r * mx: r * mx + sizes[r]] for r in want]


class PendingGather:
    """An all-gather of device updates in flight on a side stream (allgather_updates_device_async).
    views() are valid for work ordered after wait(); wait() makes the caller's current stream (or
    `stream`) wait for the gather."""

    def __init__(self, out, sizes, mx, event):
        self.out, self.sizes, self.mx, self.event = out, sizes, mx, event

    def views(self, ranks: Sequence[int] | None = None) -> list:
        want = range(len(self.sizes)) if ranks is None else ranks
        return [self.out[r * self.mx: r * self.mx + self.sizes[r]] for r in want]

    def wait(self, stream=None):
        if self.event is not None:
            (stream or torch.cuda.current_stream(self.out.device)).wait_event(self.event)


def allgather_updates_device_async(update, group=None, size_group=None, side_stream=None) -> PendingGather:
    """allgather_updates_device that does not hold up the caller's stream: the sizes go between
    the hosts first (size_group, a gloo group: nothing waits for the device), then the NCCL gather
    runs on `side_stream` after the work already queued on the current stream (the encode that
    produced `update`), so the caller can go on -- e.g. apply its own update, which it holds
    locally -- while the updates cross NVLink."""
    import torch.distributed as td

    world = td.get_world_size(group) if td.is_initialized() else 1
    if world == 1 or update.device.type != "cuda" or side_stream is None:
        views = allgather_updates_device(update, group=group, size_group=size_group)
        sizes = [v.numel() for v in views]
        mx = max(max(sizes), 1)
        out = torch.zeros(world * mx, dtype=torch.uint8, device=update.device)
        for r, v in enumerate(views):
            out[r * mx: r * mx + v.numel()].copy_(v)
        return PendingGather(out, sizes, mx, None)
    if size_group is not None:
        n = torch.tensor([update.numel()], dtype=torch.int64)
        sizes_t = torch.empty(world, dtype=torch.int64)
        td.all_gather_into_tensor(sizes_t, n, group=size_group)
    else:
        n = torch.tensor([update.numel()], dtype=torch.int64, device=update.device)
        sizes_t = torch.empty(world, dtype=torch.int64, device=update.device)
        td.all_gather_into_tensor(sizes_t, n, group=group)
    sizes = sizes_t.tolist()
    mx = max(max(sizes), 1)
    main = torch.cuda.current_stream(update.device)
    side_stream.wait_stream(main)
    with torch.cuda.stream(side_stream):
        if update.numel() == mx:
            buf = update
        else:
            buf = torch.empty(mx, dtype=torch.uint8, device=update.device)
            buf[: update.numel()].copy_(update)
            buf[update.numel():].zero_()
        out = torch.empty(world * mx, dtype=torch.uint8, device=update.device)
        td.all_gather_into_tensor(out, buf, group=group)
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(side_stream)
    update.record_stream(side_stream)
    return PendingGather(out, sizes, mx, ev)


def partition_contiguous(numels: Sequence[int], world: int) -> list[tuple[int, int]]:
    """Split tensors 0..n-1 (update order) into `world` contiguous ranges of about equal elements;
    range r = (first, end) for rank r (possibly empty)."""
    if world < 1:
        raise ValueError(f"world size must be >= 1, got {world}")
    total = sum(int(x) for x in numels)
    bounds, acc, r = [0], 0, 1
    for i, x in enumerate(numels):
        acc += int(x)
        while r < world and acc * world >= r * total and i + 1 > bounds[-1]:
            bounds.append(i + 1)
            r += 1
    while len(bounds) < world:
        bounds.append(len(numels))
    bounds.append(len(numels))
    return [(bounds[k], bounds[k + 1]) for k in range(world)]


_PART_KEYS = ("prefix", "tensors", "table", "payload")


def _pack_part(p: dict) -> bytes:
    import struct
    head = struct.pack("<6Q", *[len(p[k]) for k in _PART_KEYS], p["bit_offset"], p["total_bits"])
    return head + b"".join(p[k] for k in _PART_KEYS)


def _unpack_part(b: bytes) -> dict:
    import struct
    lens = struct.unpack_from("<6Q", b, 0)
    out, o = {}, 48
    for k, n in zip(_PART_KEYS, lens[:4]):
        out[k] = bytes(b[o: o + n])
        o += n
    out["bit_offset"], out["total_bits"] = lens[4], lens[5]
    return out


def encode_update_global(old, new, checksums: dict | None = None, group=None) -> bytes:
    """One update for the whole model, encoded by every rank of the group together: the bytes are
    identical to a single-GPU encode_update of all ranks' tensors in rank order.  `old`/`new` hold
    this rank's tensors, which must be its contiguous range of the update's tensor order (see
    partition_contiguous).  Every rank returns the whole update; the sender cache gets this rank's
    tensors.  Collectives: a 128 KiB histogram sum, small gathers, and the parts' all-gather."""
    import numpy as np
    import torch.distributed as td

    from . import codec
    from .wire import assemble

    if old.keys() != new.keys():
        raise ValueError(f"old and new differ in tensor names: {sorted(old.keys() ^ new.keys())[:5]}")
    world = td.get_world_size(group) if td.is_initialized() else 1
    rank = td.get_rank(group) if td.is_initialized() else 0
    nccl = td.is_initialized() and td.get_backend(group) == "nccl"
    cdev = torch.device("cuda", torch.cuda.current_device()) if nccl else torch.device("cpu")

    def sum_u64(arr):
        if world == 1:
            return
        t = torch.from_numpy(arr.view(np.int64).copy()).to(cdev)
        td.all_reduce(t, group=group)
        arr[:] = t.cpu().numpy().view(np.uint64)

    def allgather(mine: bytes) -> bytes:
        return b"".join(allgather_updates(mine, group=group, device=cdev)) if world > 1 else mine

    with torch.no_grad():
        enc = codec.encode_global(old, new, checksums, rank, world, sum_u64, allgather)
    part = enc.part()
    enc_checksums = enc.checksums
    enc.close()
    blobs = allgather_updates(_pack_part(part), group=group, device=cdev) if world > 1 else [_pack_part(part)]
    parts = [_unpack_part(b) for b in blobs]
    data = assemble(parts)
    if checksums is not None:
        checksums.update(enc_checksums)
    return data
