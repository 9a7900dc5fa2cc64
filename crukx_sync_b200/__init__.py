"""crukx_sync_b200: exact, compact bf16 weight updates for RL weight sync, on B200 (sm_100a).

    update = encode_update(prev, cur)   # trainer: dicts of name -> bf16 torch tensors
    apply_update(weights, update)       # worker: writes the new values into `weights` in place

A drop-in for crukx-sync's public API (src/crukx_sync/__init__.py:28-57 of the reference):
same signatures, same wire format (version 2, byte-identical updates), same all-or-nothing
``CorruptUpdate`` semantics and the same checksum-cache rules:
- Sender: ``checksums`` maps name -> checksum of the last `cur`; it is updated only once the
  update exists, and a wrong cache produces an update the receiver rejects, never wrong weights.
- Receiver: ``checksums`` maps name -> (checksum, tensor._version); a cached checksum is used
  only while the tensor's ``_version`` is unchanged since this library last wrote it.
All arithmetic runs in hand-written CUDA kernels (libcrukx_b200.so, C ABI in
include/crukx_b200.h); there is no CPU implementation and no other backend.
"""

from __future__ import annotations

import time
from collections.abc import Mapping
from dataclasses import dataclass

import torch

from . import codec
from .wire import CorruptUpdate, encoder_parse, parse, parse_device, serialize

__all__ = ["encode_update", "apply_update", "encode_update_device", "UpdateStats", "CorruptUpdate"]


@dataclass
class UpdateStats:
    tensors: int
    changed: int
    bytes: int


def encode_update(old: Mapping[str, torch.Tensor], new: Mapping[str, torch.Tensor],
                  checksums: dict | None = None) -> bytes:
    """Bytes that turn `old` into `new` exactly. Same names and shapes; tensors are bf16 or int16."""
    if old.keys() != new.keys():
        raise ValueError(f"old and new differ in tensor names: {sorted(old.keys() ^ new.keys())[:5]}")
    t0 = time.perf_counter()
    with torch.no_grad():
        update = codec.encode(old, new, checksums)
    codec._trace("encode (C-ABI call)", t0)
    t1 = time.perf_counter()
    data = serialize(update)
    codec._trace("serialize to bytes", t1)
    if checksums is not None:  # commit only once the update exists
        checksums.update(update.checksums)
    return data


def encode_update_device(old: Mapping[str, torch.Tensor], new: Mapping[str, torch.Tensor],
                         checksums: dict | None = None) -> torch.Tensor:
    """encode_update whose result stays in device memory: a uint8 CUDA tensor holding exactly the
    bytes encode_update returns, on the tensors' device (CPU tensors: the current CUDA device).
    For transports that move updates between GPUs (NCCL, NVLink) without a host round trip.
    Like any CUDA result, the bytes are written in the order of the current stream: work queued
    after this call on that stream sees them; another stream must wait for it first.  The tensor
    carries the encoder's own parse, which apply_update uses while the tensor is unmodified.
    The sender cache follows the same rule: it is updated only once the update exists."""
    if old.keys() != new.keys():
        raise ValueError(f"old and new differ in tensor names: {sorted(old.keys() ^ new.keys())[:5]}")
    with torch.no_grad():
        update = codec.encode(old, new, checksums, device_result=True)
        dev = getattr(update, "device", None)
        if dev is None or dev.type != "cuda":
            dev = torch.device("cuda", torch.cuda.current_device())
        data = update.to_device(dev)
        pre = getattr(data, "_crx_parsed", None)
        if pre is not None:   # its tensor table is the present tensors, in the caller's order
            pre[0]._table = [(n, old[n].numel(), c) for n, c in update.checksums.items()]
    update.close()
    if checksums is not None:
        checksums.update(update.checksums)
    return data


def apply_update(weights: Mapping[str, torch.Tensor], update,
                 checksums: dict | None = None) -> UpdateStats:
    """Write the update into `weights` in place; on any error nothing is written.  `update` is the
    bytes encode_update returned, or (no reference counterpart) the uint8 CUDA tensor that
    encode_update_device returned, read where it lies."""
    t0 = time.perf_counter()
    if isinstance(update, torch.Tensor):
        # a device update from encode_update_device in this process comes with the encoder's parse:
        # no header copy down, so nothing waits for the encode to finish
        u = encoder_parse(update)
        if u is None:
            u = parse_device(update)
    else:
        u = parse(update)
    codec._trace("parse", t0)
    t1 = time.perf_counter()
    with torch.no_grad():
        changed = codec.apply(weights, u, checksums)
    codec._trace("apply (C-ABI call)", t1)
    return UpdateStats(u.n_tensors, changed, update.numel() if isinstance(update, torch.Tensor) else len(update))
