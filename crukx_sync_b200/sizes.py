"""Size of the same update in other sparse formats, beside crukx-sync's own: the raw, sparserl and
ctxfree columns of the reference's size comparison (bench/compare.py:56-100 of crukx-sync).

    sizes = update_sizes(old, new)   # {"raw": ..., "sparserl": ..., "ctxfree": ...} in bytes

  raw       int32 position + bf16 value per change (6 B per change)
  sparserl  16-bit position deltas (4 more bytes where a delta needs more than 16 bits) + the new
            values at their order-0 entropy
  ctxfree   gaps coded by bit length (the lengths at their order-0 entropy, the bits below the
            leading one raw) + the old ^ new values at their order-0 entropy

The per-change work runs on the GPU (crx_size_stats: one pass over old and new, histograms of the
new values, the xor values and the gaps' bit lengths); the sizes follow here from the histograms
with the reference's formulas, in the reference's summation order.  The reference's nemo and pulse
columns compress with zstd and its arcv3 column calls a separate package; neither is computed.
"""

from __future__ import annotations

import ctypes
from collections.abc import Mapping

import numpy as np
import torch

from . import _ext, codec

STATS_WORDS = 3 + 64 + 2 * 65536
_VAL, _XOR = 3 + 64, 3 + 64 + 65536


def _entropy_bytes(counts: np.ndarray, n: int) -> int:
    """ceil(n * H / 8) for the order-0 entropy H of a histogram (bins ascending, empty ones left
    out), as compare.py computes it from np.unique / np.bincount counts."""
    c = counts[counts > 0].astype(np.int64)
    q = c / n
    return int(np.ceil(-(q * np.log2(q)).sum() * n / 8))


def sizes_from_stats(stats) -> dict:
    """The three sizes from crx_size_stats' words."""
    st = np.asarray(stats, dtype=np.uint64)
    n = int(st[0])
    if n == 0:
        return {"raw": 0, "sparserl": 0, "ctxfree": 0}
    esc, mant = int(st[1]), int(st[2])
    sparserl = 2 * n + 4 * esc + _entropy_bytes(st[_VAL:_VAL + 65536], n)
    gap_bytes = _entropy_bytes(st[3:3 + 64], n) + mant // 8
    ctxfree = gap_bytes + _entropy_bytes(st[_XOR:_XOR + 65536], n)
    return {"raw": 6 * n, "sparserl": sparserl, "ctxfree": ctxfree}


def size_stats(old: Mapping[str, torch.Tensor], new: Mapping[str, torch.Tensor]) -> np.ndarray:
    """crx_size_stats over the dicts (same names and sizes, bf16 or int16, one device)."""
    if old.keys() != new.keys():
        raise ValueError(f"old and new differ in tensor names: {sorted(old.keys() ^ new.keys())[:5]}")
    names = list(old)
    olds, news = [old[k] for k in names], [new[k] for k in names]
    for name, a, b in zip(names, olds, news):
        codec.check16(name, a)
        codec.check16(name, b)
        if a.numel() != b.numel():
            raise ValueError(f"{name}: old and new differ in shape")
    out = np.zeros(STATS_WORDS, dtype=np.uint64)
    if not names:
        return out
    devs = {t.device for t in olds} | {t.device for t in news}
    if len(devs) != 1:
        raise ValueError("all tensors must be on one device")
    dev = next(iter(devs))
    cdev = codec._cuda_device(dev)
    if dev.type != "cuda":
        olds = [a.to(cdev) for a in olds]
        news = [b.to(cdev) for b in news]
    L = _ext.load()
    err = ctypes.create_string_buffer(512)
    with torch.cuda.device(cdev):
        stream = torch.cuda.current_stream(cdev).cuda_stream
        st = L.crx_size_stats(_ext.context(cdev.index), len(names), _ext.ptr_array([a.data_ptr() for a in olds]),
                              _ext.ptr_array([b.data_ptr() for b in news]), _ext.CBuf("q", [a.numel() for a in olds]),
                              ctypes.c_void_p(stream), ctypes.c_void_p(out.ctypes.data), err, 512)
    if st != _ext.CRX_OK:
        codec._raise(st, err)
    return out


def update_sizes(old: Mapping[str, torch.Tensor], new: Mapping[str, torch.Tensor]) -> dict:
    """Bytes the raw, sparserl and ctxfree formats need for the update old -> new."""
    return sizes_from_stats(size_stats(old, new))
