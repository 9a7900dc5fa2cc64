"""TEST INFRASTRUCTURE ONLY: the raw, sparserl and ctxfree sizes of the reference's size comparison
(bench/compare.py:56-100 of crukx-sync), restated element by element with numpy.  Pinned by
tests/golden/sizes.json (made by running the reference); checks crukx_sync_b200.sizes.

For every tensor, the changed positions i (ascending) define per change a delta (i minus the
previous change's position; the first change's delta is its position) and a gap (the delta minus
one; the first change's gap is its position).  Then over all changes of all tensors:
  raw      = 6 bytes per change
  sparserl = 2 bytes per change + 4 per delta above 0xFFFF + the new values at their entropy
  ctxfree  = the gaps' bit lengths at their entropy + the bits below each gap's leading one,
             rounded down to bytes + the old ^ new values at their entropy
where "at their entropy" is ceil(count * H / 8) bytes with H the order-0 entropy of the values.
"""

from __future__ import annotations

import numpy as np


def _bits(t) -> np.ndarray:
    try:
        import torch
        if isinstance(t, torch.Tensor):
            return t.contiguous().view(torch.int16).reshape(-1).cpu().numpy()
    except ImportError:
        pass
    return np.asarray(t).reshape(-1).view(np.int16)


def _entropy_bytes(values: np.ndarray) -> int:
    _, counts = np.unique(values, return_counts=True)
    q = counts / values.size
    return int(np.ceil(-(q * np.log2(q)).sum() * values.size / 8))


def update_sizes(old, new) -> dict:
    pos_delta, gaps, news, xors = [], [], [], []
    for name in old:
        a, b = _bits(old[name]), _bits(new[name])
        idx = np.flatnonzero(a != b).astype(np.int64)
        if idx.size == 0:
            continue
        prev = np.concatenate(([-1], idx[:-1]))
        g = idx - prev - 1
        d = g + 1
        d[0] = idx[0]
        pos_delta.append(d)
        gaps.append(g)
        news.append(b[idx].view(np.uint16))
        xors.append((a[idx] ^ b[idx]).view(np.uint16))
    if not gaps:
        return {"raw": 0, "sparserl": 0, "ctxfree": 0}
    d, g = np.concatenate(pos_delta), np.concatenate(gaps)
    n = g.size
    lengths = np.array([int(x).bit_length() for x in g], dtype=np.int64) if n < 1000 else \
        np.where(g > 0, np.floor(np.log2(np.maximum(g, 1).astype(np.float64))).astype(np.int64) + 1, 0)
    sparserl = 2 * n + 4 * int((d > 0xFFFF).sum()) + _entropy_bytes(np.concatenate(news))
    ctxfree = _entropy_bytes(lengths) + int(np.maximum(lengths - 1, 0).sum()) // 8 + _entropy_bytes(np.concatenate(xors))
    return {"raw": 6 * n, "sparserl": sparserl, "ctxfree": ctxfree}
