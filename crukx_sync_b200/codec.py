"""Torch-facing side of encode/apply: argument checks with the reference's error rules, device
placement, checksum caches, and the calls into the CUDA library.

Reference behaviour kept (paths relative to the crukx-sync project):
  bits16 rules (dtype bf16/int16, contiguous)            src/crukx_sync/codec.py:35-41
  same names/shapes, one device                          codec.py:284-293, __init__.py:41-42
  sender cache: cached + delta, else a full checksum     codec.py:344-352
  receiver checks (name, numel) before anything else     codec.py:582-592
  receiver cache trusted only while _version unchanged   codec.py:457-460, 702-705, 715-716
CPU tensors are accepted the way the reference accepts them, but the work always runs on a CUDA
device: they are copied to the current CUDA device and, on apply, the result is copied back in
place.  Without a CUDA device these functions raise; there is no CPU implementation here.
"""

from __future__ import annotations

import ctypes
import os
import sys
import time
from collections.abc import Mapping

import torch

from . import _ext
from .wire import CorruptUpdate, EncodedUpdate, ParsedUpdate


_TRACE = bool(os.environ.get("CRUKX_B200_TRACE"))


def _trace(what: str, t0: float) -> None:
    if _TRACE:
        print(f"[crx-py] {what:<28} {1e3 * (time.perf_counter() - t0):9.3f} ms", file=sys.stderr, flush=True)


_BITS16 = (torch.bfloat16, torch.int16)


def check16(name: str, t) -> None:
    """The bits16 rules without building a view: bf16 or int16, contiguous."""
    if not isinstance(t, torch.Tensor) or t.dtype not in _BITS16:
        raise ValueError(f"{name}: expected a bfloat16 or int16 torch tensor, got {getattr(t, 'dtype', type(t))}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: tensor must be contiguous")


def bits16(name: str, t) -> torch.Tensor:
    """Flat int16 view of a bf16 (or int16 bit-pattern) tensor."""
    check16(name, t)
    return t.view(torch.int16).view(-1)


_NAME_TABLES: dict = {}   # the last few name lists (a model syncs the same names every step)


def _name_table(names):
    """UTF-8 names as one buffer: (keep-alive, pointer array, length array)."""
    key = tuple(names)
    hit = _NAME_TABLES.get(key)
    if hit is not None:
        return hit
    raw = [n.encode("utf-8") for n in names]
    blob = b"".join(raw) + b"\0"
    base = ctypes.cast(ctypes.c_char_p(blob), ctypes.c_void_p).value
    ptrs, lens, off = [], [], 0
    for r in raw:
        ptrs.append(base + off)
        lens.append(len(r))
        off += len(r)
    out = (blob, _ext.CBuf("Q", ptrs), _ext.CBuf("q", lens))
    if len(_NAME_TABLES) >= 8:
        _NAME_TABLES.clear()
    _NAME_TABLES[key] = out
    return out


def _cuda_device(dev: torch.device) -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("crukx_sync_b200 runs on CUDA (sm_100a) only and no CUDA device is available")
    if dev.type == "cuda":
        return dev if dev.index is not None else torch.device("cuda", torch.cuda.current_device())
    return torch.device("cuda", torch.cuda.current_device())


def _raise(status: int, err) -> None:
    msg = err.value.decode(errors="replace")
    if status == _ext.CRX_CORRUPT:
        raise CorruptUpdate(msg)
    if status == _ext.CRX_VALUE_ERROR:
        raise ValueError(msg)
    if status == _ext.CRX_NO_MEMORY:
        raise MemoryError(msg)
    raise RuntimeError(f"crukx_sync_b200: status {status}: {msg}")


def encode(old: Mapping[str, torch.Tensor], new: Mapping[str, torch.Tensor],
           checksums: dict | None = None, device_result: bool = False) -> EncodedUpdate:
    """The encoded update (not yet bytes); ``.checksums`` holds what the sender cache commits."""
    names = list(old)
    olds, news, numels, devs = [], [], [], set()
    T = torch.Tensor
    for name in names:     # the reference's order of checks (check16 inlined); one pass per tensor
        a = old[name]
        b = new[name]
        if not isinstance(a, T) or a.dtype not in _BITS16 or not a.is_contiguous():
            check16(name, a)
        if not isinstance(b, T) or b.dtype not in _BITS16 or not b.is_contiguous():
            check16(name, b)
        n = a.numel()
        if n != b.numel():
            raise ValueError(f"{name}: old and new differ in shape")
        olds.append(a)
        news.append(b)
        numels.append(n)
        devs.add(a.get_device())
        devs.add(b.get_device())
    if not names:
        return _encode_on(torch.device("cpu"), [], [], [], None, device_result)
    if len(devs) > 1:
        raise ValueError("all tensors must be on one device")
    return _encode_on(olds[0].device, names, olds, news, checksums, device_result, numels)


def _encode_on(dev, names, olds, news, checksums, device_result=False, numels=None) -> EncodedUpdate:
    cdev = _cuda_device(dev)
    if dev.type != "cuda":
        olds = [a.to(cdev) for a in olds]
        news = [b.to(cdev) for b in news]
    L = _ext.load()
    k = len(names)
    prev = _ext.ptr_array([a.data_ptr() for a in olds])
    cur = _ext.ptr_array([b.data_ptr() for b in news])
    numel = _ext.CBuf("q", numels if numels is not None else [a.numel() for a in olds])
    keep, name_ptrs, name_len = _name_table(names)
    if checksums:
        hits = [checksums.get(n) for n in names]
        cache = _ext.CBuf("Q", [int(c) & (2**64 - 1) if c is not None else 0 for c in hits])
        has = _ext.CBuf("B", [c is not None for c in hits])
    else:
        cache, has = None, None
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(1024)
    with torch.cuda.device(cdev):
        stream = torch.cuda.current_stream(cdev).cuda_stream
        fn = L.crx_encode_device if device_result else L.crx_encode
        st = fn(_ext.context(cdev.index), k, prev, cur, numel, name_ptrs, name_len, cache, has,
                ctypes.c_void_p(stream), ctypes.byref(h), err, 1024)
    del keep
    if st != _ext.CRX_OK:
        _raise(st, err)
    out = EncodedUpdate(h, names)
    out.device = cdev
    return out


def encode_global(old, new, checksums, rank: int, world: int, sum_u64, allgather, ctx=None) -> EncodedUpdate:
    """This rank's part of one update encoded by `world` ranks (crx_encode_global).

    sum_u64(values: numpy uint64 array) -> None sums in place over ranks; allgather(mine: bytes)
    -> bytes returns every rank's bytes concatenated in rank order.  Both are called on every
    rank in the same order.  The part's pieces come from EncodedUpdate.part()."""
    import numpy as np

    names = list(old)
    olds = [old[n] for n in names]
    news = [new[n] for n in names]
    for name, a, b in zip(names, olds, news):
        check16(name, a)
        check16(name, b)
        if a.numel() != b.numel():
            raise ValueError(f"{name}: old and new differ in shape")
    devs = {t.device for t in olds} | {t.device for t in news}
    if len(devs) > 1:
        raise ValueError("all tensors must be on one device")
    dev = next(iter(devs)) if devs else torch.device("cuda", torch.cuda.current_device())
    cdev = _cuda_device(dev)
    if dev.type != "cuda":
        olds = [a.to(cdev) for a in olds]
        news = [b.to(cdev) for b in news]
    L = _ext.load()
    k = len(names)
    prev = _ext.ptr_array([a.data_ptr() for a in olds])
    cur = _ext.ptr_array([b.data_ptr() for b in news])
    numel = _ext.CBuf("q", [a.numel() for a in olds])
    keep, name_ptrs, name_len = _name_table(names)
    if checksums:
        hits = [checksums.get(n) for n in names]
        cache = _ext.CBuf("Q", [int(c) & (2**64 - 1) if c is not None else 0 for c in hits])
        has = _ext.CBuf("B", [c is not None for c in hits])
    else:
        cache, has = None, None
    held = []   # gathered buffers stay alive until the call returns

    def _sum(user, data, n):
        try:
            arr = np.ctypeslib.as_array(data, shape=(n,)) if n else np.zeros(0, dtype=np.uint64)
            sum_u64(arr)
            return 0
        except Exception as exc:   # the C side turns a non-zero status into an error
            held.append(exc)
            return 1

    def _gather(user, mine, n, all_p, all_len):
        try:
            out = allgather(ctypes.string_at(mine, n) if n else b"")
            buf = ctypes.create_string_buffer(out, max(len(out), 1))
            held.append(buf)
            all_p[0] = ctypes.addressof(buf)
            all_len[0] = len(out)
            return 0
        except Exception as exc:
            held.append(exc)
            return 1

    sum_cb, gather_cb = _ext.SUM_U64_FN(_sum), _ext.ALLGATHER_FN(_gather)
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(1024)
    with torch.cuda.device(cdev):
        stream = torch.cuda.current_stream(cdev).cuda_stream
        st = L.crx_encode_global(ctx if ctx is not None else _ext.context(cdev.index), k, prev, cur, numel, name_ptrs,
                                 name_len, cache, has, ctypes.c_void_p(stream), int(rank), int(world), sum_cb, gather_cb,
                                 None, ctypes.byref(h), err, 1024)
    del keep
    errors = [x for x in held if isinstance(x, Exception)]
    if errors:
        raise RuntimeError(f"crukx_sync_b200: a collective failed: {errors[0]!r}") from errors[0]
    if st != _ext.CRX_OK:
        _raise(st, err)
    out = EncodedUpdate(h, names)
    out.device = cdev
    return out


def _cache_get(checksums, name, t):
    """A cached checksum, trusted only if the tensor was not modified since it was recorded."""
    hit = checksums.get(name) if checksums is not None else None
    return hit[0] if isinstance(hit, tuple) and hit[1] == t._version else None


def apply(weights: Mapping[str, torch.Tensor], u: ParsedUpdate, checksums: dict | None = None) -> int:
    """Verify ``u`` against ``weights``, then write the new values in place; returns changes."""
    headers = u.tensor_table()
    if not headers:
        return 0
    # one pass per tensor (check16 and the cache lookup inlined: this runs once per tensor per apply)
    targets, vers, cvals, hits = [], [], [], []
    di = None
    for name, numel, _ in headers:
        if name not in weights:
            raise ValueError(f"update has tensor {name!r} that the receiver does not have")
        a = weights[name]
        if not isinstance(a, torch.Tensor) or a.dtype not in _BITS16 or not a.is_contiguous():
            check16(name, a)
        if a.numel() != numel:
            raise ValueError(f"{name}: update is for {numel} elements, receiver has {a.numel()}")
        d = a.get_device()
        if di is None:
            di = d
        elif d != di:
            raise ValueError("all updated tensors must be on one device")
        v = a._version
        targets.append(a)
        vers.append(v)
        if checksums:   # a cached checksum is trusted only while the tensor's version is the recorded one
            hit = checksums.get(name)
            ok = isinstance(hit, tuple) and hit[1] == v and hit[0] is not None
            cvals.append(hit[0] if ok else 0)
            hits.append(ok)
    dev = targets[0].device
    cdev = _cuda_device(dev)
    work = targets if dev.type == "cuda" else [a.to(cdev) for a in targets]
    k = len(headers)
    if checksums:
        cache = _ext.CBuf("Q", cvals)
        has = _ext.CBuf("B", hits)
    else:
        cache, has = None, None
    ptrs = _ext.ptr_array([a.data_ptr() for a in work])
    changed = ctypes.c_int64()
    err = ctypes.create_string_buffer(1024)
    L = _ext.load()
    with torch.cuda.device(cdev):
        stream = torch.cuda.current_stream(cdev).cuda_stream
        if dev.type == "cuda" and checksums is not None:
            # tensors written in place on the device: the library may keep their exponent
            # histograms for the next apply, tagged with the version they will have after it
            vtab = _ext.CBuf("Q", vers)
            tag = _ext.CBuf("B", bytes([1]) * k)
            st = L.crx_apply_versioned(_ext.context(cdev.index), u.handle, ptrs, cache, has, vtab, tag,
                                       ctypes.c_void_p(stream), ctypes.byref(changed), err, 1024)
        elif dev.type == "cuda":
            st = L.crx_apply(_ext.context(cdev.index), u.handle, ptrs, cache, has, ctypes.c_void_p(stream),
                             ctypes.byref(changed), err, 1024)
        else:   # host weights: verified against the device copies, only the changed elements written back
            hptrs = _ext.ptr_array([a.data_ptr() for a in targets])
            st = L.crx_apply_to_host(_ext.context(cdev.index), u.handle, ptrs, hptrs, cache, has,
                                     ctypes.c_void_p(stream), ctypes.byref(changed), err, 1024)
    if st != _ext.CRX_OK:
        _raise(st, err)
    # the commit wrote through raw pointers (device or host): move the version like a[idx] = v
    torch.autograd.graph.increment_version(targets)
    if checksums is not None:   # record the version after our own write
        checksums.update({name: (chk, a._version) for (name, _, chk), a in zip(headers, targets)})
    return int(changed.value)


def checksum(t: torch.Tensor) -> int:
    """sum(u_i * w_i) mod 2^64 over the uint16 bits u_i, computed on the GPU."""
    a = bits16("tensor", t)
    cdev = _cuda_device(a.device)
    if a.device.type != "cuda":
        a = a.to(cdev)
    out = ctypes.c_uint64()
    err = ctypes.create_string_buffer(512)
    with torch.cuda.device(cdev):
        stream = torch.cuda.current_stream(cdev).cuda_stream
        st = _ext.load().crx_checksum(_ext.context(cdev.index), ctypes.c_void_p(a.data_ptr()), a.numel(),
                                      ctypes.c_void_p(stream), ctypes.byref(out), err, 512)
    if st != _ext.CRX_OK:
        _raise(st, err)
    return int(out.value)
