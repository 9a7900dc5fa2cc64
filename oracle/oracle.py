"""TEST INFRASTRUCTURE ONLY: Python face of the CPU oracle (crx_oracle.c).

The oracle is a sequential C restatement of crukx-sync's encode/apply path (wire format
version 2; src/crukx_sync/codec.py, src/crukx_sync/wire.py, docs/FORMAT.md of the reference).
Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use it, as
the checker or as the timed CPU baseline.  The product package never imports it.

The functions below mirror the reference's public API (src/crukx_sync/__init__.py:38-57):
``encode_update(old, new, checksums)`` and ``apply_update(weights, update, checksums)``, over
numpy int16 arrays or CPU torch tensors (bf16 or int16), with the same error classes
(``ValueError`` for caller mistakes, ``OracleCorrupt`` -- a ``ValueError`` -- for bad updates)
and the same cache rules (the receiver cache holds ``(checksum, version)`` pairs).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libcrx_oracle.so")
_lib = None


class OracleCorrupt(ValueError):
    """The oracle's CorruptUpdate: the update bytes are malformed or do not verify."""


def build() -> str:
    """Compile the oracle with its Makefile (gcc only); returns the library path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P, I64, U64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64
        L.orc_checksum.argtypes = [P, I64]
        L.orc_checksum.restype = U64
        L.orc_weight.argtypes = [U64]
        L.orc_weight.restype = U64
        L.orc_huffman_lengths.argtypes = [P, I64, P]
        L.orc_huffman_lengths.restype = ctypes.c_int
        L.orc_encode.argtypes = [ctypes.c_int, P, P, P, P, P, P, P, P, P, P, P, ctypes.c_char_p, ctypes.c_size_t]
        L.orc_encode.restype = ctypes.c_int
        L.orc_free.argtypes = [P]
        L.orc_parse.argtypes = [P, I64, ctypes.POINTER(P), ctypes.c_char_p, ctypes.c_size_t]
        L.orc_parse.restype = ctypes.c_int
        L.orc_update_n_tensors.argtypes = [P]
        L.orc_update_n_tensors.restype = I64
        L.orc_update_tensor.argtypes = [P, I64, P, P, P, P, P]
        L.orc_update_group.argtypes = [P, I64, ctypes.c_int, P, P, P]
        L.orc_update_free.argtypes = [P]
        L.orc_apply.argtypes = [P, P, P, P, P, ctypes.c_char_p, ctypes.c_size_t]
        L.orc_apply.restype = ctypes.c_int
        L.orc_set_threads.argtypes = [ctypes.c_int]
        L.orc_set_threads.restype = None
        _lib = L
    return _lib


def _bits(name, t) -> np.ndarray:
    """Flat int16 view (codec.py:35-41 rules: bf16 or int16, contiguous)."""
    try:
        import torch
        if isinstance(t, torch.Tensor):
            if t.dtype not in (torch.bfloat16, torch.int16):
                raise ValueError(f"{name}: expected a bfloat16 or int16 torch tensor, got {t.dtype}")
            if not t.is_contiguous():
                raise ValueError(f"{name}: tensor must be contiguous")
            if t.device.type != "cpu":
                raise ValueError(f"{name}: the oracle runs on CPU tensors only")
            return t.view(torch.int16).view(-1).numpy()
    except ImportError:
        pass
    a = np.asarray(t)
    if a.dtype != np.int16:
        raise ValueError(f"{name}: expected int16 bits, got {a.dtype}")
    if not a.flags.c_contiguous:
        raise ValueError(f"{name}: tensor must be contiguous")
    return a.reshape(-1)


def _version(t):
    return getattr(t, "_version", None)


def set_threads(n: int) -> None:
    """Threads of the oracle's per-tensor and per-exponent passes (0: every processor this process
    may run on, the default).  The bytes do not depend on it."""
    lib().orc_set_threads(int(n))


def checksum(a) -> int:
    a = np.ascontiguousarray(_bits("a", a))
    return int(lib().orc_checksum(a.ctypes.data, a.size))


def weight(i: int) -> int:
    return int(lib().orc_weight(i))


def huffman_lengths(counts) -> list[int]:
    c = np.ascontiguousarray(np.asarray(counts, dtype=np.uint64))
    out = np.zeros(c.size, dtype=np.int32)
    if lib().orc_huffman_lengths(c.ctypes.data, c.size, out.ctypes.data):
        raise MemoryError("oracle huffman_lengths failed")
    return out.tolist()


def encode_update(old, new, checksums: dict | None = None) -> bytes:
    """src/crukx_sync/__init__.py:38-48 over the C oracle."""
    if old.keys() != new.keys():
        raise ValueError("old and new differ in tensor names")
    names = list(old.keys())
    arrs = []
    for n in names:
        a, b = _bits(n, old[n]), _bits(n, new[n])
        if a.shape != b.shape:
            raise ValueError(f"{n}: old and new differ in shape")
        arrs.append((np.ascontiguousarray(a), np.ascontiguousarray(b)))
    k = len(names)
    prev = (ctypes.c_void_p * max(k, 1))(*[a.ctypes.data for a, _ in arrs])
    cur = (ctypes.c_void_p * max(k, 1))(*[b.ctypes.data for _, b in arrs])
    numel = np.array([a.size for a, _ in arrs] or [0], dtype=np.int64)
    raw = [n.encode() for n in names]
    cnames = (ctypes.c_char_p * max(k, 1))(*raw)
    nlen = np.array([len(r) for r in raw] or [0], dtype=np.int64)
    cache = np.array([(checksums or {}).get(n, 0) for n in names] or [0], dtype=np.uint64)
    has = np.array([1 if checksums is not None and n in checksums else 0 for n in names] or [0], dtype=np.uint8)
    new_chk = np.zeros(max(k, 1), dtype=np.uint64)
    present = np.zeros(max(k, 1), dtype=np.uint8)
    out = ctypes.c_void_p()
    out_len = ctypes.c_size_t()
    err = ctypes.create_string_buffer(256)
    st = lib().orc_encode(k, prev, cur, numel.ctypes.data, cnames, nlen.ctypes.data,
                          cache.ctypes.data, has.ctypes.data, ctypes.byref(out), ctypes.byref(out_len),
                          new_chk.ctypes.data, present.ctypes.data, err, 256)
    if st != 0:
        raise (ValueError if st == 1 else MemoryError)(err.value.decode())
    data = ctypes.string_at(out, out_len.value)
    lib().orc_free(out)
    if checksums is not None:
        checksums.update({n: int(new_chk[i]) for i, n in enumerate(names) if present[i]})
    return data


@dataclass
class Group:
    exponent: int
    count: int
    rice_r: int


@dataclass
class TensorHeader:
    name: str
    numel: int
    checksum: int
    groups: list


class _Parsed:
    def __init__(self, data: bytes):
        self._buf = ctypes.create_string_buffer(bytes(data), len(data) or 1)
        self.h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(256)
        st = lib().orc_parse(ctypes.addressof(self._buf), len(data), ctypes.byref(self.h), err, 256)
        if st == 2:
            raise OracleCorrupt(err.value.decode())
        if st != 0:
            raise MemoryError(err.value.decode())
        self.tensors = []
        for t in range(lib().orc_update_n_tensors(self.h)):
            p, nl, ne, ck, ng = ctypes.c_void_p(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_uint64(), ctypes.c_int()
            lib().orc_update_tensor(self.h, t, ctypes.byref(p), ctypes.byref(nl), ctypes.byref(ne),
                                    ctypes.byref(ck), ctypes.byref(ng))
            name = ctypes.string_at(p, nl.value).decode("utf-8")
            groups = []
            for g in range(ng.value):
                e, c, r = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int()
                lib().orc_update_group(self.h, t, g, ctypes.byref(e), ctypes.byref(c), ctypes.byref(r))
                groups.append(Group(e.value, c.value, r.value))
            self.tensors.append(TensorHeader(name, ne.value, ck.value, groups))

    def __del__(self):
        try:
            if getattr(self, "h", None) and self.h.value:
                lib().orc_update_free(self.h)
        except TypeError:   # interpreter shutdown: module globals already cleared
            pass


def parse(data: bytes) -> _Parsed:
    """wire.parse (wire.py:126-212): raises OracleCorrupt on any limit."""
    return _Parsed(data)


@dataclass
class UpdateStats:
    tensors: int
    changed: int
    bytes: int


def apply_update(weights, update: bytes, checksums: dict | None = None) -> UpdateStats:
    """src/crukx_sync/__init__.py:51-57 + codec.apply (codec.py:578-717) over the C oracle."""
    u = parse(update)
    if not u.tensors:
        return UpdateStats(0, 0, len(update))
    arrs = []
    for h in u.tensors:
        if h.name not in weights:
            raise ValueError(f"update has tensor {h.name!r} that the receiver does not have")
        a = _bits(h.name, weights[h.name])
        if a.size != h.numel:
            raise ValueError(f"{h.name}: update is for {h.numel} elements, receiver has {a.size}")
        if not a.flags.writeable:
            raise ValueError(f"{h.name}: read-only")
        arrs.append(a)
    k = len(arrs)
    ptrs = (ctypes.c_void_p * k)(*[a.ctypes.data for a in arrs])
    old = np.zeros(k, dtype=np.uint64)
    has = np.zeros(k, dtype=np.uint8)
    for i, h in enumerate(u.tensors):
        hit = checksums.get(h.name) if checksums is not None else None
        if isinstance(hit, tuple) and hit[1] == _version(weights[h.name]):
            old[i], has[i] = hit[0], 1
    changed = ctypes.c_int64()
    err = ctypes.create_string_buffer(256)
    st = lib().orc_apply(u.h, ptrs, old.ctypes.data, has.ctypes.data, ctypes.byref(changed), err, 256)
    if st == 2:
        raise OracleCorrupt(err.value.decode())
    if st != 0:
        raise MemoryError(err.value.decode())
    for h in u.tensors:   # the write went through raw memory: move the version like an in-place op
        t = weights[h.name]
        try:
            import torch
            if isinstance(t, torch.Tensor):
                torch.autograd.graph.increment_version(t)
        except ImportError:
            pass
    if checksums is not None:
        checksums.update({h.name: (h.checksum, _version(weights[h.name])) for h in u.tensors})
    return UpdateStats(len(u.tensors), changed.value, len(update))
