"""The update container (wire format version 2): types, constants, varint writer, and parsing.

Mirrors the reference module src/crukx_sync/wire.py (constants :8-13, ``CorruptUpdate`` :16-17,
dataclasses :20-48, ``write_varint`` :55-61, ``serialize`` :64-89, ``parse`` :126-212).  Parsing
and validation run in the C++ host code of libcrukx_b200.so (``crx_parse``); ``parse`` returns a
``ParsedUpdate`` that holds that handle and exposes the reference's dataclass view lazily.
"""

from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass, field

from . import _ext

MAGIC = b"CRXS"
VERSION = 2
MAX_CODE_LEN = 17
MAX_SYMBOL = 131070
MAX_RICE = 30
BLOCK = 256


class CorruptUpdate(ValueError):
    """The update bytes are malformed, truncated, or do not reproduce the expected weights."""


@dataclass
class Table:
    """Canonical Huffman table for residual symbols of one old-weight exponent."""
    exponent: int
    symbols: list[int]
    lengths: list[int]


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
    groups: list[Group]


@dataclass
class Update:
    tables: list[Table]
    tensors: list[TensorHeader]
    block_bits: list[int] = field(default_factory=list)
    payload: bytes = b""


def n_blocks(count: int) -> int:
    return -(-count // BLOCK)


def write_varint(out: bytearray, v: int) -> None:
    if not 0 <= v < 1 << 63:
        raise ValueError(f"varint out of range: {v}")
    while v >= 0x80:
        out.append((v & 0x7F) | 0x80)
        v >>= 7
    out.append(v)


def _serialize_update(u: Update) -> bytes:
    out = bytearray(MAGIC)
    out.append(VERSION)
    write_varint(out, len(u.tables))
    for t in u.tables:
        out.append(t.exponent)
        write_varint(out, len(t.symbols))
        for s, L in zip(t.symbols, t.lengths):
            write_varint(out, s)
            out.append(L)
    write_varint(out, len(u.tensors))
    for t in u.tensors:
        raw = t.name.encode()
        write_varint(out, len(raw))
        out += raw
        write_varint(out, t.numel)
        out += struct.pack("<Q", t.checksum)
        write_varint(out, len(t.groups))
        for g in t.groups:
            out.append(g.exponent)
            write_varint(out, g.count)
            out.append(g.rice_r)
    out += struct.pack(f"<{len(u.block_bits)}I", *u.block_bits)
    write_varint(out, len(u.payload))
    out += u.payload
    return bytes(out)


_PyBytes_FromStringAndSize = ctypes.pythonapi.PyBytes_FromStringAndSize
_PyBytes_FromStringAndSize.restype = ctypes.py_object
_PyBytes_FromStringAndSize.argtypes = [ctypes.c_void_p, ctypes.c_ssize_t]
_PyBytes_AsString = ctypes.pythonapi.PyBytes_AsString
_PyBytes_AsString.restype = ctypes.c_void_p
_PyBytes_AsString.argtypes = [ctypes.py_object]


class EncodedUpdate:
    """An update produced by the CUDA encoder, not yet serialized to ``bytes``."""

    def __init__(self, handle, names):
        self._h = handle
        self.names = names
        L = _ext.load()
        chk = (ctypes.c_uint64 * max(len(names), 1))()
        present = (ctypes.c_uint8 * max(len(names), 1))()
        L.crx_encoded_checksums(handle, chk, present)
        self.checksums = {n: int(chk[i]) for i, n in enumerate(names) if present[i]}
        self.changes = int(L.crx_encoded_changes(handle))

    def to_bytes(self) -> bytes:
        L = _ext.load()
        n = int(L.crx_encoded_size(self._h))
        out = _PyBytes_FromStringAndSize(None, n)   # a fresh bytes object, filled in place once
        if n and L.crx_encoded_copy(self._h, _PyBytes_AsString(out), n) != _ext.CRX_OK:
            raise RuntimeError("crukx_sync_b200: encoded update copy failed")
        return out

    def to_device(self, device, stream=None):
        """The serialized update as a uint8 tensor on `device` (a CUDA device): the same bytes as
        to_bytes(), written on the device without a host round trip of the payload."""
        import torch

        L = _ext.load()
        n = int(L.crx_encoded_size(self._h))
        out = torch.empty(n, dtype=torch.uint8, device=device)
        st = stream if stream is not None else torch.cuda.current_stream(out.device).cuda_stream
        if n and L.crx_encoded_copy_device(self._h, ctypes.c_void_p(out.data_ptr()), n, ctypes.c_void_p(st)) != _ext.CRX_OK:
            raise RuntimeError("crukx_sync_b200: encoded update device copy failed")
        if n:   # the encoder's own parse of these bytes, for apply_update while they stay unchanged
            h = ctypes.c_void_p()
            err = ctypes.create_string_buffer(256)
            if L.crx_encoded_parse_device(self._h, ctypes.c_void_p(out.data_ptr()), ctypes.byref(h), err, 256) == _ext.CRX_OK:
                out._crx_parsed = (ParsedUpdate(_handle=h), out._version, out.data_ptr(), n)
        return out

    def part(self) -> dict:
        """A rank's part of a global update: prefix, tensors, table and payload bytes, with the
        part's bit offset in the update's payload and the update's payload bits."""
        L = _ext.load()
        v = [ctypes.c_int64() for _ in range(4)] + [ctypes.c_uint64(), ctypes.c_uint64()]
        if L.crx_encoded_part(self._h, *[ctypes.byref(x) for x in v]) != _ext.CRX_OK:
            raise ValueError("not a part of a global update")
        bufs = [ctypes.create_string_buffer(max(int(x.value), 1)) for x in v[:4]]
        if L.crx_encoded_part_copy(self._h, *bufs) != _ext.CRX_OK:
            raise RuntimeError("crukx_sync_b200: part copy failed")
        keys = ("prefix", "tensors", "table", "payload")
        out = {k: b.raw[: int(x.value)] for k, b, x in zip(keys, bufs, v[:4])}
        out["bit_offset"], out["total_bits"] = int(v[4].value), int(v[5].value)
        return out

    def close(self):
        if self._h:
            _ext.load().crx_encoded_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def assemble(parts: list) -> bytes:
    """The update of a global encode from every rank's part, in rank order (see
    crx_encode_global): prefix + tensor headers + block tables + payload length + payloads, the
    parts' boundary bytes OR-ed together."""
    import numpy as np

    total_bits = parts[0]["total_bits"]
    pay = np.zeros((total_bits + 7) // 8, dtype=np.uint8)
    for p in parts:
        b = np.frombuffer(p["payload"], dtype=np.uint8)
        lo = p["bit_offset"] // 8
        if len(b):
            pay[lo: lo + len(b)] |= b[: len(pay) - lo]
    out = bytearray(parts[0]["prefix"])
    for p in parts:
        out += p["tensors"]
    for p in parts:
        out += p["table"]
    write_varint(out, len(pay))
    out += pay.tobytes()
    return bytes(out)


def serialize(u) -> bytes:
    """Bytes of an update: an EncodedUpdate from the CUDA encoder, or an Update dataclass."""
    if isinstance(u, EncodedUpdate):
        return u.to_bytes()
    return _serialize_update(u)


class ParsedUpdate:
    """A validated update (C handle).  Borrows ``data``; attribute views match wire.Update."""

    def __init__(self, data: bytes | None = None, *, _handle=None, _keep=None):
        self._tensors = None
        self._tables = None
        self._table = None
        if _handle is not None:   # made by parse_device / parse_head
            self._data = _keep
            self._h = _handle
            return
        L = _ext.load()
        self._data = data if isinstance(data, bytes) else bytes(data)
        self._h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        buf = ctypes.cast(ctypes.c_char_p(self._data), ctypes.c_void_p)
        st = L.crx_parse(buf, len(self._data), ctypes.byref(self._h), err, 512)
        if st == _ext.CRX_CORRUPT:
            raise CorruptUpdate(err.value.decode(errors="replace"))
        if st != _ext.CRX_OK:
            raise RuntimeError(f"crukx_sync_b200: parse failed ({st}): {err.value.decode(errors='replace')}")

    @property
    def handle(self):
        return self._h

    def tensor_table(self) -> list[tuple[str, int, int]]:
        """(name, numel, checksum) of every tensor, in update order, in one call."""
        if self._table is None:
            L = _ext.load()
            n = int(L.crx_update_n_tensors(self._h))
            names = (ctypes.c_void_p * max(n, 1))()
            lens = (ctypes.c_int64 * max(n, 1))()
            numels = (ctypes.c_int64 * max(n, 1))()
            chks = (ctypes.c_uint64 * max(n, 1))()
            L.crx_update_tensor_table(self._h, names, lens, numels, chks)
            if n == 0:
                self._table = []
            else:   # the names lie in one header buffer: one copy, then a slice per name
                ptrs, ls = names[:n], lens[:n]
                base = min(ptrs)
                blob = ctypes.string_at(base, max(q + k for q, k in zip(ptrs, ls)) - base)
                self._table = [(blob[q - base:q - base + k].decode("utf-8"), e, c)
                               for q, k, e, c in zip(ptrs, ls, numels[:n], chks[:n])]
        return self._table

    @property
    def n_tensors(self) -> int:
        return int(_ext.load().crx_update_n_tensors(self._h))

    @property
    def tensors(self) -> list[TensorHeader]:
        if self._tensors is None:
            L = _ext.load()
            out = []
            for t in range(int(L.crx_update_n_tensors(self._h))):
                p, nl, ne, ck, ng = (ctypes.c_void_p(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_uint64(),
                                     ctypes.c_int32())
                L.crx_update_tensor(self._h, t, ctypes.byref(p), ctypes.byref(nl), ctypes.byref(ne), ctypes.byref(ck),
                                    ctypes.byref(ng))
                name = ctypes.string_at(p, nl.value).decode("utf-8")
                groups = []
                for k in range(ng.value):
                    e, c, r = ctypes.c_int32(), ctypes.c_int64(), ctypes.c_int32()
                    L.crx_update_group(self._h, t, k, ctypes.byref(e), ctypes.byref(c), ctypes.byref(r))
                    groups.append(Group(e.value, c.value, r.value))
                out.append(TensorHeader(name, ne.value, ck.value, groups))
            self._tensors = out
        return self._tensors

    @property
    def tables(self) -> list[Table]:
        if self._tables is None:
            L = _ext.load()
            out = []
            for k in range(int(L.crx_update_n_tables(self._h))):
                e, n = ctypes.c_int32(), ctypes.c_int64()
                L.crx_update_table(self._h, k, ctypes.byref(e), ctypes.byref(n))
                syms = (ctypes.c_uint32 * max(n.value, 1))()
                lens = (ctypes.c_uint8 * max(n.value, 1))()
                L.crx_update_table_entries(self._h, k, syms, lens)
                out.append(Table(e.value, list(syms)[: n.value], list(lens)[: n.value]))
            self._tables = out
        return self._tables

    @property
    def block_bits(self) -> list[int]:
        L = _ext.load()
        n = int(L.crx_update_n_blocks(self._h))
        arr = (ctypes.c_uint32 * max(n, 1))()
        L.crx_update_block_bits(self._h, arr)
        return list(arr)[:n]

    @property
    def payload(self) -> bytes:
        p, n = ctypes.c_void_p(), ctypes.c_int64()
        _ext.load().crx_update_payload(self._h, ctypes.byref(p), ctypes.byref(n))
        return ctypes.string_at(p, n.value) if n.value and p.value else b""

    @property
    def changes(self) -> int:
        return int(_ext.load().crx_update_changes(self._h))

    def to_update(self) -> Update:
        return Update(self.tables, self.tensors, self.block_bits, self.payload)

    def close(self):
        if self._h:
            _ext.load().crx_update_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def parse(data: bytes) -> ParsedUpdate:
    """Parse and structurally validate an update (every limit of the format); CorruptUpdate if not."""
    return ParsedUpdate(data)


def encoder_parse(update):
    """The parse that to_device attached to a device update, while the tensor is the one it wrote
    and was not modified since (same address, size and version counter); else None."""
    pre = getattr(update, "_crx_parsed", None)
    if pre is not None and pre[1] == update._version and pre[2] == update.data_ptr() and pre[3] == update.numel():
        return pre[0]
    return None


def parse_device(update, stream=None) -> ParsedUpdate:
    """parse() for an update held in device memory (a contiguous uint8 CUDA tensor): the header is
    copied to the host and validated there, the block table is checked on the device (same
    verdicts as parse()); the block table and payload stay on the device for apply."""
    import torch

    if not (isinstance(update, torch.Tensor) and update.dtype == torch.uint8 and update.is_cuda
            and update.dim() == 1 and update.is_contiguous()):
        raise ValueError("a device update must be a contiguous 1-D uint8 CUDA tensor")
    L = _ext.load()
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(512)
    st = stream if stream is not None else torch.cuda.current_stream(update.device).cuda_stream
    with torch.cuda.device(update.device):
        rc = L.crx_parse_device(ctypes.c_void_p(update.data_ptr() if update.numel() else 0), update.numel(),
                                ctypes.c_void_p(st), ctypes.byref(h), err, 512)
    if rc == _ext.CRX_CORRUPT:
        raise CorruptUpdate(err.value.decode(errors="replace"))
    if rc != _ext.CRX_OK:
        raise RuntimeError(f"crukx_sync_b200: device parse failed ({rc}): {err.value.decode(errors='replace')}")
    return ParsedUpdate(_handle=h, _keep=update)


def parse_head(head: bytes, length: int, last: int):
    """Validate an update from its first bytes: ``head`` = the first bytes of an update of
    ``length`` bytes whose final byte is ``last``.  Returns a ParsedUpdate (header view only; it
    cannot be applied), or, when ``head`` is too short, a length the head must at least have (grow
    it geometrically); CorruptUpdate when the update is invalid (the same verdict as parse())."""
    L = _ext.load()
    head = bytes(head)
    h = ctypes.c_void_p()
    need = ctypes.c_int64()
    err = ctypes.create_string_buffer(512)
    buf = ctypes.cast(ctypes.c_char_p(head), ctypes.c_void_p)
    rc = L.crx_parse_head(buf, len(head), int(length), int(last) & 0xFF, ctypes.byref(h), ctypes.byref(need), err, 512)
    if rc == _ext.CRX_NEED_MORE:
        return int(need.value)
    if rc == _ext.CRX_CORRUPT:
        raise CorruptUpdate(err.value.decode(errors="replace"))
    if rc != _ext.CRX_OK:
        raise RuntimeError(f"crukx_sync_b200: head parse failed ({rc}): {err.value.decode(errors='replace')}")
    return ParsedUpdate(_handle=h, _keep=head)
