"""Hand-built malformed updates (wire format version 2) and the receiver weights they target.

Each entry is ``(label, weights_factory, update_bytes)``.  The golden script records what the
reference's apply_update does with each (hostile.json); the oracle and the CUDA path must do the
same, and must leave the weights untouched.
"""

from __future__ import annotations

import torch


def varint(v: int) -> bytes:
    out = bytearray()
    while v >= 0x80:
        out.append((v & 0x7F) | 0x80)
        v >>= 7
    out.append(v)
    return bytes(out)


def _one_tensor(tables: bytes, tail: bytes, numel: int = 100, name: bytes = b"w") -> bytes:
    return b"CRXS\x02" + tables + varint(1) + varint(len(name)) + name + varint(numel) + bytes(8) + tail


ONE_TABLE = b"\x01\x00\x01\x02\x01"   # 1 table: exponent 0, 1 symbol (2), code length 1


def _zeros(n=100):
    return lambda: {"w": torch.zeros(n, dtype=torch.int16)}


def cases():
    out = []
    z = _zeros()
    out.append(("varint_2^63", z, _one_tensor(b"\x01\x00" + b"\xff" * 9 + b"\x7f", b"")))
    out.append(("varint_too_long", z, b"CRXS\x02" + b"\x80" * 11 + b"\x00"))
    out.append(("huge_count", z, _one_tensor(ONE_TABLE, b"\x01\x00" + varint(1 << 62) + b"\x00")))
    out.append(("rice_31", z, _one_tensor(ONE_TABLE, b"\x01\x00\x05\x1f")))
    out.append(("zero_groups", z, _one_tensor(ONE_TABLE, b"\x00")))
    out.append(("kraft_overflow", z, _one_tensor(b"\x01\x00\x02\x01\x01\x02\x01", b"")))
    out.append(("duplicate_group_exp", z, _one_tensor(ONE_TABLE, b"\x02\x00\x05\x00\x00\x05\x00")))
    out.append(("group_without_table", z, _one_tensor(ONE_TABLE, b"\x01\x07\x05\x00")))
    out.append(("bad_magic", z, b"CRXT\x02\x00\x00" + varint(0)))
    out.append(("bad_version", z, b"CRXS\x01\x00\x00" + varint(0)))
    out.append(("too_many_tables", z, b"CRXS\x02" + varint(257)))
    out.append(("dup_table_exp", z, b"CRXS\x02\x02\x00\x01\x02\x01\x00\x01\x02\x01"))
    out.append(("symbol_too_big", z, _one_tensor(b"\x01\x00\x01" + varint(131071) + b"\x01", b"")))
    out.append(("dup_symbols", z, _one_tensor(b"\x01\x00\x02\x02\x01\x02\x01", b"")))
    out.append(("len_zero", z, _one_tensor(b"\x01\x00\x01\x02\x00", b"")))
    out.append(("len_18", z, _one_tensor(b"\x01\x00\x01\x02\x12", b"")))
    out.append(("nsym_exceeds_bytes", z, b"CRXS\x02\x01\x00" + varint(1000) + b"\x02\x01"))
    out.append(("too_many_tensors", z, b"CRXS\x02" + ONE_TABLE[0:0] + b"\x00" + varint(50) + b"\x00"))
    out.append(("bad_utf8_name", z, _one_tensor(ONE_TABLE, b"\x01\x00\x01\x00", name=b"\xff")))
    out.append(("surrogate_name", z, _one_tensor(ONE_TABLE, b"\x01\x00\x01\x00", name=b"\xed\xa0\x80")))
    # one valid change: exponent 0, count 1, rice 0; gap 0 -> "0", symbol 2 -> code "0": 2 bits
    good_tail = b"\x01\x00\x01\x00" + (2).to_bytes(4, "little") + varint(1) + b"\x00"
    out.append(("valid_but_wrong_checksum", z, _one_tensor(ONE_TABLE, good_tail)))
    out.append(("trailing_byte", z, _one_tensor(ONE_TABLE, good_tail + b"\x00")))
    out.append(("payload_len_mismatch", z, _one_tensor(ONE_TABLE, b"\x01\x00\x01\x00" + (2).to_bytes(4, "little") + varint(2) + b"\x00\x00")))
    out.append(("nonzero_padding", z, _one_tensor(ONE_TABLE, b"\x01\x00\x01\x00" + (2).to_bytes(4, "little") + varint(1) + b"\x01")))
    out.append(("block_too_short", z, _one_tensor(ONE_TABLE, b"\x01\x00\x01\x00" + (1).to_bytes(4, "little") + varint(1) + b"\x00")))
    out.append(("count_exceeds_numel", z, _one_tensor(ONE_TABLE, b"\x01\x00" + varint(101) + b"\x00")))
    two_tables = b"\x02\x00\x01\x02\x01\x05\x01\x02\x01"
    out.append(("table_unused", z, _one_tensor(two_tables, good_tail)))
    out.append(("dup_tensor_name", z, b"CRXS\x02" + ONE_TABLE + varint(2)
                + (varint(1) + b"w" + varint(100) + bytes(8) + b"\x01\x00\x01\x00") * 2
                + (2).to_bytes(4, "little") * 2 + varint(1) + b"\x00"))
    # checksum of the target weights after the change is right, but the block overruns
    out.append(("block_longer_than_symbols", z, _one_tensor(ONE_TABLE, b"\x01\x00\x01\x00" + (3).to_bytes(4, "little") + varint(1) + b"\x00")))
    # a group claiming more changes than elements of its exponent (all weights have exponent 0)
    big = 1 << 22
    out.append(("count_beyond_group", lambda: {"w": torch.full((100,), 0x3F80, dtype=torch.int16)},
                _one_tensor(ONE_TABLE, good_tail)))
    hostile = bytearray(b"CRXS\x02") + varint(1) + b"\x00\x01\x02\x01" + varint(1) + varint(1) + b"w"
    hostile += varint(big) + bytes(8) + varint(1) + b"\x00" + varint(big) + b"\x00"
    hostile += bytes(4 * (big // 256)) + varint(0)
    out.append(("hostile_count_before_alloc", lambda: {"w": torch.zeros(big, dtype=torch.int16)}, bytes(hostile)))
    # many blocks over one long run of one-bits: must be rejected in time linear in the payload
    n, count = 1 << 20, 1 << 18
    payload = b"\xff" * (count * 2 // 8)
    lr = bytearray(b"CRXS\x02") + varint(1) + b"\x7f\x01\x02\x01" + varint(1) + varint(1) + b"w"
    lr += varint(n) + bytes(8) + varint(1) + b"\x7f" + varint(count) + b"\x00"
    lr += (512).to_bytes(4, "little") * (count // 256) + varint(len(payload)) + payload
    out.append(("long_unary_ones", lambda: {"w": torch.full((n,), 0x3F80, dtype=torch.int16)}, bytes(lr)))
    # receiver mismatch (ValueError): name or size differs from the receiver's
    out.append(("receiver_missing_name", lambda: {"other": torch.zeros(100, dtype=torch.int16)},
                _one_tensor(ONE_TABLE, good_tail)))
    out.append(("receiver_numel_mismatch", lambda: {"w": torch.zeros(99, dtype=torch.int16)},
                _one_tensor(ONE_TABLE, good_tail)))
    return out


def prefixes(upd: bytes):
    """Every proper prefix of a valid update: each must be rejected as truncated or malformed."""
    return [upd[:k] for k in range(len(upd))]
