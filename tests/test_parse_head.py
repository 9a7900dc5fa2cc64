"""crx_parse_head (validation from an update's head, for transports and device-resident updates)
against crx_parse: the same verdict on every fixture, reached from any starting head length by
following its need-more answers.  Host only."""

import json
import os
import random

import pytest

import cases
import hostile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")


def _view(p):
    return (p.tensor_table(), p.changes, [(t.exponent, t.symbols, t.lengths) for t in p.tables], p.block_bits)


def _full(data):
    from crukx_sync_b200.wire import CorruptUpdate, parse
    try:
        return _view(parse(data))
    except CorruptUpdate:
        return None


def _from_head(data, start):
    """Verdict of parse_head starting with `start` bytes, fetching what it asks for."""
    from crukx_sync_b200.wire import CorruptUpdate, parse_head
    k = min(start, len(data))
    last = data[-1] if data else 0
    for _ in range(64):
        try:
            r = parse_head(data[:k], len(data), last)
        except CorruptUpdate:
            return None
        if isinstance(r, int):
            assert k < r <= len(data), (k, r, len(data))   # asks for more, never past the update
            k = min(len(data), max(r, 2 * k))             # `need` is a lower bound: grow geometrically
            continue
        if k < len(data):
            assert r.payload == b""   # a head without the whole payload gives no payload view
        return _view(r)
    raise AssertionError("parse_head did not settle")


def _inputs():
    out = [open(os.path.join(GOLD, f), "rb").read() for f in sorted(os.listdir(GOLD)) if f.endswith(".bin")]
    flips = json.load(open(os.path.join(GOLD, "flips.json")))
    upd = bytes.fromhex(flips["update_hex"])
    out.append(upd)
    for i in range(0, len(upd), 3):
        for x in (0x01, 0x80, 0xFF):
            b = bytearray(upd)
            b[i] ^= x
            out.append(bytes(b))
    out += [d for _, _, d in hostile.cases()]
    out += hostile.prefixes(upd)
    rng = random.Random(11)
    for _ in range(100):
        out.append(b"CRXS\x02" + bytes(rng.randrange(256) for _ in range(rng.randrange(0, 64))))
    return out


def test_head_parse_gives_the_full_parse_verdict():
    inputs = _inputs()
    assert len(inputs) > 300
    for n, data in enumerate(inputs):
        want = _full(data)
        for start in (0, 1, 5, 7, 16, 64, len(data) // 3, len(data)):
            assert _from_head(data, start) == want, (n, start)


def test_head_without_payload_bytes():
    # a valid update parses from its head alone: the payload bytes are never needed (only the last)
    from crukx_sync_b200.wire import parse, parse_head
    data = open(os.path.join(GOLD, "rl_200k_0.bin"), "rb").read()
    full = parse(data)
    head_len = len(data) - len(full.payload)
    r = parse_head(data[:head_len], len(data), data[-1])
    assert not isinstance(r, int)
    assert _view(r) == _view(full)
    # a wrong final byte is caught as non-zero padding when the payload ends mid-byte
    bits = sum(full.block_bits)
    if bits % 8:
        from crukx_sync_b200.wire import CorruptUpdate
        with pytest.raises(CorruptUpdate):
            parse_head(data[:head_len], len(data), data[-1] | 1)


def test_head_view_matches_reference_dataclasses():
    from crukx_sync_b200.wire import parse, parse_head
    data = open(os.path.join(GOLD, "rl_200k_0.bin"), "rb").read()
    r = parse_head(data[: len(data) - len(parse(data).payload)], len(data), data[-1])
    assert [t.name for t in r.tensors] == [t.name for t in parse(data).tensors]
    assert r.n_tensors >= 1 and r.payload == b""
