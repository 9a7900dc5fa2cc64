"""Host-side checks of the product that need no GPU: the C-ABI library loads and exports every
symbol of include/crukx_b200.h, its parser accepts exactly what the oracle (and so the
reference) accepts, its Huffman builder matches, and caller mistakes raise the reference's
errors before any device work."""

import ctypes
import json
import os
import random
import re

import pytest
import torch

import cases
import hostile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="module")
def lib():
    from crukx_sync_b200 import _ext, build
    build.build()
    return _ext.load()


def header_symbols():
    text = open(os.path.join(ROOT, "include", "crukx_b200.h")).read()
    return sorted(set(re.findall(r"\b(crx_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lib):
    from crukx_sync_b200 import _ext
    names = header_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(_ext.EXPORTS) == names
    assert lib.crx_wire_version() == 2


def _golden_updates():
    out = []
    for f in sorted(os.listdir(GOLD)):
        if f.endswith(".bin"):
            out.append((f, open(os.path.join(GOLD, f), "rb").read()))
    return out


def _product_parse(data):
    from crukx_sync_b200.wire import CorruptUpdate, parse
    try:
        return parse(data)
    except CorruptUpdate:
        return None


def _oracle_parse(oracle, data):
    try:
        return oracle.parse(data)
    except oracle.OracleCorrupt:
        return None


@pytest.mark.parametrize("fname,data", _golden_updates())
def test_parse_matches_oracle_on_reference_updates(lib, oracle, fname, data):
    p = _product_parse(data)
    o = _oracle_parse(oracle, data)
    assert p is not None and o is not None
    assert [(t.name, t.numel, t.checksum, [(g.exponent, g.count, g.rice_r) for g in t.groups]) for t in p.tensors] == \
           [(t.name, t.numel, t.checksum, [(g.exponent, g.count, g.rice_r) for g in t.groups]) for t in o.tensors]
    from crukx_sync_b200.wire import serialize
    assert serialize(p.to_update()) == data          # the dataclass view re-serializes exactly
    assert p.changes == sum(g.count for t in p.tensors for g in t.groups)


def test_parse_accepts_exactly_what_the_oracle_accepts(lib, oracle):
    inputs = []
    flips = json.load(open(os.path.join(GOLD, "flips.json")))
    upd = bytes.fromhex(flips["update_hex"])
    for i in range(len(upd)):
        for x in (0x01, 0x80, 0xFF):
            b = bytearray(upd)
            b[i] ^= x
            inputs.append(bytes(b))
    inputs += [d for _, _, d in hostile.cases()]
    old, new = cases.case_multi()[0]
    inputs += hostile.prefixes(oracle.encode_update(old, new))
    rng = random.Random(5)
    for _ in range(300):                                  # random byte soup after a valid magic
        n = rng.randrange(0, 64)
        inputs.append(b"CRXS\x02" + bytes(rng.randrange(256) for _ in range(n)))
    mismatches = [k for k, d in enumerate(inputs)
                  if (_product_parse(d) is None) != (_oracle_parse(oracle, d) is None)]
    assert not mismatches, mismatches[:10]


def test_huffman_lengths_match_oracle(lib, oracle):
    rng = random.Random(3)
    for trial in range(400):
        n = rng.randint(1, 600)
        if trial % 7 == 0:
            counts = [int(1.7 ** (i % 45)) + 1 for i in range(n)]      # forces length limiting
        else:
            counts = [rng.choice([1, 1, 2, 3, 5, rng.randint(1, 10**9)]) for _ in range(n)]
        c = (ctypes.c_uint64 * n)(*counts)
        out = (ctypes.c_uint8 * n)()
        assert lib.crx_huffman_lengths(c, n, out) == 0
        assert list(out) == oracle.huffman_lengths(counts), trial


def test_huffman_lengths_match_oracle_on_large_tables(lib, oracle):
    """Alphabets of thousands of symbols (the radix-sorted path), with counts that need several
    length-limit rounds, the flat fallback, runs of equal counts, and counts on both sides of the
    packed-key limit (2^40)."""
    rng = random.Random(11)
    cases = []
    for n in (256, 257, 1000, 4247, 9000, 20000):
        cases.append([rng.randint(1, 1 << 30) for _ in range(n)])                      # flat fallback
        cases.append([rng.choice([1, 2, 3, 4, 5, 8, 13, 1000, rng.randint(1, 10**7)]) for _ in range(n)])
        cases.append([int(1.3 ** (i % 60)) + rng.randint(0, 3) for i in range(n)])   # a few rounds
        cases.append([7] * n)                                                          # all tied
    cases.append([rng.randint(1, 1 << 30) for _ in range(999)] + [(1 << 40) + 5])       # one count too big to pack
    cases.append([(1 << 40) - 1] + [rng.randint(1, 99) for _ in range(3000)])
    for k, counts in enumerate(cases):
        n = len(counts)
        c = (ctypes.c_uint64 * n)(*counts)
        out = (ctypes.c_uint8 * n)()
        assert lib.crx_huffman_lengths(c, n, out) == 0
        assert list(out) == oracle.huffman_lengths(counts), k


def test_caller_mistakes_raise_before_device_work():
    from crukx_sync_b200 import CorruptUpdate, apply_update, encode_update
    a, b = cases.rl_pair(1000)
    with pytest.raises(ValueError):
        encode_update({"w": a}, {"x": b})
    with pytest.raises(ValueError):
        encode_update({"w": a}, {"w": b.float()})
    with pytest.raises(ValueError):
        encode_update({"w": a}, {"w": b[:999]})
    with pytest.raises(ValueError):
        encode_update({"w": a.view(10, 100).t()}, {"w": b.view(10, 100).t()})
    upd = open(os.path.join(GOLD, "rl_200k_0.bin"), "rb").read()
    with pytest.raises(ValueError):
        apply_update({"other": a}, upd)
    with pytest.raises(ValueError):
        apply_update({"w": torch.zeros(7, dtype=torch.int16)}, upd)
    for label, make_w, data in hostile.cases():
        if json.load(open(os.path.join(GOLD, "hostile.json")))["cases"][label] != "CorruptUpdate":
            continue
        if _product_parse(data) is None:                 # parse-level rejections need no GPU
            w = make_w()
            with pytest.raises(CorruptUpdate):
                apply_update(w, data)


def test_empty_update_needs_no_device():
    from crukx_sync_b200 import apply_update
    st = apply_update({}, b"CRXS\x02\x00\x00\x00")
    assert (st.tensors, st.changed, st.bytes) == (0, 0, 8)


@pytest.mark.timeout(60)
def test_first_context_call_does_not_deadlock(lib, monkeypatch):
    """context() before any load(): must return or raise, never block on its own lock."""
    from crukx_sync_b200 import _ext
    monkeypatch.setattr(_ext, "_lib", None)
    monkeypatch.setattr(_ext, "_ctx", {})
    if torch.cuda.is_available():
        assert _ext.context(0)
    else:
        with pytest.raises(RuntimeError):
            _ext.context(0)
