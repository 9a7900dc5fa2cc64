"""Pin the CPU oracle to the reference: byte-identical updates, equal checksum caches, exact
round trips, and the reference's own verdict on every corrupted or hostile update (fixtures in
tests/golden/, produced by running the reference; see tests/golden/make_golden.py)."""

import hashlib
import json
import os

import pytest
import torch

import cases
import hostile

GOLD = os.path.join(os.path.dirname(__file__), "golden")
MANIFEST = json.load(open(os.path.join(GOLD, "manifest.json")))
FLIPS = json.load(open(os.path.join(GOLD, "flips.json")))
HOSTILE = json.load(open(os.path.join(GOLD, "hostile.json")))


def _eq(x, y):
    return torch.equal(x.contiguous().view(torch.int16).reshape(-1), y.contiguous().view(torch.int16).reshape(-1))


@pytest.mark.parametrize("name", list(cases.CASES))
def test_oracle_matches_reference_bytes(oracle, name):
    fn, chained = cases.CASES[name]
    steps = fn()
    sender, receiver = ({}, {}) if chained else (None, None)
    recv = None
    for k, (old, new) in enumerate(steps):
        row = MANIFEST[name]["steps"][k]
        assert cases.digest_inputs(old, new) == row["inputs_sha256"], "input generator drifted"
        upd = oracle.encode_update(old, new, sender)
        if "file" in row:
            assert upd == open(os.path.join(GOLD, row["file"]), "rb").read()
        assert len(upd) == row["update_len"]
        assert hashlib.sha256(upd).hexdigest() == row["update_sha256"]
        if sender is not None:
            assert {n: str(v) for n, v in sender.items()} == row["sender_checksums"]
        if recv is None or not chained:
            recv = {n: v.clone() for n, v in old.items()}
        stats = oracle.apply_update(recv, upd, receiver)
        assert (stats.tensors, stats.changed) == (row["tensors"], row["changed"])
        for n in new:
            assert _eq(recv[n], new[n]), n
    if chained:
        assert sender == {k: v[0] for k, v in receiver.items()}


def test_oracle_byte_flip_verdicts_match_reference(oracle):
    a, b = cases.flip_case()
    assert cases.digest_inputs({"w": a}, {"w": b}) == FLIPS["inputs_sha256"]
    upd = bytes.fromhex(FLIPS["update_hex"])
    assert oracle.encode_update({"w": a}, {"w": b}) == upd
    got = []
    for i in range(len(upd)):
        for x in FLIPS["xors"]:
            bad = bytearray(upd)
            bad[i] ^= x
            w = {"w": a.clone()}
            try:
                oracle.apply_update(w, bytes(bad))
                v = "ok"
                assert _eq(w["w"], b)
            except oracle.OracleCorrupt:
                v = "CorruptUpdate"
                assert _eq(w["w"], a)
            except ValueError:
                v = "ValueError"
                assert _eq(w["w"], a)
            got.append(v)
    assert got == FLIPS["verdicts"]


@pytest.mark.parametrize("label", [c[0] for c in hostile.cases()])
def test_oracle_hostile_verdicts_match_reference(oracle, label):
    _, make_w, data = next(c for c in hostile.cases() if c[0] == label)
    w = make_w()
    before = {k: v.clone() for k, v in w.items()}
    try:
        oracle.apply_update(w, data)
        v = "ok"
    except oracle.OracleCorrupt:
        v = "CorruptUpdate"
    except ValueError:
        v = "ValueError"
    assert v == HOSTILE["cases"][label]
    for k in w:
        assert torch.equal(w[k], before[k])


def test_oracle_prefix_verdicts_match_reference(oracle):
    old, new = cases.case_multi()[0]
    upd = oracle.encode_update(old, new)
    got = []
    for p in hostile.prefixes(upd):
        w = {k: v.clone() for k, v in old.items()}
        try:
            oracle.apply_update(w, p)
            got.append("o")
        except oracle.OracleCorrupt:
            got.append("C")
        except ValueError:
            got.append("V")
    assert "".join(got) == HOSTILE["multi_prefix_verdicts"]


def test_oracle_checksum_known_answers(oracle):
    # FORMAT.md:61-64 splitmix64 of i+1; w_0 = splitmix64(1) | 1
    z = 0x9E3779B97F4A7C15
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & (2**64 - 1)
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & (2**64 - 1)
    w0 = (z ^ (z >> 31)) | 1
    assert oracle.weight(0) == w0
    a = torch.tensor([1, -1, 0x3F80], dtype=torch.int16)
    want = sum((int(v) & 0xFFFF) * oracle.weight(i) for i, v in enumerate(a.tolist())) % 2**64
    assert oracle.checksum(a) == want


def test_oracle_huffman_tie_order(oracle):
    # equal counts: the heap pops lower ids first, merged nodes after leaves of equal count
    assert oracle.huffman_lengths([1]) == [1]
    assert oracle.huffman_lengths([5, 5]) == [1, 1]
    assert oracle.huffman_lengths([1, 1, 1, 1]) == [2, 2, 2, 2]
    assert oracle.huffman_lengths([1, 1, 2]) == [2, 2, 1]
    assert oracle.huffman_lengths([2, 1, 1]) == [1, 2, 2]
    # more than 17 levels forces the flattening rounds
    fib = [1, 1]
    while len(fib) < 30:
        fib.append(fib[-1] + fib[-2])
    assert max(oracle.huffman_lengths(fib)) <= 17
