"""Parity of the CUDA path with the reference (golden fixtures) and the CPU oracle, through the
public API and the C ABI: byte-identical updates, bit-exact weights, identical verdicts on
corrupted and hostile updates, the reference's cache and all-or-nothing semantics, and
size-independent properties at large sizes."""

import hashlib
import json
import os
import time

import pytest
import torch

import cases
import hostile

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")
MANIFEST = json.load(open(os.path.join(GOLD, "manifest.json")))
FLIPS = json.load(open(os.path.join(GOLD, "flips.json")))
HOSTILE = json.load(open(os.path.join(GOLD, "hostile.json")))


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from crukx_sync_b200 import _ext
    _ext.load()   # fails loudly when the library was not built


def crx():
    import crukx_sync_b200
    return crukx_sync_b200


def cu(d):
    return {k: v.cuda() for k, v in d.items()}


def eq(x, y):
    return torch.equal(x.contiguous().view(torch.int16).reshape(-1).cpu(), y.contiguous().view(torch.int16).reshape(-1).cpu())


def verdict(fn):
    from crukx_sync_b200 import CorruptUpdate
    try:
        fn()
        return "ok"
    except CorruptUpdate:
        return "CorruptUpdate"
    except ValueError:
        return "ValueError"


@pytest.mark.parametrize("name", list(cases.CASES))
def test_encode_and_apply_match_reference(name):
    c = crx()
    fn, chained = cases.CASES[name]
    steps = fn()
    sender, receiver = ({}, {}) if chained else (None, None)
    recv = None
    for k, (old, new) in enumerate(steps):
        row = MANIFEST[name]["steps"][k]
        assert cases.digest_inputs(old, new) == row["inputs_sha256"]
        go, gn = cu(old), cu(new)
        upd = c.encode_update(go, gn, sender)
        if "file" in row:
            assert upd == open(os.path.join(GOLD, row["file"]), "rb").read()
        assert (len(upd), hashlib.sha256(upd).hexdigest()) == (row["update_len"], row["update_sha256"])
        if sender is not None:
            assert {n: str(v) for n, v in sender.items()} == row["sender_checksums"]
        if recv is None or not chained:
            recv = {n: v.clone() for n, v in go.items()}
        stats = c.apply_update(recv, upd, receiver)
        assert (stats.tensors, stats.changed, stats.bytes) == (row["tensors"], row["changed"], len(upd))
        for n in new:
            assert eq(recv[n], new[n]), n
    if chained:
        assert sender == {k: v[0] for k, v in receiver.items()}


def test_byte_flip_verdicts_match_reference():
    c = crx()
    a, b = cases.flip_case()
    upd = bytes.fromhex(FLIPS["update_hex"])
    ga, gb = a.cuda(), b.cuda()
    assert c.encode_update({"w": ga}, {"w": gb}) == upd
    got = []
    for i in range(len(upd)):
        for x in FLIPS["xors"]:
            bad = bytearray(upd)
            bad[i] ^= x
            w = {"w": ga.clone()}
            v = verdict(lambda: c.apply_update(w, bytes(bad)))
            assert eq(w["w"], b if v == "ok" else a), (i, x, v)
            got.append(v)
    assert got == FLIPS["verdicts"]


@pytest.mark.parametrize("label", [x[0] for x in hostile.cases()])
def test_hostile_verdicts_match_reference(label):
    c = crx()
    _, make_w, data = next(x for x in hostile.cases() if x[0] == label)
    w = cu(make_w())
    before = {k: v.clone() for k, v in w.items()}
    t0 = time.time()
    assert verdict(lambda: c.apply_update(w, data)) == HOSTILE["cases"][label]
    assert time.time() - t0 < 30
    for k in w:
        assert torch.equal(w[k], before[k])


def test_truncated_update_verdicts_match_reference():
    c = crx()
    old, new = cases.case_multi()[0]
    go = cu(old)
    upd = c.encode_update(go, cu(new))
    got = "".join(verdict(lambda p=p: c.apply_update({k: v.clone() for k, v in go.items()}, p))[0]
                  for p in hostile.prefixes(upd))
    assert got == HOSTILE["multi_prefix_verdicts"]


def test_cpu_tensors_are_routed_through_the_gpu():
    c = crx()
    old, new = cases.case_rl_200k()[0]
    upd = c.encode_update(old, new)           # CPU in, same bytes out
    assert upd == open(os.path.join(GOLD, "rl_200k_0.bin"), "rb").read()
    w = {k: v.clone() for k, v in old.items()}
    view = w["w"][:]
    st = c.apply_update(w, upd)
    assert st.changed == MANIFEST["rl_200k"]["steps"][0]["changed"]
    assert eq(w["w"], new["w"]) and eq(view, new["w"]) and w["w"].device.type == "cpu"


def test_encode_on_gpu_apply_on_cpu_and_back():
    c = crx()
    a, b = cases.rl_pair(200_000, seed=3)
    upd = c.encode_update({"w": a.cuda()}, {"w": b.cuda()})
    w = {"w": a.clone()}
    c.apply_update(w, upd)
    assert eq(w["w"], b)
    upd2 = c.encode_update({"w": a}, {"w": b})
    assert upd2 == upd
    g = {"w": a.cuda()}
    c.apply_update(g, upd2)
    assert eq(g["w"], b)


def test_apply_writes_through_to_views():
    c = crx()
    a, b = cases.rl_pair(10_000, seed=5)
    buf = a.cuda()
    view = buf[:]
    c.apply_update({"w": buf}, c.encode_update({"w": a.cuda()}, {"w": b.cuda()}))
    assert eq(view, b)


def test_mixed_devices_and_mismatched_receivers_are_errors():
    c = crx()
    a, b = cases.rl_pair(1000)
    with pytest.raises(ValueError):
        c.encode_update({"w": a, "x": a.cuda()}, {"w": b, "x": b.cuda()})
    upd = c.encode_update({"w": a.cuda()}, {"w": b.cuda()})
    for bad in ({"other": a.cuda()}, {"w": a[:999].cuda()}):
        with pytest.raises(ValueError):
            c.apply_update(bad, upd)


def test_wrong_receiver_cache_is_rejected_not_silently_wrong():
    c = crx()
    a, b = cases.rl_pair(20_000, seed=8)
    upd = c.encode_update({"w": a.cuda()}, {"w": b.cuda()})
    old = {"w": a.cuda()}
    with pytest.raises(c.CorruptUpdate):
        c.apply_update(old, upd, {"w": (12345, old["w"]._version)})
    assert eq(old["w"], a)


def test_receiver_cache_does_not_hide_weights_that_drifted():
    c = crx()
    g = torch.Generator().manual_seed(9)
    w = torch.randn(50_000, generator=g) * 0.02
    s1, s2, s3 = (w.bfloat16().cuda(), (w + 1e-6).bfloat16().cuda(), (w + 2e-6).bfloat16().cuda())
    sender, receiver = {}, {}
    recv = {"w": s1.clone()}
    c.apply_update(recv, c.encode_update({"w": s1}, {"w": s2}, sender), receiver)
    recv["w"].view(torch.int16)[7] ^= 1
    with pytest.raises(c.CorruptUpdate):
        c.apply_update(recv, c.encode_update({"w": s2}, {"w": s3}, sender), receiver)


def test_sender_cache_is_not_committed_when_serialize_fails(monkeypatch):
    c = crx()
    a, b = cases.rl_pair(20_000, seed=10)
    cache = {}

    def boom(_):
        raise RuntimeError("serialize failed")
    monkeypatch.setattr(c, "serialize", boom)
    with pytest.raises(RuntimeError):
        c.encode_update({"w": a.cuda()}, {"w": b.cuda()}, cache)
    assert cache == {}


def test_sender_cache_gives_the_same_bytes_as_a_full_checksum():
    c = crx()
    steps = cases.case_chain5()
    cache = {}
    for old, new in steps:
        with_cache = c.encode_update(cu(old), cu(new), cache)
        assert with_cache == c.encode_update(cu(old), cu(new))


def test_device_checksum_matches_oracle(oracle):
    from crukx_sync_b200 import codec
    for n in (1, 7, 4099, 1 << 20, (1 << 22) + 3):
        a = torch.randint(-32768, 32768, (n,), dtype=torch.int16, generator=torch.Generator().manual_seed(n))
        assert codec.checksum(a.cuda()) == oracle.checksum(a)


@pytest.mark.parametrize("offset", [1, 3, 8])
def test_unaligned_views_match_oracle(oracle, offset):
    c = crx()
    a, b = cases.heavy_tail((1 << 19) + 77, 0.03, seed=50 + offset)
    ga, gb = a.cuda(), b.cuda()
    va, vb = ga[offset:], gb[offset:]
    assert va.data_ptr() % 16 != 0 or offset == 8
    upd = c.encode_update({"x": va}, {"x": vb})
    assert upd == oracle.encode_update({"x": a[offset:]}, {"x": b[offset:]})
    w = {"x": ga.clone()[offset:]}
    c.apply_update(w, upd)
    assert eq(w["x"], b[offset:])


@pytest.mark.parametrize("n,frac,single", [(16 << 20, 0.01, False), (16 << 20, 0.10, False),
                                           ((16 << 20) + 5, 0.03, True)])
def test_byte_parity_with_oracle_at_16m(oracle, n, frac, single):
    c = crx()
    a, b = cases.heavy_tail(n, frac, seed=60, single_group=single)
    sender, osender = {}, {}
    upd = c.encode_update({"flat": a.cuda()}, {"flat": b.cuda()}, sender)
    assert upd == oracle.encode_update({"flat": a}, {"flat": b}, osender)
    assert sender == osender


def test_blocks_longer_than_a_pack_slot_match_oracle(oracle):
    """Blocks of more than 4 Kbit (a pack slot) are encoded a second time straight into the payload:
    few changes spread over 2^24 elements of one exponent (a large Rice parameter) with random new
    bits (long codes) make blocks of about 7 Kbit; a second tensor has the usual short blocks.
    The bytes must be the reference's, on the bytes and the device paths, and apply must round-trip."""
    c = crx()
    g = torch.Generator().manual_seed(77)
    n = 1 << 24
    sign = torch.randint(0, 2, (n,), generator=g, dtype=torch.int32) << 15
    old_bits = (sign | 0x3F80 | torch.randint(0, 128, (n,), generator=g, dtype=torch.int32)).to(torch.int16)
    new_bits = old_bits.clone()
    pos = torch.randperm(n, generator=g)[:3 * 256 + 17]
    new_bits[pos] = torch.randint(-32768, 32768, (pos.numel(),), generator=g, dtype=torch.int32).to(torch.int16)
    a2, b2 = cases.heavy_tail((1 << 20) + 3, 0.05, seed=78)
    old = {"sparse": old_bits.view(torch.bfloat16), "dense": a2}
    new = {"sparse": new_bits.view(torch.bfloat16), "dense": b2}
    upd = c.encode_update(cu(old), cu(new))
    assert upd == oracle.encode_update(old, new)
    from crukx_sync_b200 import wire
    assert max(wire.parse(upd).block_bits) > 4096   # some blocks took the long path
    assert host_bytes(c.encode_update_device(cu(old), cu(new))) == upd
    w = {k: v.clone() for k, v in cu(old).items()}
    c.apply_update(w, upd)
    for k in new:
        assert eq(w[k], new[k]), k


def host_bytes(t):
    return t.cpu().numpy().tobytes()


@pytest.mark.parametrize("frac", [0.001, 0.01, 0.03, 0.10, 1.0])
def test_stress_256m_round_trip(frac):
    """BASELINE stress config at 256M elements: size-independent properties (exact round trip,
    cache of checksums equal on both sides, re-encode of the result is empty)."""
    c = crx()
    n = 256 << 20
    g = torch.Generator(device="cuda").manual_seed(int(frac * 1000))
    a = (0.02 * torch.randn(n, device="cuda", generator=g)).bfloat16().view(torch.int16)
    b = a.clone()
    if frac >= 1.0:
        b ^= 1 + (torch.rand(n, device="cuda", generator=g) * 7).to(torch.int16)
    else:
        idx = torch.randint(0, n, (int(n * frac),), device="cuda", generator=g)
        b[idx] += torch.randint(-3, 4, (idx.numel(),), device="cuda", generator=g, dtype=torch.int16) * 2 + 1
    sender, receiver = {}, {}
    upd = c.encode_update({"flat": a}, {"flat": b}, sender)
    w = {"flat": a.clone()}
    st = c.apply_update(w, upd, receiver)
    assert st.changed == int((a != b).sum())
    assert torch.equal(w["flat"], b)
    assert sender == {k: v[0] for k, v in receiver.items()}
    assert c.encode_update({"flat": w["flat"]}, {"flat": b}) == b"CRXS\x02\x00\x00\x00"
    del a, b, w
    torch.cuda.empty_cache()


def test_hostile_long_unary_runs_finish_quickly():
    c = crx()
    label, make_w, data = next(x for x in hostile.cases() if x[0] == "long_unary_ones")
    t = time.time()
    with pytest.raises(c.CorruptUpdate):
        c.apply_update(cu(make_w()), data)
    assert time.time() - t < 30
