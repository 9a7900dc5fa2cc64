"""Device-resident updates: encode_update_device / apply_update from a CUDA uint8 tensor give the
reference's bytes and verdicts, with the payload never leaving the GPU."""

import hashlib
import json
import os

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
    _ext.load()


def crx():
    import crukx_sync_b200
    return crukx_sync_b200


def cu(d):
    return {k: v.cuda() for k, v in d.items()}


def eq(x, y):
    return torch.equal(x.contiguous().view(torch.int16).reshape(-1).cpu(), y.contiguous().view(torch.int16).reshape(-1).cpu())


def dev(b):
    return torch.frombuffer(bytearray(b), dtype=torch.uint8).cuda() if b else torch.empty(0, dtype=torch.uint8, device="cuda")


def host(t):
    return t.cpu().numpy().tobytes()


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
def test_device_updates_are_the_reference_bytes(name):
    c = crx()
    fn, chained = cases.CASES[name]
    steps = fn()
    sender, receiver = ({}, {}) if chained else (None, None)
    recv = None
    for k, (old, new) in enumerate(steps):
        row = MANIFEST[name]["steps"][k]
        go, gn = cu(old), cu(new)
        t = c.encode_update_device(go, gn, sender)
        assert t.is_cuda and t.dtype == torch.uint8
        upd = host(t)
        assert (len(upd), hashlib.sha256(upd).hexdigest()) == (row["update_len"], row["update_sha256"])
        if sender is not None:
            assert {n: str(v) for n, v in sender.items()} == row["sender_checksums"]
        if recv is None or not chained:
            recv = {n: v.clone() for n, v in go.items()}
        stats = c.apply_update(recv, t, receiver)
        assert (stats.tensors, stats.changed, stats.bytes) == (row["tensors"], row["changed"], len(upd))
        for n in new:
            assert eq(recv[n], new[n]), n
    if chained:
        assert sender == {k: v[0] for k, v in receiver.items()}


def test_bytes_and_device_paths_interoperate():
    c = crx()
    old, new = cases.case_multi()[0]
    go, gn = cu(old), cu(new)
    b = c.encode_update(go, gn)
    t = c.encode_update_device(go, gn)
    assert host(t) == b
    w1 = {k: v.clone() for k, v in go.items()}
    w2 = {k: v.clone() for k, v in go.items()}
    c.apply_update(w1, dev(b))          # host-encoded bytes, applied from the device
    c.apply_update(w2, host(t))         # device-encoded, applied from host bytes
    for k in new:
        assert eq(w1[k], new[k]) and eq(w2[k], new[k])


def test_device_flip_verdicts_match_reference():
    c = crx()
    a, b = cases.flip_case()
    upd = bytes.fromhex(FLIPS["update_hex"])
    ga, gb = a.cuda(), b.cuda()
    assert host(c.encode_update_device({"w": ga}, {"w": gb})) == upd
    got = []
    for i in range(len(upd)):
        for x in FLIPS["xors"]:
            bad = bytearray(upd)
            bad[i] ^= x
            w = {"w": ga.clone()}
            v = verdict(lambda: c.apply_update(w, dev(bytes(bad))))
            assert eq(w["w"], b if v == "ok" else a), (i, x, v)
            got.append(v)
    assert got == FLIPS["verdicts"]


@pytest.mark.parametrize("label", [x[0] for x in hostile.cases()])
def test_device_hostile_verdicts_match_reference(label):
    c = crx()
    _, make_w, data = next(x for x in hostile.cases() if x[0] == label)
    w = cu(make_w())
    before = {k: v.clone() for k, v in w.items()}
    assert verdict(lambda: c.apply_update(w, dev(data))) == HOSTILE["cases"][label]
    for k in w:
        assert torch.equal(w[k], before[k])


def test_device_truncations_match_host_truncations():
    c = crx()
    old, new = cases.case_multi()[0]
    go = cu(old)
    upd = c.encode_update(go, cu(new))
    for p in hostile.prefixes(upd):
        wh = {k: v.clone() for k, v in go.items()}
        wd = {k: v.clone() for k, v in go.items()}
        assert verdict(lambda: c.apply_update(wh, p)) == verdict(lambda: c.apply_update(wd, dev(p))), len(p)
        for k in go:
            assert torch.equal(wh[k], wd[k])


def test_large_header_needs_several_head_copies():
    # 300 small tensors: a header of several KB; parse_device grows its head copy until it fits
    c = crx()
    old, new = cases.CASES["many_small"][0]()[0] if "many_small" in cases.CASES else cases.case_multi()[0]
    go, gn = cu(old), cu(new)
    t = c.encode_update_device(go, gn)
    w = {k: v.clone() for k, v in go.items()}
    c.apply_update(w, t)
    for k in new:
        assert eq(w[k], new[k])


def test_block_table_past_the_first_head_copy():
    """A block table longer than parse_device's first head copy: the parse stops past the table and
    resumes on the few bytes after it.  The first apply in a process grows its head buffer, which
    moves it, so the header is parsed anew; the later ones resume.  All must give the sender's state."""
    c = crx()
    g = torch.Generator().manual_seed(21)
    states = [{"a": (0.02 * torch.randn(6_000_000, generator=g)).bfloat16(),
               "b": (0.02 * torch.randn(3_000_000, generator=g)).bfloat16()}]
    for _ in range(3):   # most elements change: about 29 K blocks, a 113 KB table after a small header
        states.append({k: (v.float() + 2e-4 * torch.randn(v.numel(), generator=g)).bfloat16() for k, v in states[-1].items()})
    w = cu(states[0])
    send, recv = {}, {}
    for i in range(1, len(states)):
        t = c.encode_update_device(cu(states[i - 1]), cu(states[i]), send)
        st = c.apply_update(w, t, recv)
        assert st.changed > 0
        for k in w:
            assert eq(w[k], states[i][k]), (i, k)


def test_head_only_update_cannot_be_applied():
    from crukx_sync_b200 import codec
    from crukx_sync_b200.wire import parse, parse_head
    c = crx()
    old, new = cases.case_multi()[0]
    go = cu(old)
    upd = c.encode_update(go, cu(new))
    head = parse_head(upd[: len(upd) - len(parse(upd).payload)], len(upd), upd[-1])
    w = {k: v.clone() for k, v in go.items()}
    with pytest.raises(ValueError):
        codec.apply(w, head)
    for k in go:
        assert torch.equal(w[k], go[k])


def test_encoder_parse_until_the_update_is_modified():
    """A device update carries its encoder's parse: applied as it is, it gives the new weights;
    after an in-place change of one byte (the tensor's version moves) it is parsed anew from the
    device and gets the same verdict as the changed bytes do on the host path."""
    from crukx_sync_b200 import wire
    c = crx()
    old, new = cases.case_multi()[0]
    go, gn = cu(old), cu(new)
    t = c.encode_update_device(go, gn)
    assert wire.encoder_parse(t) is not None
    assert wire.encoder_parse(t).tensor_table() == wire.parse_device(t).tensor_table()
    assert wire.encoder_parse(t).changes == wire.parse_device(t).changes
    w = {k: v.clone() for k, v in go.items()}
    assert c.apply_update(w, t).changed > 0
    for k in new:
        assert eq(w[k], new[k])
    good = host(t)
    for i in (5, len(good) // 2, len(good) - 1):
        t2 = c.encode_update_device(go, gn)
        t2[i] ^= 0x41
        assert wire.encoder_parse(t2) is None
        bad = bytearray(good)
        bad[i] ^= 0x41
        wh = {k: v.clone() for k, v in go.items()}
        wd = {k: v.clone() for k, v in go.items()}
        vh = verdict(lambda: c.apply_update(wh, bytes(bad)))
        vd = verdict(lambda: c.apply_update(wd, t2))
        assert vh == vd, i
        for k in go:
            assert torch.equal(wh[k], wd[k])


def test_empty_update_on_device():
    c = crx()
    a, _ = cases.rl_pair(1000)
    ga = a.cuda()
    t = c.encode_update_device({"w": ga}, {"w": ga.clone()})
    assert host(t) == b"CRXS\x02\x00\x00\x00"
    assert c.apply_update({"w": ga}, t).changed == 0
