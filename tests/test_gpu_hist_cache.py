"""The receiver's exponent-histogram cache (crx_apply_versioned): hits after the first apply,
bit-exact results, misses after in-place edits, and a stale entry can only end in CorruptUpdate
with nothing written."""

import ctypes

import pytest
import torch

import cases

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


def hits():
    from crukx_sync_b200 import _ext
    return int(_ext.load().crx_ctx_hist_cache_hits(_ext.context(torch.cuda.current_device())))


def chain(n_steps=5, seed=3):
    rng = torch.Generator().manual_seed(seed)
    w = (0.02 * torch.randn(3 * 400_000, generator=rng)).bfloat16()
    states = [w]
    for _ in range(n_steps):
        m = states[-1].float() + 2e-4 * torch.randn(w.numel(), generator=rng)
        states.append(m.bfloat16())
    return [{"a": s[:400_000].clone(), "b": s[400_000:1_000_000].clone(), "c": s[1_000_000:].clone()} for s in states]


def test_cache_hits_and_results_match():
    import crukx_sync_b200 as crx
    states = chain()
    send, recv_cache = {}, {}
    w = {k: v.cuda() for k, v in states[0].items()}
    w_plain = {k: v.cuda() for k, v in states[0].items()}
    h0 = hits()
    for i in range(1, len(states)):
        prev = {k: v.cuda() for k, v in states[i - 1].items()}
        cur = {k: v.cuda() for k, v in states[i].items()}
        upd = crx.encode_update(prev, cur, send)
        crx.apply_update(w, upd, recv_cache)          # cached checksums -> histogram cache
        crx.apply_update(w_plain, upd)                # no caches
        for k in cur:
            assert torch.equal(w[k], cur[k]) and torch.equal(w_plain[k], cur[k]), (i, k)
    # every apply after the first found all three tensors' histograms
    assert hits() - h0 == 3 * (len(states) - 2)


def test_in_place_edit_misses_and_stays_exact():
    import crukx_sync_b200 as crx
    states = chain(3, seed=5)
    send, recv_cache = {}, {}
    w = {k: v.cuda() for k, v in states[0].items()}
    upd = crx.encode_update({k: v.cuda() for k, v in states[0].items()}, {k: v.cuda() for k, v in states[1].items()}, send)
    crx.apply_update(w, upd, recv_cache)
    w["a"].add_(0)                                     # bumps a's version: its caches are no longer trusted
    upd = crx.encode_update({k: v.cuda() for k, v in states[1].items()}, {k: v.cuda() for k, v in states[2].items()}, send)
    h0 = hits()
    crx.apply_update(w, upd, recv_cache)
    assert hits() - h0 == 2                            # b and c hit, a recomputed
    for k in w:
        assert torch.equal(w[k].cpu(), states[2][k])


def test_stale_entry_fails_verification_and_writes_nothing():
    import crukx_sync_b200 as crx
    states = chain(2, seed=7)
    send, recv_cache = {}, {}
    w = {k: v.cuda() for k, v in states[0].items()}
    upd = crx.encode_update({k: v.cuda() for k, v in states[0].items()}, {k: v.cuda() for k, v in states[1].items()}, send)
    crx.apply_update(w, upd, recv_cache)
    # an edit the version counter does not see: both caches are now stale, as in the reference
    x = w["b"].data.view(torch.int16)
    x[12345] = x[12345] ^ 0x0100                       # moves one element's exponent
    before = {k: v.clone() for k, v in w.items()}
    upd = crx.encode_update({k: v.cuda() for k, v in states[1].items()}, {k: v.cuda() for k, v in states[2].items()}, send)
    with pytest.raises(crx.CorruptUpdate):
        crx.apply_update(w, upd, recv_cache)
    for k in w:
        assert torch.equal(w[k], before[k])


def test_device_path_uses_the_cache_too():
    import crukx_sync_b200 as crx
    states = chain(3, seed=9)
    send, recv_cache = {}, {}
    w = {k: v.cuda() for k, v in states[0].items()}
    for i in (1, 2):
        t = crx.encode_update_device({k: v.cuda() for k, v in states[i - 1].items()}, {k: v.cuda() for k, v in states[i].items()}, send)
        h0 = hits()
        crx.apply_update(w, t, recv_cache)
        if i == 2:
            assert hits() - h0 == 3
    for k in w:
        assert torch.equal(w[k].cpu(), states[2][k])
