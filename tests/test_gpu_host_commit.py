"""Applying an update to weights that live on the host (crx_apply_to_host).  Pinned tensors at the
end of the list come down whole by DMA after a device-side commit, the others are scattered from
the commit list by host threads; both must leave exactly the sender's new weights, whatever mix of
pinned and pageable memory, tensor sizes and unchanged tensors the receiver has."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


SIZES = [300_000, 1_000_000, 17, 2_500_000, 4096, 700_001, 1_300_000, 262_144, 3, 900_000]


def states(seed=11, n_steps=3):
    rng = torch.Generator().manual_seed(seed)
    w = {f"t{i}": (0.02 * torch.randn(n, generator=rng)).bfloat16() for i, n in enumerate(SIZES)}
    w["t9"] = torch.zeros(SIZES[9], dtype=torch.bfloat16)   # stays unchanged
    out = [w]
    for _ in range(n_steps):
        nxt = {}
        for k, v in out[-1].items():
            if k == "t9":
                nxt[k] = v.clone()
            else:
                nxt[k] = (v.float() + 2e-4 * torch.randn(v.numel(), generator=rng)).bfloat16()
        out.append(nxt)
    return out


def host_copy(w, pinned):
    return {k: (v.clone().pin_memory() if pinned(i, k) else v.clone()) for i, (k, v) in enumerate(w.items())}


@pytest.mark.parametrize("mode", ["all_pinned", "pageable", "mixed", "pinned_head"])
def test_host_receiver_matches_sender(mode):
    import crukx_sync_b200 as crx
    pick = {
        "all_pinned": lambda i, k: True,
        "pageable": lambda i, k: False,
        "mixed": lambda i, k: i % 2 == 1,
        "pinned_head": lambda i, k: i < 5,
    }[mode]
    seq = states()
    send, recv_cache = {}, {}
    host = host_copy(seq[0], pick)
    ctrl = {k: v.cuda() for k, v in seq[0].items()}
    for i in range(1, len(seq)):
        prev = {k: v.cuda() for k, v in seq[i - 1].items()}
        cur = {k: v.cuda() for k, v in seq[i].items()}
        upd = crx.encode_update(prev, cur, send)
        st_h = crx.apply_update(host, upd, recv_cache)
        st_d = crx.apply_update(ctrl, upd)
        assert st_h.changed == st_d.changed
        for k in cur:
            assert host[k].device.type == "cpu"
            assert torch.equal(host[k].view(torch.int16), seq[i][k].view(torch.int16)), (mode, i, k)
            assert torch.equal(ctrl[k].cpu().view(torch.int16), seq[i][k].view(torch.int16)), (mode, i, k)
    assert host["t0"].is_pinned() == pick(0, "t0")


def test_host_receiver_rejects_and_keeps_weights():
    """A corrupt update is refused before anything is written, on either way down."""
    import crukx_sync_b200 as crx
    seq = states(seed=12, n_steps=1)
    upd = bytearray(crx.encode_update({k: v.cuda() for k, v in seq[0].items()},
                                      {k: v.cuda() for k, v in seq[1].items()}))
    upd[-5] ^= 0x40
    host = host_copy(seq[0], lambda i, k: i >= 5)
    with pytest.raises(ValueError):
        crx.apply_update(host, bytes(upd))
    for k in seq[0]:
        assert torch.equal(host[k].view(torch.int16), seq[0][k].view(torch.int16)), k
