"""Byte identity with the CPU oracle at the sizes the benchmark configurations name.

The oracle (oracle/crx_oracle.c) restates the reference's encode/apply and is pinned to bytes the
reference itself produced (tests/golden); here it checks the CUDA path on the same inputs at full
model and stress sizes, where no fixture can be stored:

* the Qwen2.5-1.5B shape (338 tensors, 1.54B params), lr 1e-6, 7 chained steps with the sender
  and receiver checksum caches kept (reference src/crukx_sync/__init__.py:38-57, codec.py:344-352,
  457-460);
* one 8-way tensor-parallel shard of the Qwen2.5-32B shape (qkv/gate/up and the vocabulary
  column-split, o/down row-split; 4.1B params), lr 1e-6, 2 chained steps;
* single flat tensors with the heavy-tailed delta (85% +-1 ULP, 10% +-2..7, 5% up to +-2^10 with
  sign flips) at 2^28 elements for 0.1/1/3/10/100% changed and with every element in one exponent
  group, and at 2^31 elements (int64 indexing throughout) for 1% and 100%.

Every update must equal the oracle's byte for byte (whole-dict updates, one Huffman table per
exponent over the whole update), the sender caches must agree, and the receiver must end bit-exact
equal to the sender's state.  Inputs are generated on the GPU with a seeded generator and copied
to the host for the oracle, so both sides read the same bits.
"""

import hashlib
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from crukx_sync_b200 import _ext
    _ext.load()   # fails loudly when the library was not built


def need_host_gb(gb):
    import psutil
    avail = psutil.virtual_memory().available / 2**30
    if avail < gb:
        pytest.skip(f"needs ~{gb} GiB of free host memory for the oracle, {avail:.0f} GiB free")


def need_device_gb(gb):
    free, _ = torch.cuda.mem_get_info()
    if free / 2**30 < gb:
        pytest.skip(f"needs ~{gb} GiB of free device memory, {free / 2**30:.0f} GiB free")


def sha(b):
    return hashlib.sha256(b).hexdigest()


def qwen_shapes(layers, d, q_heads, kv_heads, hd, ffn, vocab, tied):
    import bench
    return bench.qwen_shapes(layers, d, q_heads, kv_heads, hd, ffn, vocab, tied=tied)


def model_chain(shapes, steps, lr, seed=0):
    """Chained (prev, cur) broadcasts of fp32 master weights on the GPU: m ~ N(0, 0.02) (norm
    weights 1 + N(0, 1e-3)); each step m += lr * clip(N(0, 1), +-3) and the broadcast is bf16(m)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    master = {}
    for name, shape in shapes.items():
        if "norm" in name:
            master[name] = 1.0 + 1e-3 * torch.randn(shape, device="cuda", generator=g)
        else:
            master[name] = 0.02 * torch.randn(shape, device="cuda", generator=g)
    prev = {k: v.bfloat16() for k, v in master.items()}
    for _ in range(steps):
        for k in master:
            master[k].add_(torch.randn(master[k].shape, device="cuda", generator=g).clamp_(-3, 3), alpha=lr)
        cur = {k: v.bfloat16() for k, v in master.items()}
        yield prev, cur
        prev = cur


def run_chain(shapes, steps, lr):
    """Every step: CUDA update == oracle update (bytes), equal sender caches, receiver == sender."""
    import crukx_sync_b200 as crx
    from oracle import oracle
    sender, o_sender, receiver = {}, {}, {}
    recv = None
    host_prev = None
    for k, (prev, cur) in enumerate(model_chain(shapes, steps, lr)):
        if recv is None:
            recv = {n: v.clone() for n, v in prev.items()}
            host_prev = {n: v.cpu() for n, v in prev.items()}
        host_cur = {n: v.cpu() for n, v in cur.items()}
        upd = crx.encode_update(prev, cur, sender)
        want = oracle.encode_update(host_prev, host_cur, o_sender)
        assert (len(upd), sha(upd)) == (len(want), sha(want)), f"step {k}: update differs from the oracle"
        assert sender == o_sender, f"step {k}: sender caches differ"
        st = crx.apply_update(recv, upd, receiver)
        changed = sum(int((prev[n].view(torch.int16) != cur[n].view(torch.int16)).sum()) for n in cur)
        assert st.changed == changed
        for n in cur:
            assert torch.equal(recv[n], cur[n]), f"step {k}: {n} differs after apply"
        host_prev = host_cur
    return sender


def test_qwen15b_seven_chained_steps():
    need_device_gb(30)
    need_host_gb(24)
    shapes = qwen_shapes(28, 1536, 12, 2, 128, 8960, 151936, tied=True)
    assert sum(int(torch.tensor(s).prod()) for s in shapes.values()) == 1_543_714_304
    run_chain(shapes, steps=7, lr=1e-6)
    torch.cuda.empty_cache()


def test_qwen32b_tp8_shard():
    need_device_gb(70)
    need_host_gb(60)
    import bench
    shapes = bench.tp8_shard(qwen_shapes(64, 5120, 40, 8, 128, 27648, 152064, tied=False))
    assert shapes["model.layers.0.self_attn.q_proj.weight"] == (640, 5120)
    assert shapes["model.layers.0.self_attn.o_proj.weight"] == (5120, 640)
    assert shapes["model.layers.0.mlp.down_proj.weight"] == (5120, 3456)
    assert shapes["lm_head.weight"] == (19008, 5120)
    run_chain(shapes, steps=2, lr=1e-6)
    torch.cuda.empty_cache()


def heavy_tail_device(n, frac, seed, single_group=False):
    """prev ~ N(0, 0.02) (or every element in [1, 2): one exponent group); a fraction `frac` of
    the elements changes by a heavy-tailed number of ULPs: 85% +-1, 10% +-(2..7), 5% +-(8..1023),
    a third of the last also with the sign bit flipped.  Generated on the GPU (seeded)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    if single_group:
        prev = (1.0 + torch.rand(n, device="cuda", generator=g)).bfloat16()
    else:
        prev = (0.02 * torch.randn(n, device="cuda", generator=g)).bfloat16()
    a = prev.view(torch.int16)
    del prev
    if frac >= 1.0:
        sel = None
    else:
        sel = torch.rand(n, device="cuda", generator=g) < frac
    u = torch.rand(n, device="cuda", generator=g)
    mag = torch.ones(n, dtype=torch.int32, device="cuda")
    mid = (u >= 0.85) & (u < 0.95)
    mag = torch.where(mid, torch.randint(2, 8, (n,), device="cuda", generator=g, dtype=torch.int32), mag)
    big = u >= 0.95
    del u
    mag = torch.where(big, torch.randint(8, 1 << 10, (n,), device="cuda", generator=g, dtype=torch.int32), mag)
    sgn = torch.randint(0, 2, (n,), device="cuda", generator=g, dtype=torch.int32) * 2 - 1
    vals = a.to(torch.int32) + sgn * mag
    del sgn, mag
    flip = big & (torch.rand(n, device="cuda", generator=g) < 0.3)
    del big
    vals = torch.where(flip, a.to(torch.int32) ^ -0x8000, vals)
    del flip
    vals = ((vals + 0x8000) & 0xFFFF) - 0x8000
    b = vals.to(torch.int16)
    del vals
    if sel is not None:
        b = torch.where(sel, b, a)
        del sel
    else:
        same = b == a          # a wrap back to the same bits would be no change
        b = torch.where(same, a ^ 1, b)
        del same
    torch.cuda.empty_cache()
    return a, b


def run_flat(n, frac, seed, single_group=False):
    import crukx_sync_b200 as crx
    from oracle import oracle
    a, b = heavy_tail_device(n, frac, seed, single_group)
    changed = int((a != b).sum())
    if frac >= 1.0:
        assert changed == n
    sender, o_sender, receiver = {}, {}, {}
    upd = crx.encode_update({"flat": a}, {"flat": b}, sender)
    ha, hb = a.cpu(), b.cpu()
    want = oracle.encode_update({"flat": ha}, {"flat": hb}, o_sender)
    del ha, hb
    assert (len(upd), sha(upd)) == (len(want), sha(want)), "update differs from the oracle"
    assert sender == o_sender
    del want
    w = {"flat": a.clone()}
    st = crx.apply_update(w, upd, receiver)
    assert st.changed == changed
    assert torch.equal(w["flat"], b)
    assert receiver["flat"][0] == sender["flat"]
    del a, b, w
    torch.cuda.empty_cache()


@pytest.mark.parametrize("frac", [0.001, 0.01, 0.03, 0.10, 1.0])
def test_stress_2pow28_heavy_tail(frac):
    need_device_gb(30)
    need_host_gb(16)
    run_flat(1 << 28, frac, seed=11)


def test_stress_2pow28_single_group():
    need_device_gb(30)
    need_host_gb(16)
    run_flat(1 << 28, 0.10, seed=12, single_group=True)


@pytest.mark.parametrize("frac", [0.01, 1.0])
def test_stress_2pow31_heavy_tail(frac):
    """2^31 elements: positions, ranks and checksum weights past 2^31 on both sides."""
    need_device_gb(150)
    need_host_gb(80 if frac >= 1.0 else 24)
    run_flat(1 << 31, frac, seed=13)
