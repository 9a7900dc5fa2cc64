"""Seeded synthetic inputs shared by the golden-fixture script, the CPU oracle tests and the GPU
parity tests.  Every generator uses a CPU ``torch.Generator`` so the same seed gives the same
bits on any machine with this torch build; the fixtures also record a SHA-256 of every input so
drift is detected instead of silently comparing different data.

A case is a list of steps; each step is ``(old, new)``, two dicts name -> CPU tensor (bf16 or
int16 bit patterns).  ``chained`` cases are run with sender/receiver checksum caches kept across
steps, the way a trainer and a worker use the library.
"""

from __future__ import annotations

import hashlib

import torch


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def rl_pair(n: int, lr: float = 1e-6, seed: int = 0):
    """bf16 weights N(0, 0.02) and the next broadcast after one sign step of size lr*U(0.5, 1.5)."""
    g = _gen(seed)
    w = torch.randn(n, generator=g) * 0.02
    step = lr * torch.sign(torch.randn(n, generator=g)) * (0.5 + torch.rand(n, generator=g))
    return w.bfloat16(), (w + step).bfloat16()


def adam_chain(shapes: dict, steps: int, lr: float, seed: int = 0, norm_suffix: str = "norm"):
    """Chained bf16 broadcasts of fp32 master weights: m ~ N(0, 0.02) (norm weights 1 + N(0, 1e-3)),
    each step m += lr * clip(N(0, 1), +-3); the broadcast is bf16(m)."""
    g = _gen(seed)
    master = {}
    for name, shape in shapes.items():
        if norm_suffix in name:
            master[name] = 1.0 + 1e-3 * torch.randn(shape, generator=g)
        else:
            master[name] = 0.02 * torch.randn(shape, generator=g)
    out = []
    prev = {k: v.bfloat16() for k, v in master.items()}
    for _ in range(steps):
        for k in master:
            master[k] += lr * torch.randn(master[k].shape, generator=g).clamp_(-3, 3)
        cur = {k: v.bfloat16() for k, v in master.items()}
        out.append((prev, cur))
        prev = cur
    return out


def heavy_tail(n: int, frac: float, seed: int, single_group: bool = False):
    """prev ~ N(0, 0.02) (or one exponent group); a fraction `frac` changes with a heavy-tailed
    delta in ULPs: 85% +-1, 10% +-(2..7), 5% up to +-2^10, and within that 5% sign flips."""
    g = _gen(seed)
    if single_group:
        prev = (1.0 + torch.rand(n, generator=g)).bfloat16()          # all in [1, 2): exponent 127
    else:
        prev = (0.02 * torch.randn(n, generator=g)).bfloat16()
    a = prev.view(torch.int16).clone()
    if frac >= 1.0:
        idx = torch.arange(n)
    else:
        idx = torch.randperm(n, generator=g)[: max(1, int(n * frac))]
    m = idx.numel()
    u = torch.rand(m, generator=g)
    sgn = torch.where(torch.rand(m, generator=g) < 0.5, -1, 1)
    mag = torch.ones(m, dtype=torch.int32)
    mid = (u >= 0.85) & (u < 0.95)
    mag[mid] = torch.randint(2, 8, (int(mid.sum()),), generator=g, dtype=torch.int32)
    big = u >= 0.95
    mag[big] = torch.randint(8, 1 << 10, (int(big.sum()),), generator=g, dtype=torch.int32)
    vals = a[idx].to(torch.int32) + sgn * mag
    flip = big & (torch.rand(m, generator=g) < 0.3)
    vals = torch.where(flip, a[idx].to(torch.int32) ^ -0x8000, vals)   # sign flip
    vals = ((vals + 0x8000) & 0xFFFF) - 0x8000
    b = a.clone()
    b[idx] = vals.to(torch.int16)
    if frac >= 1.0:                      # a wrap back to the same bits would be no change
        same = b == a
        b[same] = a[same] ^ 1
    return a, b


# ---------------------------------------------------------------- named cases


def case_rl_200k():
    a, b = rl_pair(200_000)
    return [({"w": a.view(400, 500)}, {"w": b.view(400, 500)})]


def case_multi():
    a, b = rl_pair(50_000, seed=1)
    return [({"a": a, "same": a.clone(), "c": a[:777].clone()},
             {"a": b, "same": a.clone(), "c": b[:777].clone()})]


def case_arbitrary():
    g = _gen(2)
    a = torch.randint(-32768, 32768, (5000,), generator=g, dtype=torch.int16)
    b = a ^ torch.randint(1, 32768, (5000,), generator=g, dtype=torch.int16)
    return [({"w": a}, {"w": b})]


def case_one_group_wide():
    a = torch.full((200_000,), 0x3C00, dtype=torch.int16)
    b = torch.randint(-32768, 32768, (200_000,), generator=_gen(4), dtype=torch.int16)
    return [({"w": a}, {"w": b})]


def case_rice_dense():
    a = torch.full((1 << 20,), 0x3F80, dtype=torch.int16)
    b = a.clone()
    b[:4096] += 1
    return [({"w": a}, {"w": b})]


def case_rice_tail():
    a = torch.full((1 << 20,), 0x3F80, dtype=torch.int16)
    b = a.clone()
    b[-1] += 1
    return [({"w": a}, {"w": b})]


def case_single():
    return [({"w": torch.tensor([0x3F80], dtype=torch.int16)}, {"w": torch.tensor([0x3F81], dtype=torch.int16)})]


def case_extreme():
    a = torch.tensor([0x7FFF, -0x8000, 0, 0x7FFF], dtype=torch.int16)
    b = torch.tensor([-0x8000, 0x7FFF, 0x7FFF, 0], dtype=torch.int16)
    return [({"w": a}, {"w": b})]


def case_long_unary():
    a = torch.full((1 << 20,), 0x3F80, dtype=torch.int16)
    b = a.clone()
    b[:2000] += 1
    b[-1] += 1
    return [({"w": a}, {"w": b})]


def case_no_change():
    a, _ = rl_pair(1000)
    return [({"w": a}, {"w": a.clone()})]


def case_empty():
    return [({}, {})]


def case_chain5():
    g = _gen(7)
    w = torch.randn(300_000, generator=g) * 0.02
    steps, prev = [], {"w": w.bfloat16()}
    for _ in range(5):
        w = w + 1e-6 * torch.sign(torch.randn(w.shape, generator=g))
        cur = {"w": w.bfloat16()}
        steps.append((prev, cur))
        prev = cur
    return steps


def case_heavy_10pct():
    a, b = heavy_tail(1 << 20, 0.10, seed=21)
    return [({"flat": a}, {"flat": b})]


def case_heavy_100pct():
    a, b = heavy_tail(1 << 18, 1.0, seed=22)
    return [({"flat": a}, {"flat": b})]


def case_single_group():
    a, b = heavy_tail(1 << 20, 0.01, seed=23, single_group=True)
    return [({"flat": a}, {"flat": b})]


def case_many_small():
    g = _gen(31)
    old, new = {}, {}
    for i in range(300):
        n = int(torch.randint(1, 5000, (1,), generator=g))
        a, b = rl_pair(n, lr=5e-5, seed=1000 + i)
        old[f"t{i:03d}"] = a
        new[f"t{i:03d}"] = b if i % 7 else a.clone()
    return [(old, new)]


def case_multislab():
    a, b = rl_pair((1 << 24) + 4099, lr=3e-6, seed=41)
    return [({"big": a}, {"big": b})]


def toy_decoder_shapes(layers=4, d=1024, heads=16, hd=64, ffn=2816, vocab=32768):
    """a 4-layer decoder, tied embedding, RMSNorm weights."""
    s = {"model.embed_tokens.weight": (vocab, d)}
    for i in range(layers):
        p = f"model.layers.{i}."
        s[p + "input_layernorm.weight"] = (d,)
        s[p + "self_attn.q_proj.weight"] = (heads * hd, d)
        s[p + "self_attn.k_proj.weight"] = (heads * hd, d)
        s[p + "self_attn.v_proj.weight"] = (heads * hd, d)
        s[p + "self_attn.o_proj.weight"] = (d, heads * hd)
        s[p + "post_attention_layernorm.weight"] = (d,)
        s[p + "mlp.gate_proj.weight"] = (ffn, d)
        s[p + "mlp.up_proj.weight"] = (ffn, d)
        s[p + "mlp.down_proj.weight"] = (d, ffn)
    s["model.norm.weight"] = (d,)
    return s


def case_toy_decoder():
    return adam_chain(toy_decoder_shapes(), steps=3, lr=1e-6, seed=0)


CASES = {
    "rl_200k": (case_rl_200k, False),
    "multi": (case_multi, False),
    "arbitrary": (case_arbitrary, False),
    "one_group_wide": (case_one_group_wide, False),
    "rice_dense": (case_rice_dense, False),
    "rice_tail": (case_rice_tail, False),
    "single": (case_single, False),
    "extreme": (case_extreme, False),
    "long_unary": (case_long_unary, False),
    "no_change": (case_no_change, False),
    "empty": (case_empty, False),
    "chain5": (case_chain5, True),
    "heavy_10pct": (case_heavy_10pct, False),
    "heavy_100pct": (case_heavy_100pct, False),
    "single_group": (case_single_group, False),
    "many_small": (case_many_small, False),
    "multislab": (case_multislab, False),
    "toy_decoder": (case_toy_decoder, True),
}

# cases small enough for the quick CPU suite (the others run in the GPU suite / marked slow)
QUICK = ["rl_200k", "multi", "arbitrary", "one_group_wide", "rice_dense", "rice_tail", "single",
         "extreme", "long_unary", "no_change", "empty", "chain5", "heavy_10pct", "heavy_100pct",
         "single_group", "many_small"]


def digest_inputs(old: dict, new: dict) -> str:
    h = hashlib.sha256()
    for d in (old, new):
        for k, v in d.items():
            h.update(k.encode())
            h.update(v.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def flip_case():
    """The small update whose every single-byte corruption is replayed against the reference."""
    return rl_pair(3000, seed=6)
