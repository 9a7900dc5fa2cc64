"""The reference-side binding printed in INTEGRATION.md §4, executed as written inside the installed
reference package (baseline/_ref): its two code blocks become crukx_sync._b200 and the patched
crukx_sync.encode_update / apply_update.  The patched reference must produce the bytes of its own
CPU path and of crukx_sync_b200, apply them bit-exactly with its own UpdateStats, keep the cache
rules, and raise its own CorruptUpdate for a corrupted update with nothing written.  Skipped when
the reference is not installed beside this repository."""

import os
import re
import sys
import types

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.path.join(ROOT, "baseline", "_ref")


def blocks():
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    sec = text[text.index("## 4."):text.index("## 5.")]
    return re.findall(r"```python\n(.*?)```", sec, re.S)


@pytest.fixture(scope="module")
def ref():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    if not os.path.exists(os.path.join(REF, "crukx_sync", "__init__.py")):
        pytest.skip("the reference package is not installed at baseline/_ref")
    from crukx_sync_b200 import _ext
    os.environ["CRUKX_B200_LIB"] = _ext.LIB_PATH
    saved = {k: v for k, v in sys.modules.items() if k == "crukx_sync" or k.startswith("crukx_sync.")}
    for k in saved:
        del sys.modules[k]
    sys.path.insert(0, REF)
    try:
        import crukx_sync
        mod_src, init_src = blocks()
        b200 = types.ModuleType("crukx_sync._b200")
        b200.__package__ = "crukx_sync"
        sys.modules["crukx_sync._b200"] = b200
        exec(compile(mod_src, "INTEGRATION.md:_b200.py", "exec"), b200.__dict__)
        crukx_sync._b200 = b200
        cpu_encode, cpu_apply = crukx_sync.encode_update, crukx_sync.apply_update
        exec(compile(init_src, "INTEGRATION.md:__init__.py", "exec"), crukx_sync.__dict__)
        assert crukx_sync.encode_update is not cpu_encode
        yield crukx_sync, cpu_encode, cpu_apply
    finally:
        sys.path.remove(REF)
        for k in [k for k in sys.modules if k == "crukx_sync" or k.startswith("crukx_sync.")]:
            del sys.modules[k]
        sys.modules.update(saved)


def states(seed=0, n=300_000):
    g = torch.Generator().manual_seed(seed)
    m = 0.02 * torch.randn(n, generator=g)
    a = m.bfloat16()
    b = (m + 2e-5 * torch.randn(n, generator=g).clamp(-3, 3)).bfloat16()
    return {"w": a.view(600, 500), "b": a[:777].clone()}, {"w": b.view(600, 500), "b": b[:777].clone()}


def test_patched_reference_matches_its_cpu_path_and_this_package(ref):
    crukx_sync, cpu_encode, _ = ref
    import crukx_sync_b200
    old, new = states()
    want = cpu_encode(old, new)                       # the reference's own torch code on CPU
    go, gn = {k: v.cuda() for k, v in old.items()}, {k: v.cuda() for k, v in new.items()}
    s1, s2 = {}, {}
    got = crukx_sync.encode_update(go, gn, s1)        # the patched reference, through _b200
    assert got == want == crukx_sync_b200.encode_update(go, gn, s2)
    assert s1 == s2
    w, rc = {k: v.clone() for k, v in go.items()}, {}
    st = crukx_sync.apply_update(w, got, rc)
    assert isinstance(st, crukx_sync.UpdateStats)
    assert (st.tensors, st.changed, st.bytes) == (2, sum(int((old[k].view(torch.int16) != new[k].view(torch.int16)).sum())
                                                          for k in old), len(got))
    for k in new:
        assert torch.equal(w[k].cpu().view(torch.int16), new[k].view(torch.int16))
    # chained: the next update through both caches
    m2 = {k: (v.float() + 3e-5).bfloat16() for k, v in gn.items()}
    u2 = crukx_sync.encode_update(gn, m2, s1)
    crukx_sync.apply_update(w, u2, rc)
    for k in m2:
        assert torch.equal(w[k], m2[k])


def test_patched_reference_rejects_a_corrupt_update_and_writes_nothing(ref):
    crukx_sync, _, _ = ref
    old, new = states(1)
    go, gn = {k: v.cuda() for k, v in old.items()}, {k: v.cuda() for k, v in new.items()}
    upd = bytearray(crukx_sync.encode_update(go, gn))
    upd[len(upd) // 2] ^= 0xFF
    w = {k: v.clone() for k, v in go.items()}
    with pytest.raises(crukx_sync.CorruptUpdate):
        crukx_sync.apply_update(w, bytes(upd))
    for k in go:
        assert torch.equal(w[k], go[k])
    with pytest.raises(ValueError):
        crukx_sync.apply_update({"w": go["w"]}, crukx_sync.encode_update(go, gn))   # receiver lacks "b"
