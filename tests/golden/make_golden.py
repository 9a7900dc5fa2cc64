"""Generate the golden fixtures in this directory by running the REAL reference implementation
(crukx-sync, pure Python + torch, imported unchanged from its source tree) on the seeded inputs
of tests/cases.py.

    python tests/golden/make_golden.py /path/to/crukx-sync/src

Writes:
  manifest.json   per case and step: SHA-256 of the inputs, the update's length and SHA-256,
                  UpdateStats, and the sender checksum cache after the step
  <case>_<step>.bin  the update bytes themselves when they are at most 64 KiB
  flips.json      for every single-byte corruption (xor 0x01/0x80/0xFF) of one small update, what
                  the reference's apply_update did: "ok", "CorruptUpdate" or "ValueError"

The fixtures pin the CPU oracle and the CUDA path to the reference's own output; nothing at test
time reads the reference source.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))   # tests/ for cases.py

import torch  # noqa: E402

import cases  # noqa: E402
import hostile  # noqa: E402

SMALL = 64 * 1024


def main(ref_src: str, only: list[str] | None = None):
    sys.path.insert(0, ref_src)
    import crukx_sync as ref  # the reference, unchanged

    torch.set_num_threads(os.cpu_count() or 1)
    path = os.path.join(HERE, "manifest.json")
    manifest = json.load(open(path)) if os.path.exists(path) else {}
    for name, (fn, chained) in cases.CASES.items():
        if only and name not in only:
            continue
        t0 = time.time()
        steps = fn()
        sender, receiver = ({}, {}) if chained else (None, None)
        recv = None
        rows = []
        for k, (old, new) in enumerate(steps):
            upd = ref.encode_update(old, new, sender)
            if recv is None or not chained:
                recv = {n: v.clone() for n, v in old.items()}
            stats = ref.apply_update(recv, upd, receiver)
            for n in new:
                assert torch.equal(recv[n].view(torch.int16), new[n].view(torch.int16)), (name, k, n)
            row = {
                "inputs_sha256": cases.digest_inputs(old, new),
                "update_len": len(upd),
                "update_sha256": hashlib.sha256(upd).hexdigest(),
                "tensors": stats.tensors,
                "changed": stats.changed,
                "sender_checksums": {n: str(v) for n, v in (sender or {}).items()},
            }
            if len(upd) <= SMALL:
                fname = f"{name}_{k}.bin"
                with open(os.path.join(HERE, fname), "wb") as f:
                    f.write(upd)
                row["file"] = fname
            rows.append(row)
        manifest[name] = {"chained": chained, "steps": rows}
        print(f"{name}: {len(steps)} step(s), {[r['update_len'] for r in rows]} bytes, {time.time() - t0:.1f}s",
              flush=True)
    with open(path, "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)

    if not only or "hostile" in only:
        rows = {}
        for label, make_w, data in hostile.cases():
            w = make_w()
            before = {k: v.clone() for k, v in w.items()}
            t = time.time()
            rows[label] = _verdict(ref, w, data)
            assert all(torch.equal(w[k], before[k]) for k in w), label
            print(f"hostile {label}: {rows[label]} ({time.time() - t:.2f}s)", flush=True)
        old, new = cases.case_multi()[0]
        upd = ref.encode_update(old, new)
        pref = []
        for p in hostile.prefixes(upd):
            w = {k: v.clone() for k, v in old.items()}
            pref.append(_verdict(ref, w, p))
        with open(os.path.join(HERE, "hostile.json"), "w") as f:
            json.dump({"cases": rows, "multi_prefix_verdicts": "".join(v[0] for v in pref)}, f, indent=1)

    if only and "flips" not in only:
        return
    a, b = cases.flip_case()
    upd = ref.encode_update({"w": a}, {"w": b})
    verdicts = []
    for i in range(len(upd)):
        for x in (0x01, 0x80, 0xFF):
            bad = bytearray(upd)
            bad[i] ^= x
            w = {"w": a.clone()}
            try:
                ref.apply_update(w, bytes(bad))
                assert torch.equal(w["w"].view(torch.int16), b.view(torch.int16))
                verdicts.append("ok")
            except ref.CorruptUpdate:
                assert torch.equal(w["w"].view(torch.int16), a.view(torch.int16))
                verdicts.append("CorruptUpdate")
            except ValueError:
                assert torch.equal(w["w"].view(torch.int16), a.view(torch.int16))
                verdicts.append("ValueError")
    with open(os.path.join(HERE, "flips.json"), "w") as f:
        json.dump({"inputs_sha256": cases.digest_inputs({"w": a}, {"w": b}),
                   "update_hex": upd.hex(), "xors": [1, 128, 255], "verdicts": verdicts}, f, indent=0)
    print(f"flips: {len(verdicts)} corruptions, {verdicts.count('ok')} still decode")


def _verdict(ref, w, data):
    try:
        ref.apply_update(w, data)
        return "ok"
    except ref.CorruptUpdate:
        return "CorruptUpdate"
    except ValueError:
        return "ValueError"


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2:] or None)
