#!/usr/bin/env python
"""Benchmark: encode & apply GB/s of bf16 weights on Qwen2.5-7B-shaped random-init weights.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 7b|1.5b|toy|32b-tp8]

One step = one weight sync through the public API: ``encode_update(prev, cur, send_chk)`` then
``apply_update(recv, update, recv_chk)``, checksum caches kept.  The synthetic workload follows
fp32 master weights m ~ N(0, 0.02) (norm weights 1 + N(0, 1e-3)); one
Adam-like step m += lr * clip(N(0,1), +-3) with lr = 2e-6; prev = bf16(m_before), cur =
bf16(m_after).  Timed steps alternate prev->cur and cur->prev (the same change statistics every
step, caches stay valid), so all K steps run back to back between two barriers.  Every state is
15 GB, far larger than L2, so no flush is needed between steps.

N > 1 (torchrun): tensors are partitioned by LPT on numel; each rank encodes its partition, the
compressed payloads are all-gathered over NCCL (their sizes between the hosts over gloo), and each
rank applies its own partition's update taken from the gathered buffer (the headline's receiver).
The reported time is the max over ranks.  Beside the headline the line carries:
  roofline_step   whole encode and whole apply against the HBM roofline, per GPU
  full_replica    (N > 1) every rank applies all N gathered updates to a whole copy of the model
  tp8_32b         BASELINE config 4: each rank encodes and applies its own 32B 8-way TP shard
  parity          the first update's SHA-256 against the CPU oracle's whole-dict update
  cpu_baseline    the oracle port on the host cores, and the reference's own torch code beside it
  reference_gpu   the reference's own GPU path (torch CUDA + Triton) on the same GPU (secondary)
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "encode & apply GB/s of bf16 weights (7B shape, 1/8 B200); bytes/changed wt"


# ---------------------------------------------------------------- workloads

def qwen_shapes(layers, d, q_heads, kv_heads, hd, ffn, vocab, tied, bias=True):
    s = {"model.embed_tokens.weight": (vocab, d)}
    for i in range(layers):
        p = f"model.layers.{i}."
        s[p + "self_attn.q_proj.weight"] = (q_heads * hd, d)
        s[p + "self_attn.k_proj.weight"] = (kv_heads * hd, d)
        s[p + "self_attn.v_proj.weight"] = (kv_heads * hd, d)
        if bias:
            s[p + "self_attn.q_proj.bias"] = (q_heads * hd,)
            s[p + "self_attn.k_proj.bias"] = (kv_heads * hd,)
            s[p + "self_attn.v_proj.bias"] = (kv_heads * hd,)
        s[p + "self_attn.o_proj.weight"] = (d, q_heads * hd)
        s[p + "mlp.gate_proj.weight"] = (ffn, d)
        s[p + "mlp.up_proj.weight"] = (ffn, d)
        s[p + "mlp.down_proj.weight"] = (d, ffn)
        s[p + "input_layernorm.weight"] = (d,)
        s[p + "post_attention_layernorm.weight"] = (d,)
    s["model.norm.weight"] = (d,)
    if not tied:
        s["lm_head.weight"] = (vocab, d)
    return s


def tp8_shard(shapes):
    """One of 8 tensor-parallel shards: column-split q/k/v/gate/up (+ vocab), row-split o/down."""
    out = {}
    for n, sh in shapes.items():
        if any(k in n for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj", "embed_tokens", "lm_head")):
            out[n] = (sh[0] // 8,) + tuple(sh[1:])
        elif any(k in n for k in ("o_proj", "down_proj")):
            out[n] = (sh[0], sh[1] // 8)
        else:
            out[n] = sh
    return out


CONFIGS = {
    "7b": dict(shapes=lambda: qwen_shapes(28, 3584, 28, 4, 128, 18944, 152064, tied=False), lr=2e-6,
               name="qwen2.5-7b-shape"),
    "1.5b": dict(shapes=lambda: qwen_shapes(28, 1536, 12, 2, 128, 8960, 151936, tied=True), lr=1e-6,
                 name="qwen2.5-1.5b-shape"),
    "toy": dict(shapes=lambda: qwen_shapes(4, 1024, 16, 16, 64, 2816, 32768, tied=True, bias=False), lr=1e-6,
                name="toy-4l-d1024"),
    # two decoder layers of the 7B shape (0.47B params): the small case for ncu captures
    "7b-2l": dict(shapes=lambda: qwen_shapes(2, 3584, 28, 4, 128, 18944, 152064, tied=True, bias=True) | {},
                  lr=2e-6, name="qwen2.5-7b-shape-2-layers", drop_embed=True),
    "32b-tp8": dict(shapes=lambda: tp8_shard(qwen_shapes(64, 5120, 40, 8, 128, 27648, 152064, tied=False)), lr=1e-6,
                    name="qwen2.5-32b-shape-tp8-shard"),
}


def make_states(shapes, lr, device, seed=0):
    """(prev, cur) bf16 dicts on `device` for one Adam-like step of the fp32 master weights."""
    g = torch.Generator(device=device).manual_seed(seed)
    prev, cur = {}, {}
    for name, shape in shapes.items():
        if "norm" in name:
            m = 1.0 + 1e-3 * torch.randn(shape, device=device, generator=g)
        else:
            m = 0.02 * torch.randn(shape, device=device, generator=g)
        prev[name] = m.bfloat16()
        m.add_(torch.randn(shape, device=device, generator=g).clamp_(-3, 3), alpha=lr)
        cur[name] = m.bfloat16()
        del m
    return prev, cur


# ---------------------------------------------------------------- clocks during the timed region

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.dev)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- our arm

def measured_peak():
    try:
        j = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(j["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def kernel_times(ctx):
    from crukx_sync_b200 import _ext
    L = _ext.load()
    names = ctypes.create_string_buffer(8192)
    ms = (ctypes.c_double * 64)()
    cnt = (ctypes.c_int32 * 64)()
    n = L.crx_ctx_kernel_times(ctx, names, 8192, ms, cnt, 64)
    out = {}
    for i, nm in enumerate(names.value.decode().split("\n")[:n]):
        out[nm] = (ms[i], cnt[i])
    return out


def kernel_gaps(ctx):
    """Per kernel: ms its stream sat idle before it (host work and round trips in between)."""
    from crukx_sync_b200 import _ext
    L = _ext.load()
    names = ctypes.create_string_buffer(8192)
    ms = (ctypes.c_double * 64)()
    n = L.crx_ctx_kernel_gaps(ctx, names, 8192, ms, 64)
    return {nm: ms[i] for i, nm in enumerate(names.value.decode().split("\n")[:n])}


def cpu_baseline_sample(shapes, lr, budget_elems, seed=1):
    """A bounded sample of the workload (whole tensors, in order, up to budget) on the CPU."""
    names, tot = [], 0
    for k, sh in shapes.items():
        n = int(torch.tensor(sh).prod())
        if tot + n > budget_elems:
            continue
        names.append(k)
        tot += n
        if tot >= budget_elems:
            break
    sub = {k: shapes[k] for k in names}
    prev, cur = make_states(sub, lr, "cpu", seed=seed)
    return prev, cur, tot


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def time_oracle(prev, cur, steps=1, threads=None, warmup=0, whole=False):
    """The CPU oracle (the C restatement of the reference) on one sample, on every host thread.
    Default: tensors cut into pieces of at most 2^24 elements, one update per piece, the pieces
    spread over a thread pool (the C calls release the GIL) -- the per-element work of the
    reference with the parallelism of a CPU implementation that splits large tensors.
    whole=True: one whole-dict update per step, the oracle's per-tensor and per-exponent passes on
    the threads (a step then waits for its largest tensor on one thread).  `warmup` untimed steps
    come first.  Returns seconds per timed step (encode + apply) and the threads used."""
    import concurrent.futures

    from oracle import oracle
    threads = threads or host_threads()
    sender, receiver = {}, {}
    recv = {k: v.clone() for k, v in prev.items()}
    state = {"a": prev, "b": cur}
    if whole:
        oracle.set_threads(threads)

        def run_step():
            upd = oracle.encode_update(state["a"], state["b"], sender)
            oracle.apply_update(recv, upd, receiver)
    else:
        oracle.set_threads(1)
        piece = 1 << 24
        pieces = [(k, a, min(a + piece, prev[k].numel())) for k in prev for a in range(0, prev[k].numel(), piece)]
        pieces.sort(key=lambda p: p[1] - p[2])   # big pieces first: better balance
        pool = concurrent.futures.ThreadPoolExecutor(max_workers=threads)

        def one(p):
            k, lo, hi = p
            name = f"{k}#{lo}"
            upd = oracle.encode_update({name: state["a"][k].view(-1)[lo:hi]}, {name: state["b"][k].view(-1)[lo:hi]},
                                       sender)
            oracle.apply_update({name: recv[k].view(-1)[lo:hi]}, upd, receiver)

        def run_step():
            list(pool.map(one, pieces))
    times = []
    try:
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            run_step()
            if i >= warmup:
                times.append(time.perf_counter() - t0)
            state["a"], state["b"] = state["b"], state["a"]
    finally:
        if not whole:
            pool.shutdown()
        oracle.set_threads(0)
    for k in recv:   # the oracle reproduced the sender's state
        assert torch.equal(recv[k], state["a"][k]), k
    return sum(times) / len(times), threads


def reference_src():
    """Import path of the reference package installed beside this repository (baseline/_ref), or
    None when it is not there."""
    p = os.path.join(ROOT, "baseline", "_ref")
    return p if os.path.exists(os.path.join(p, "crukx_sync", "__init__.py")) else None


def time_reference_torch(prev, cur, steps=1, threads=None):
    """The reference's own torch implementation (crukx_sync, unmodified, from baseline/_ref) on CPU
    tensors with every host thread: seconds per steady-state step (encode_update + apply_update,
    checksum caches kept, after one untimed step that fills them), or None without the package."""
    src = reference_src()
    if src is None:
        return None, 0
    if src not in sys.path:
        sys.path.insert(0, src)
    import crukx_sync as ref   # the reference, unchanged
    threads = threads or host_threads()
    torch.set_num_threads(threads)
    sender, receiver = {}, {}
    recv = {k: v.clone() for k, v in prev.items()}
    state = {"a": prev, "b": cur}
    times = []
    for i in range(1 + steps):
        t0 = time.perf_counter()
        upd = ref.encode_update(state["a"], state["b"], sender)
        ref.apply_update(recv, upd, receiver)
        if i >= 1:
            times.append(time.perf_counter() - t0)
        state["a"], state["b"] = state["b"], state["a"]
    for k in recv:
        assert torch.equal(recv[k].view(torch.int16), state["a"][k].view(torch.int16)), k
    return sum(times) / len(times), threads


def parity_check(A, B, threads):
    """The first step's update (no caches) through encode_update_device, against the CPU oracle's
    whole-dict update of the same state: SHA-256 of both.  Run once, outside the timed region.
    Raises when they differ: a wrong encoder produces no bench line."""
    import hashlib

    import psutil

    import crukx_sync_b200 as crx
    from oracle import oracle
    need = 2.6 * sum(v.numel() * 2 for v in A.values())   # host copies of both states + the oracle's lists
    if psutil.virtual_memory().available < need:
        return {"checked": False, "why": "not enough free host memory for the oracle"}
    t0 = time.perf_counter()
    dev_upd = crx.encode_update_device(A, B, None)
    ours = dev_upd.cpu().numpy().tobytes()
    del dev_upd
    hA = {k: v.cpu() for k, v in A.items()}
    hB = {k: v.cpu() for k, v in B.items()}
    oracle.set_threads(threads)
    want = oracle.encode_update(hA, hB)
    del hA, hB
    a, b = hashlib.sha256(ours).hexdigest(), hashlib.sha256(want).hexdigest()
    if (len(ours), a) != (len(want), b):
        raise AssertionError(f"update differs from the CPU oracle: {len(ours)} B {a[:16]} vs {len(want)} B {b[:16]}")
    return {"checked": True, "sha256": a, "bytes": len(ours), "result": "sha256 matches oracle",
            "what": "first update of this rank's tensors (no caches) vs the CPU oracle's whole-dict update of the "
                    "same state", "oracle_threads": threads, "seconds": round(time.perf_counter() - t0, 1)}


def log(*a):
    if os.environ.get("CRUKX_B200_TRACE"):
        print(f"[bench {time.strftime('%H:%M:%S')}]", *a, file=sys.stderr, flush=True)


def step_roofline(my_params, changed, upd_bytes, ms_enc, ms_app, peak):
    """Whole encode and whole apply of one rank against the HBM roofline: algorithmic bytes (encode:
    prev + cur, 4 B per element; apply: the old weights 2 B per element + the update + 2 B per
    changed element) over the rank's measured time."""
    enc_b = 4.0 * my_params
    app_b = 2.0 * my_params + upd_bytes + 2.0 * changed
    enc = enc_b / (ms_enc * 1e-3) / 1e9
    app = app_b / (ms_app * 1e-3) / 1e9
    return {"encode": {"achieved": round(enc, 1), "frac": round(enc / peak, 4), "algorithmic_bytes": enc_b},
            "apply": {"achieved": round(app, 1), "frac": round(app / peak, 4), "algorithmic_bytes": app_b},
            "peak": peak, "unit": "GB/s", "per": "GPU (max over ranks of its time)"}


def run_ours(args, rank, world, dist):
    import crukx_sync_b200 as crx
    from crukx_sync_b200 import _ext
    from crukx_sync_b200 import dist as cdist

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    shapes_all = cfg["shapes"]()
    if cfg.get("drop_embed"):
        shapes_all = {k: v for k, v in shapes_all.items() if "embed" not in k}
    if args.emulate:   # one rank's share of an N-way run, alone on this GPU (no exchange)
        er, en = (int(x) for x in args.emulate.split("/"))
        owner = cdist.partition({k: int(torch.tensor(v).prod()) for k, v in shapes_all.items()}, en)
        shapes_all = {k: v for k, v in shapes_all.items() if owner[k] == er}
    owner = cdist.partition({k: int(torch.tensor(v).prod()) for k, v in shapes_all.items()}, world)
    mine = [k for k in shapes_all if owner[k] == rank]
    total_params = sum(int(torch.tensor(s).prod()) for s in shapes_all.values())
    my_params = sum(int(torch.tensor(shapes_all[k]).prod()) for k in mine)
    # every rank holds the whole model's two states (same seed everywhere): its own tensors are the
    # partition it encodes and applies; the whole states serve the full-replica receiver
    log("generating", len(shapes_all), "tensors,", total_params, "params")
    A_full, B_full = make_states(shapes_all, cfg["lr"], dev, seed=0)
    A = {k: A_full[k] for k in mine}
    B = {k: B_full[k] for k in mine}
    log("generated")
    changed = sum(int((A[k].view(torch.int16) != B[k].view(torch.int16)).sum()) for k in A)
    parity = None
    if not args.no_parity:
        log("parity check against the oracle")
        parity = parity_check(A, B, max(1, host_threads() // max(world, 1)))
        log("parity", parity)
    size_cmp = None
    if world == 1:   # the same update in other sparse formats (the reference's bench/compare.py columns)
        from crukx_sync_b200 import sizes as csizes
        size_cmp = csizes.update_sizes(A, B)
    recv = {k: v.clone() for k, v in A.items()}
    sender, receiver = {}, {}
    ctx = _ext.context(dev.index)
    L = _ext.load()
    stream = torch.cuda.current_stream(dev)
    size_group = cdist.host_size_group() if dist is not None else None
    side = torch.cuda.Stream(dev)   # the all-gather runs here, beside the apply

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def exchange(upd, ranks=(rank,)):
        """All-gather of the device-resident updates over NCCL (sizes between the hosts); the
        requested ranks' updates from the gathered buffer."""
        return cdist.allgather_updates_device(upd, ranks=list(ranks), size_group=size_group)

    def start_exchange(upd):
        """The same all-gather on the side stream, overlapping the caller's next work (N > 1)."""
        if dist is None:
            return None
        return cdist.allgather_updates_device_async(upd, size_group=size_group, side_stream=side)

    state = {"src": A, "dst": B, "src_is_A": True}

    def flip():
        state["src"], state["dst"] = state["dst"], state["src"]
        state["src_is_A"] = not state["src_is_A"]

    def step(events=None):
        """One sync step with the updates resident in HBM: encode_update_device (the reference's
        bytes, in device memory); the NCCL all-gather that gives every rank every update, on a side
        stream while this rank applies its own update (which it holds); the step ends when both
        are done.  events: start, encode done, apply done, step done (gather included)."""
        src, dst = state["src"], state["dst"]
        if events:
            events[0].record(stream)
        upd = crx.encode_update_device(src, dst, sender)
        if events:
            events[1].record(stream)
        pg = start_exchange(upd)
        st = crx.apply_update(recv, upd, receiver)
        if events:
            events[2].record(stream)
        if pg is not None:
            pg.wait()
            if events is not None:
                gathers.append((events[1], pg.event))
        if events:
            events[3].record(stream)
        flip()
        return upd, st

    gathers = []   # (encode done, gather done) per timed step

    for i in range(args.warmup):
        log("warmup step", i)
        step()
    barrier()
    # correctness of the warm state before timing
    for k in recv:
        assert torch.equal(recv[k], state["src"][k]), f"receiver differs from the sender state: {k}"
    launches0 = L.crx_ctx_launches(ctx) + L.crx_parse_device_launches()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    sizes = []
    with ClockSampler(dev.index) as clk:
        barrier()
        t_wall0 = time.perf_counter()
        for k in range(args.steps):
            upd, st = step(evs[k])
            sizes.append(upd.numel())
        barrier()
        t_wall = time.perf_counter() - t_wall0
    launches = int(L.crx_ctx_launches(ctx) + L.crx_parse_device_launches() - launches0)   # + the device parses' table checks
    enc = [e[0].elapsed_time(e[1]) for e in evs]
    app = [e[1].elapsed_time(e[2]) for e in evs]
    tot = [e[0].elapsed_time(e[3]) for e in evs]
    # the gather: from the end of the encode to the end of the NCCL all-gather (it overlaps the apply)
    ex = [a.elapsed_time(b) for a, b in gathers[-args.steps:]] or [0.0]
    for k in recv:
        assert torch.equal(recv[k], state["src"][k]), f"receiver differs after timing: {k}"
    ms_step = sum(tot) / len(tot)
    ms_enc, ms_ex, ms_app = (sum(x) / len(x) for x in (enc, ex, app))
    my_upd = sum(sizes) / len(sizes)
    if dist is not None:
        t = torch.tensor([ms_step, ms_enc, ms_app, ms_ex], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step, ms_enc, ms_app, ms_ex = t.tolist()
        c = torch.tensor([changed, my_upd], dtype=torch.float64, device=dev)
        dist.all_reduce(c)
        changed_all, upd_bytes = c.tolist()
    else:
        changed_all, upd_bytes = changed, my_upd
    weight_bytes = 2.0 * total_params
    value = weight_bytes / (ms_step * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    # this rank's share against the slowest rank's time
    per_rank = step_roofline(my_params, changed, my_upd, ms_enc, ms_app, peak)
    per_rank["peak_kind"] = peak_kind

    # ---- the same steps through the host-bytes API (encode_update -> bytes -> apply_update), the
    #      reference's own interface: the update crosses PCIe twice; each rank applies its own
    #      update (no exchange of host bytes between processes)
    bytes_api = None
    if not args.no_bytes_api:
        def bstep(events):
            src, dst = state["src"], state["dst"]
            events[0].record(stream)
            u = crx.encode_update(src, dst, sender)
            events[1].record(stream)
            crx.apply_update(recv, u, receiver)
            events[2].record(stream)
            flip()

        for _ in range(2):
            bstep([torch.cuda.Event(enable_timing=True) for _ in range(3)])
        bevs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
        barrier()
        for k in range(args.steps):
            bstep(bevs[k])
        barrier()
        for k in recv:
            assert torch.equal(recv[k], state["src"][k]), f"receiver differs after the bytes API: {k}"
        bt = torch.tensor([sum(e[0].elapsed_time(e[2]) for e in bevs) / args.steps,
                           sum(e[0].elapsed_time(e[1]) for e in bevs) / args.steps,
                           sum(e[1].elapsed_time(e[2]) for e in bevs) / args.steps], dtype=torch.float64, device=dev)
        if dist is not None:
            dist.all_reduce(bt, op=dist.ReduceOp.MAX)
        b_step, b_enc, b_app = bt.tolist()
        bytes_api = {"value": round(2.0 * total_params / (b_step * 1e-3) / 1e9, 2), "unit": "GB/s",
                     "ms_per_step": round(b_step, 4), "encode_ms": round(b_enc, 4), "apply_ms": round(b_app, 4),
                     "note": "encode_update -> host bytes -> apply_update(bytes), weights resident in HBM"}

    # ---- per-kernel times on this stream (a separate profiled pass of 2 steps)
    L.crx_ctx_profile(ctx, 1)
    for _ in range(2):
        step()
    torch.cuda.synchronize(dev)
    kt = kernel_times(ctx)
    kg = kernel_gaps(ctx)
    L.crx_ctx_profile(ctx, 0)
    # k_map reads the old weights (2 B/element) and writes every changed element in place (2 B/change)
    algo = {"k_enc_rank": 4.0 * my_params, "k_map": 2.0 * my_params + 2.0 * changed, "k_app_hist": 2.0 * my_params}
    kernels = {}
    for nm, (ms, n) in sorted(kt.items(), key=lambda x: -x[1][0]):
        per = ms / max(n, 1)
        row = {"ms_per_launch": round(per, 4), "launches": n, "share": None,
               "idle_before_ms": round(kg.get(nm, 0.0) / max(n, 1), 4)}
        if nm in algo:
            row["algo_gbs"] = round(algo[nm] / (per * 1e-3) / 1e9, 1)
        kernels[nm] = row
    tot_k = sum(ms for ms, _ in kt.values()) or 1.0
    for nm in kernels:
        kernels[nm]["share"] = round(kt[nm][0] / tot_k, 4)
    dom = max(kt, key=lambda k: kt[k][0]) if kt else None
    roofline = None
    if dom in algo:
        per = kt[dom][0] / kt[dom][1]
        achieved = algo[dom] / (per * 1e-3) / 1e9
        traffic = None
        try:
            tj = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
            if dom in tj:
                traffic = tj[dom]["bytes_per_element"] * my_params
        except (OSError, KeyError, ValueError):
            pass
        roofline = {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                    "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                    "traffic_source": "scaled from profiles/traffic.json: ncu dram__bytes_read.sum + "
                                      "dram__bytes_write.sum per element of the kernel's 7b-2l capture, times this "
                                      "launch's elements (not measured in this run)",
                    "algorithmic_bytes": algo[dom]}

    # ---- full-replica receiver (N > 1): every rank applies all N gathered updates to a whole copy
    #      of the model (inference replicas that each hold the whole model)
    full_replica = None
    if dist is not None and not args.no_receivers:
        src_full = A_full if state["src_is_A"] else B_full
        replica = {k: v.clone() for k, v in src_full.items()}
        rep_chk = {}

        def rstep(events=None):
            src, dst = state["src"], state["dst"]
            if events:
                events[0].record(stream)
            upd = crx.encode_update_device(src, dst, sender)
            pg = start_exchange(upd)
            if events:
                events[1].record(stream)
            crx.apply_update(replica, upd, rep_chk)   # its own update first, while the others arrive
            pg.wait()
            for r, u in enumerate(pg.views()):
                if r != rank:
                    crx.apply_update(replica, u, rep_chk)
            if events:
                events[2].record(stream)
            flip()

        for _ in range(2):
            rstep()
        nrep = max(3, min(args.steps, 10))
        revs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(nrep)]
        barrier()
        for k in range(nrep):
            rstep(revs[k])
        barrier()
        src_full = A_full if state["src_is_A"] else B_full
        for k in replica:
            assert torch.equal(replica[k], src_full[k]), f"replica differs from the sender state: {k}"
        rt = torch.tensor([sum(e[0].elapsed_time(e[2]) for e in revs) / nrep,
                           sum(e[0].elapsed_time(e[1]) for e in revs) / nrep,
                           sum(e[1].elapsed_time(e[2]) for e in revs) / nrep], dtype=torch.float64, device=dev)
        dist.all_reduce(rt, op=dist.ReduceOp.MAX)
        r_step, r_encx, r_app = rt.tolist()
        full_replica = {"value": round(2.0 * total_params / (r_step * 1e-3) / 1e9, 2), "unit": "GB/s",
                        "ms_per_step": round(r_step, 4), "encode_ms": round(r_encx, 4),
                        "apply_all_ms": round(r_app, 4), "steps": nrep, "scaling": "strong",
                        "receiver": "full replica: every rank applies all N updates to a whole copy of the model",
                        "note": "GB/s of bf16 weights per sync step (the model's bytes over the step time)"}
        del replica
    del A_full, B_full
    torch.cuda.empty_cache()

    # ---- end to end through the public API with host (pinned) buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, A, B, dev, weight_bytes, exchange, barrier, dist)

    # ---- 32B shape, 8-way tensor parallel: every rank encodes and applies its
    #      own TP shard (weak scaling: one shard per GPU)
    tp8 = None
    if not args.no_receivers:
        state.clear()
        del A, B, recv
        torch.cuda.empty_cache()
        tp8 = run_tp8_shard(args, rank, world, dev, dist, start_exchange, barrier, peak)

    # ---- CPU baselines on a bounded sample of the same workload (rank 0, N = 1): the oracle port
    #      (one whole-dict update per step on every host thread) and the reference's own torch code
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        prev_s, cur_s, n_s = cpu_baseline_sample(shapes_all, cfg["lr"], args.cpu_sample)
        t_step, thr = time_oracle(prev_s, cur_s, steps=2)
        cpu = {"value": round(2.0 * n_s / t_step / 1e9, 4), "unit": "GB/s", "cores": thr, "kind": "port",
               "sample": f"{len(prev_s)} whole tensors of the workload ({n_s / 1e6:.0f}M params), cut into pieces of at "
                         f"most 2^24 elements with one update each, encode + apply on {thr} threads, {t_step:.2f} s "
                         f"per step (mean of 2)"}
        t_whole, _ = time_oracle(prev_s, cur_s, steps=1, whole=True)
        cpu["whole_dict_update"] = {
            "value": round(2.0 * n_s / t_whole / 1e9, 4), "unit": "GB/s", "cores": thr,
            "note": "the same sample as one whole-dict update per step (the oracle's passes run one tensor or exponent "
                    "per thread, so a step waits for its largest tensor); the piecewise figure above is the baseline"}
        tprev, tcur, tn = cpu_baseline_sample(shapes_all, cfg["lr"], args.torch_sample)
        t_ref, thr_ref = time_reference_torch(tprev, tcur, steps=1)
        if t_ref is not None:
            cpu["reference_torch"] = {
                "value": round(2.0 * tn / t_ref / 1e9, 4), "unit": "GB/s", "cores": thr_ref, "kind": "reference",
                "sample": f"{len(tprev)} whole tensors ({tn / 1e6:.0f}M params), the reference's own torch code "
                          f"(crukx_sync from baseline/_ref, unmodified) on CPU tensors with {thr_ref} threads, one "
                          f"steady-state step after one that fills the checksum caches, {t_ref:.2f} s"}
    ref_gpu = None
    if rank == 0 and world == 1 and not args.no_ref_gpu:
        ref_gpu = run_reference_gpu_line(args)

    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16 bits (int16 integer work)",
        "data": f"synthetic: random-init {cfg['name']} weights, one Adam-like step (lr {cfg['lr']}), seed 0",
        "config": {"workload": cfg["name"], "params": total_params, "tensors": len(shapes_all),
                   "lr": cfg["lr"], "changed_frac": round(changed_all / total_params, 5),
                   "parallelism": f"tensor partition x{world} (LPT on numel), NCCL all-gather of the device-resident updates"
                   if world > 1 else "single GPU",
                   "receiver": "partitioned: every rank applies the update of its own tensors, taken from the "
                               "gathered buffer" if world > 1 else "single GPU: the sender's GPU applies the update",
                   "path": "encode_update_device -> apply_update of the device update; at N > 1 the NCCL all-gather "
                           "that gives every rank every update (sizes between the hosts) runs on a side stream beside "
                           "the apply, and the step ends when both are done; the reference's bytes, kept in HBM",
                   "l2": "inputs larger than L2 (each state 2 B x params; no flush needed)"},
        "encode_gbs": round(weight_bytes / (ms_enc * 1e-3) / 1e9, 2),
        "apply_gbs": round(weight_bytes / (ms_app * 1e-3) / 1e9, 2),
        "exchange_ms": round(ms_ex, 4), "exchange_note": "encode end to all-gather end, overlapping the apply",
        "encode_ms": round(ms_enc, 4), "apply_ms": round(ms_app, 4),
        "update_bytes": int(upd_bytes), "bytes_per_changed": round(upd_bytes / max(changed_all, 1), 4),
        "wall_s_timed": round(t_wall, 3), "roofline_step": per_rank,
        "roofline": roofline, "kernels": kernels, "cpu_baseline": cpu, "e2e": e2e, "bytes_api": bytes_api,
        "full_replica": full_replica, "tp8_32b": tp8, "reference_gpu": ref_gpu,
        "sizes": None if size_cmp is None else dict(size_cmp, crukx=int(upd_bytes), changed=int(changed_all),
                                                    unit="bytes per update",
                                                    note="raw, sparserl and ctxfree as the reference's bench/compare.py "
                                                         "computes them (crx_size_stats); its zstd columns are not "
                                                         "computed"),
        "gpu_launches": launches, "clocks": clk.summary(), "parity": parity,
    }
    return result


def run_tp8_shard(args, rank, world, dev, dist, start_exchange, barrier, peak):
    """Qwen2.5-32B shapes cut 8 ways tensor-parallel; rank r holds shard r
    (seed 100 + r) and encodes and applies it, the updates crossing an NCCL all-gather."""
    import crukx_sync_b200 as crx
    shapes = CONFIGS["32b-tp8"]["shapes"]()
    params = sum(int(torch.tensor(s).prod()) for s in shapes.values())
    A, B = make_states(shapes, CONFIGS["32b-tp8"]["lr"], dev, seed=100 + rank)
    changed = sum(int((A[k].view(torch.int16) != B[k].view(torch.int16)).sum()) for k in A)
    recv = {k: v.clone() for k, v in A.items()}
    sender, receiver = {}, {}
    stream = torch.cuda.current_stream(dev)
    st = {"src": A, "dst": B}

    def one(events=None):
        if events:
            events[0].record(stream)
        upd = crx.encode_update_device(st["src"], st["dst"], sender)
        if events:
            events[1].record(stream)
        pg = start_exchange(upd)
        crx.apply_update(recv, upd, receiver)
        if events:
            events[2].record(stream)
        if pg is not None:
            pg.wait()
        if events:
            events[3].record(stream)
        st["src"], st["dst"] = st["dst"], st["src"]
        return upd.numel()

    for _ in range(args.warmup):
        one()
    n = max(3, min(args.steps, 10))
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n)]
    barrier()
    sizes = [one(evs[k]) for k in range(n)]
    barrier()
    for k in recv:
        assert torch.equal(recv[k], st["src"][k]), f"tp8 receiver differs: {k}"
    t = torch.tensor([sum(e[0].elapsed_time(e[3]) for e in evs) / n, sum(e[0].elapsed_time(e[1]) for e in evs) / n,
                      sum(e[1].elapsed_time(e[2]) for e in evs) / n, sum(e[2].elapsed_time(e[3]) for e in evs) / n],
                     dtype=torch.float64, device=dev)   # step, encode, apply, gather tail after the apply
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e, ms_a, ms_x = t.tolist()
    upd = sum(sizes) / len(sizes)
    out = {"value": round(world * 2.0 * params / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
           "encode_ms": round(ms_e, 4), "apply_ms": round(ms_a, 4), "gather_tail_ms": round(ms_x, 4), "steps": n,
           "params_per_rank": params, "changed_frac": round(changed / params, 5), "update_bytes_per_rank": int(upd),
           "scaling": "weak", "workload": "qwen2.5-32b-shape, 8-way TP shard per rank (seed 100 + rank)",
           "receiver": "per shard: every rank applies its own shard's update, taken from the gathered buffer",
           "roofline_step": step_roofline(params, changed, upd, ms_e, ms_a, peak)}
    del A, B, recv
    torch.cuda.empty_cache()
    return out


def run_reference_gpu_line(args):
    """The reference's own GPU path (crukx_sync from baseline/_ref, unmodified: torch CUDA ops and
    its Triton block decoder) on this B200, same workload and steps of encode_update (bytes) and
    apply_update, in a child process with a time limit; a secondary line, not a target."""
    if reference_src() is None or args.config not in ("7b", "1.5b", "toy", "7b-2l"):
        return None
    cmd = [sys.executable, os.path.abspath(__file__), "--ref-gpu-child", "--config", args.config]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=args.ref_gpu_timeout)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"did not finish within {args.ref_gpu_timeout} s"}
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"unavailable": f"child exited {r.returncode}: {(r.stderr or r.stdout)[-300:]}"}
    return json.loads(lines[-1])


def ref_gpu_child(args):
    src = reference_src()
    sys.path.insert(0, src)
    import crukx_sync as ref   # the reference, unchanged
    dev = torch.device("cuda", 0)
    cfg = CONFIGS[args.config]
    shapes = cfg["shapes"]()
    if cfg.get("drop_embed"):
        shapes = {k: v for k, v in shapes.items() if "embed" not in k}
    params = sum(int(torch.tensor(s).prod()) for s in shapes.values())
    A, B = make_states(shapes, cfg["lr"], dev, seed=0)
    recv = {k: v.clone() for k, v in A.items()}
    sender, receiver = {}, {}
    st = {"src": A, "dst": B}
    enc_t, app_t = [], []
    for i in range(3):
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        upd = ref.encode_update(st["src"], st["dst"], sender)
        torch.cuda.synchronize(dev)
        t1 = time.perf_counter()
        ref.apply_update(recv, upd, receiver)
        torch.cuda.synchronize(dev)
        t2 = time.perf_counter()
        if i:
            enc_t.append(t1 - t0)
            app_t.append(t2 - t1)
        st["src"], st["dst"] = st["dst"], st["src"]
    for k in recv:
        assert torch.equal(recv[k], st["src"][k]), k
    e, a = sum(enc_t) / len(enc_t), sum(app_t) / len(app_t)
    print(json.dumps({"value": round(2.0 * params / (e + a) / 1e9, 3), "unit": "GB/s", "encode_s": round(e, 3),
                      "apply_s": round(a, 3), "steps": len(enc_t), "workload": cfg["name"],
                      "what": "the reference's own GPU path (torch CUDA + its Triton block decoder), host bytes "
                              "between encode_update and apply_update as in its API, caches kept, wall clock "
                              "with synchronize; steady-state steps after one that fills the caches"}), flush=True)


def run_e2e(args, A, B, dev, weight_bytes, exchange, barrier, dist):
    """Same step through the public API with pinned host tensors: every step copies the inputs
    host->device and the update and weights device->host inside the timed region."""
    import crukx_sync_b200 as crx
    import psutil
    need = 3 * sum(v.numel() * 2 for v in A.values())
    if psutil.virtual_memory().available < need * 1.5:
        return {"value": None, "unit": "GB/s", "note": "not enough host RAM for pinned host copies"}
    Ah = {k: v.cpu().pin_memory() for k, v in A.items()}
    Bh = {k: v.cpu().pin_memory() for k, v in B.items()}
    Rh = {k: v.clone().pin_memory() for k, v in Ah.items()}
    sender, receiver = {}, {}
    st = {"src": Ah, "dst": Bh}
    nsteps = max(1, min(args.steps, args.e2e_steps))
    n_el = sum(v.numel() for v in A.values())

    chg, t_enc, t_app = [], [], []

    def one():   # each rank applies its own update (host bytes are not exchanged between processes)
        t0 = time.perf_counter()
        upd = crx.encode_update(st["src"], st["dst"], sender)
        t1 = time.perf_counter()
        chg.append(crx.apply_update(Rh, upd, receiver).changed)
        t_enc.append(t1 - t0)
        t_app.append(time.perf_counter() - t1)
        st["src"], st["dst"] = st["dst"], st["src"]
        return len(upd)

    one()
    barrier()
    t0 = time.perf_counter()
    sizes = [one() for _ in range(nsteps)]
    barrier()
    dt = (time.perf_counter() - t0) / nsteps
    if dist is not None:
        t = torch.tensor([dt], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = t.item()
    for k in Rh:
        assert torch.equal(Rh[k], st["src"][k])
    ub = sum(sizes) / len(sizes)
    # down: the update bytes, then the apply's commit list (a bit per element and a span table per
    # 2^18-element super-tile, the new values of the changed elements), scattered on the host
    n_super = sum((v.numel() + (1 << 18) - 1) >> 18 for v in A.values())
    changed = sum(chg[-nsteps:]) / nsteps
    return {"value": round(weight_bytes / dt / 1e9, 3), "unit": "GB/s", "ms_per_step": round(dt * 1e3, 2),
            "encode_ms": round(1e3 * sum(t_enc[-nsteps:]) / nsteps, 2), "apply_ms": round(1e3 * sum(t_app[-nsteps:]) / nsteps, 2),
            "steps": nsteps, "h2d_bytes_per_step": int(6 * n_el + ub),
            "d2h_bytes_per_step": int(ub + n_super * (32768 + 2048) + 2 * changed),
            "note": "public API with pinned host tensors: prev + cur and the receiver's weights up, the update "
                    "bytes and the apply's commit list down (only changed elements written back on the host)"}


# ---------------------------------------------------------------- reference arm

def run_reference(args, rank, world):
    """The reference's algorithm on the host cores: the C restatement in oracle/ (the reference
    itself is Python/torch; its own torch code is timed as a secondary figure in our arm's
    cpu_baseline.reference_torch), on a bounded sample of the same workload per step."""
    cfg = CONFIGS[args.config]
    shapes_all = cfg["shapes"]()
    total_params = sum(int(torch.tensor(s).prod()) for s in shapes_all.values())
    prev, cur, n_s = cpu_baseline_sample(shapes_all, cfg["lr"], args.ref_sample)
    from oracle import oracle
    oracle.build()
    t_step, thr = time_oracle(prev, cur, steps=args.steps, warmup=args.warmup)
    ms = 1e3 * t_step
    value = 2.0 * n_s / (ms * 1e-3) / 1e9
    sample = (f"{len(prev)} whole tensors of {cfg['name']} ({n_s / 1e6:.0f}M of {total_params / 1e9:.2f}B params) "
              f"per step, oracle/ C port, cut into pieces of at most 2^24 elements with one update each, "
              f"encode + apply on {thr} threads")
    return {"metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16 bits (int16 integer work)",
            "data": "synthetic, same generator as our arm", "config": {"workload": cfg["name"], "params": total_params},
            "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": thr, "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="7b", choices=sorted(CONFIGS))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-bytes-api", action="store_true", help="skip the host-bytes API measurement")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the first update")
    ap.add_argument("--no-receivers", action="store_true", help="skip the full-replica and 32B-TP8 lines")
    ap.add_argument("--emulate", default="", help="R/N: time rank R's tensors of an N-way partition on one GPU "
                                                   "(a development aid; the line then describes that share)")
    ap.add_argument("--no-ref-gpu", action="store_true", help="skip the reference's own GPU path line")
    ap.add_argument("--ref-gpu-timeout", type=int, default=300)
    ap.add_argument("--ref-gpu-child", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--torch-sample", type=int, default=100_000_000,
                    help="elements of the sample the reference's torch code runs on the host cores")
    ap.add_argument("--cpu-sample", type=int, default=1_000_000_000, help="elements in the CPU-baseline sample")
    ap.add_argument("--ref-sample", type=int, default=1_000_000_000, help="elements per reference-arm step")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.ref_gpu_child:
        ref_gpu_child(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, rank, world)), flush=True)
        return
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as td
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        dist = td
    try:
        res = run_ours(args, rank, world, dist)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
