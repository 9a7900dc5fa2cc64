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
compressed payloads are all-gathered over NCCL, and each rank applies its own partition's update
taken from the gathered buffer.  The reported time is the max over ranks.
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


def time_oracle(prev, cur, steps=1, threads=None, warmup=0):
    """The CPU oracle (the C restatement of the reference) on one sample, with all host threads:
    tensors cut into pieces of at most 2^24 elements, one update per piece, pieces spread over a
    thread pool (the C calls release the GIL); the per-element work is the reference's.
    `warmup` untimed steps come first.  Returns seconds per timed step (encode + apply, whole
    sample) and the threads used."""
    import concurrent.futures

    from oracle import oracle
    threads = threads or host_threads()
    sender, receiver = {}, {}
    recv = {k: v.clone() for k, v in prev.items()}
    piece = 1 << 24
    pieces = [(k, a, min(a + piece, prev[k].numel())) for k in prev for a in range(0, prev[k].numel(), piece)]
    pieces.sort(key=lambda p: p[1] - p[2])   # big pieces first: better balance
    state = {"a": prev, "b": cur}

    def one(p):
        k, lo, hi = p
        name = f"{k}#{lo}"
        upd = oracle.encode_update({name: state["a"][k].view(-1)[lo:hi]}, {name: state["b"][k].view(-1)[lo:hi]}, sender)
        oracle.apply_update({name: recv[k].view(-1)[lo:hi]}, upd, receiver)

    times = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=threads) as pool:
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            list(pool.map(one, pieces))
            if i >= warmup:
                times.append(time.perf_counter() - t0)
            state["a"], state["b"] = state["b"], state["a"]
    for k in recv:   # the oracle reproduced the sender's state
        assert torch.equal(recv[k], state["a"][k]), k
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
    owner = cdist.partition({k: int(torch.tensor(v).prod()) for k, v in shapes_all.items()}, world)
    shapes = {k: v for k, v in shapes_all.items() if owner[k] == rank}
    total_params = sum(int(torch.tensor(s).prod()) for s in shapes_all.values())
    my_params = sum(int(torch.tensor(s).prod()) for s in shapes.values())
    log("generating", len(shapes), "tensors,", my_params, "params")
    A, B = make_states(shapes, cfg["lr"], dev, seed=0)
    log("generated")
    changed = sum(int((A[k].view(torch.int16) != B[k].view(torch.int16)).sum()) for k in A)
    parity = None
    if not args.no_parity:
        log("parity check against the oracle")
        parity = parity_check(A, B, max(1, host_threads() // max(world, 1)))
        log("parity", parity)
    recv = {k: v.clone() for k, v in A.items()}
    sender, receiver = {}, {}
    ctx = _ext.context(dev.index)
    L = _ext.load()
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def exchange(upd):
        """All-gather of the device-resident updates over NCCL; this rank's update from the gather."""
        return cdist.allgather_updates_device(upd, ranks=[rank])[0]

    state = {"src": A, "dst": B}

    def step(events=None):
        """One sync step with the updates resident in HBM: encode_update_device (the reference's
        bytes, in device memory), NCCL all-gather, apply_update of the device update."""
        src, dst = state["src"], state["dst"]
        if events:
            events[0].record(stream)
        upd = crx.encode_update_device(src, dst, sender)
        if events:
            events[1].record(stream)
        mine = exchange(upd)
        if events:
            events[2].record(stream)
        st = crx.apply_update(recv, mine, receiver)
        if events:
            events[3].record(stream)
        state["src"], state["dst"] = dst, src
        return upd, st

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
    ex = [e[1].elapsed_time(e[2]) for e in evs]
    app = [e[2].elapsed_time(e[3]) for e in evs]
    tot = [e[0].elapsed_time(e[3]) for e in evs]
    for k in recv:
        assert torch.equal(recv[k], state["src"][k]), f"receiver differs after timing: {k}"
    ms_step = sum(tot) / len(tot)
    ms_enc, ms_ex, ms_app = (sum(x) / len(x) for x in (enc, ex, app))
    if dist is not None:
        t = torch.tensor([ms_step, ms_enc, ms_app, ms_ex], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step, ms_enc, ms_app, ms_ex = t.tolist()
        c = torch.tensor([changed, sum(sizes) / len(sizes)], dtype=torch.float64, device=dev)
        dist.all_reduce(c)
        changed_all, upd_bytes = c.tolist()
    else:
        changed_all, upd_bytes = changed, sum(sizes) / len(sizes)
    weight_bytes = 2.0 * total_params
    value = weight_bytes / (ms_step * 1e-3) / 1e9

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
            state["src"], state["dst"] = dst, src

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
    L.crx_ctx_profile(ctx, 0)
    peak, peak_kind = measured_peak()
    algo = {"k_enc_rank": 4.0 * my_params, "k_map": 2.0 * my_params, "k_app_hist": 2.0 * my_params}
    kernels = {}
    for nm, (ms, n) in sorted(kt.items(), key=lambda x: -x[1][0]):
        per = ms / max(n, 1)
        row = {"ms_per_launch": round(per, 4), "launches": n, "share": None}
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
                    "algorithmic_bytes": algo[dom]}

    # ---- end to end through the public API with host (pinned) buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, A, B, dev, weight_bytes, exchange, barrier, dist)

    # ---- CPU baseline: the oracle on a bounded sample of the same workload (rank 0, N = 1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        prev_s, cur_s, n_s = cpu_baseline_sample(shapes_all, cfg["lr"], args.cpu_sample)
        t_step, thr = time_oracle(prev_s, cur_s, steps=2)
        cpu = {"value": round(2.0 * n_s / t_step / 1e9, 4), "unit": "GB/s", "cores": thr, "kind": "port",
               "sample": f"{len(prev_s)} whole tensors of the workload ({n_s / 1e6:.0f}M params), encode + apply "
                         f"per tensor on {thr} threads, {t_step:.2f} s per step (mean of 2)"}
    del A, B, recv
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16 bits (int16 integer work)",
        "data": f"synthetic: random-init {cfg['name']} weights, one Adam-like step (lr {cfg['lr']}), seed 0",
        "config": {"workload": cfg["name"], "params": total_params, "tensors": len(shapes_all),
                   "lr": cfg["lr"], "changed_frac": round(changed_all / total_params, 5),
                   "parallelism": f"tensor partition x{world} (LPT on numel), NCCL all-gather of the device-resident updates"
                   if world > 1 else "single GPU",
                   "path": "encode_update_device -> (NCCL all-gather) -> apply_update of the device update; "
                           "the reference's bytes, kept in HBM",
                   "l2": "inputs larger than L2 (each state 2 B x params; no flush needed)"},
        "encode_gbs": round(weight_bytes / (ms_enc * 1e-3) / 1e9, 2),
        "apply_gbs": round(weight_bytes / (ms_app * 1e-3) / 1e9, 2),
        "exchange_ms": round(ms_ex, 4), "encode_ms": round(ms_enc, 4), "apply_ms": round(ms_app, 4),
        "update_bytes": int(upd_bytes), "bytes_per_changed": round(upd_bytes / max(changed_all, 1), 4),
        "wall_s_timed": round(t_wall, 3),
        "roofline": roofline, "kernels": kernels, "cpu_baseline": cpu, "e2e": e2e, "bytes_api": bytes_api,
        "gpu_launches": launches, "clocks": clk.summary(), "parity": parity,
    }
    return result


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

    def one():   # each rank applies its own update (host bytes are not exchanged between processes)
        upd = crx.encode_update(st["src"], st["dst"], sender)
        crx.apply_update(Rh, upd, receiver)
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
    return {"value": round(weight_bytes / dt / 1e9, 3), "unit": "GB/s", "ms_per_step": round(dt * 1e3, 2),
            "steps": nsteps, "h2d_bytes_per_step": int(6 * n_el + ub), "d2h_bytes_per_step": int(2 * n_el + ub),
            "note": "public API with pinned host tensors: prev+cur up, weights up and back, update bytes down"}


# ---------------------------------------------------------------- reference arm

def run_reference(args, rank, world):
    """The reference's algorithm on the host cores: the C restatement in oracle/ (the reference
    itself is Python/torch and cannot be installed on the GPU box), on a bounded sample of the
    same workload per step."""
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
              f"per step, oracle/ C port, encode + apply per tensor on {thr} threads")
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
    ap.add_argument("--cpu-sample", type=int, default=1_000_000_000, help="elements in the CPU-baseline sample")
    ap.add_argument("--ref-sample", type=int, default=1_000_000_000, help="elements per reference-arm step")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
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
