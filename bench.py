#!/usr/bin/env python3
"""Benchmark of the KVMem per-step retrieval path on B200 (BASELINE metric:
retrieval+stage-in us per decode step, 64 layers, 256K history).

One step = accumulate the decode query, score every block on every layer,
reduce the per-layer terms in layer order (exchanged between ranks when the
layers are sharded), select the top-k, diff the plan, stage newly selected
blocks host -> HBM pool and rebuild every changed window slot (K re-roped at
its window position, V copied).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU, each owning n_layer / N layers;
the only cross-rank traffic per step is the per-(layer, block) score terms
(f64, each layer's query flag packed in its row, ~1 MiB in total at 64
layers): by default the scoring kernel writes them into every rank's buffer
over NVLink peer memory (CUDA IPC, set up once through the process group) and
the reduction waits on per-rank step flags; --exchange nccl uses an NCCL
all-gather instead.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "kvmem-llama.cpp_b200")
sys.path.insert(0, PKG)

METRIC = "retrieval+stage-in µs/decode step (64 layers, 256K); KV GB/s vs HBM/link peak"
FALLBACK_HBM_GBS = 6650.0


def workloads():
    """The workload definitions (kvmret/workloads.py), loaded by path: plain
    data, so the reference arm never imports the kvmret package or loads its
    native library."""
    import importlib.util
    name = "kvmret_bench_workloads"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(
            name, os.path.join(PKG, "kvmret", "workloads.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod  # dataclasses resolve the module while building the class
        spec.loader.exec_module(mod)
    return sys.modules[name]


def decode_workload(w):
    """config.workload and dtype of a decode-step line (both arms print these)."""
    TYPE_F16 = workloads().TYPE_F16
    desc = (f"{w.name}: {w.n_layer} layers, {w.n_head}q/{w.n_head_kv}kv heads, d{w.d_head}, "
            f"{w.n_blocks} blocks x {w.block_tokens} tok ({w.n_tokens // 1024}K), budget "
            f"{w.budget_blocks} blocks, sink {w.sink_blocks}, gen-reserve {w.reserve_blocks} slots")
    return desc, ("f16" if w.k_type == TYPE_F16 else "q8_0/q4_0")


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------
class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", f"--id={index}", f"--query-gpu={self.Q}", "--format=csv,noheader",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = [l.split(",") for l in open(self.f.name).read().splitlines() if l.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1].split()[0]))
                mx = float(r[2].split()[0])
                for n, v in zip(names, r[5:9]):
                    if "Active" in v and "Not" not in v:
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def link_gbps(nbytes=1 << 30, reps=3, d2h=False):
    """Host link bandwidth: best of `reps` 1 GiB copies between pinned host
    memory and the device (host to device unless d2h), CUDA events."""
    import torch
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    best = 1e30
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            e0.record(s)
            if d2h:
                h.copy_(d, non_blocking=True)
            else:
                d.copy_(h, non_blocking=True)
            e1.record(s)
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) / 1e3)
    del h, d
    return nbytes / best / 1e9


# ---------------------------------------------------------------------------
def cpu_sample(w, n_h2d, n_asm, threads, use_ref, budget_s=10.0):
    """CPU time of one step of the same workload, from timed samples of each
    component (restated score_retrieval; pick_topk / set_selection /
    rope_neox_apply from the reference's libkvmem when built, else the
    oracle's restatement; memcpy staging of the stage-in bytes into a pinned
    slab), scaled by the step's unit counts."""
    import concurrent.futures as cf

    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as po
    use_ref = use_ref and po.ref is not None
    rng = np.random.default_rng(0)
    L, N, E, T = w.n_layer, w.n_blocks, w.E, w.block_tokens
    ls = 2  # layers scored per sample
    mean = rng.standard_normal((N, ls, E)).astype(np.float32)
    has = np.ones(N, np.uint8)
    q_sum = rng.standard_normal((ls, w.qdim)).astype(np.float32)
    q_count = np.ones(ls, np.uint32)
    pool = cf.ThreadPoolExecutor(max_workers=threads)

    def timed(fn, reps):
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) / reps

    # S3: score N blocks x ls layers; threads split the blocks
    parts = np.array_split(np.arange(N), threads)

    def score_all():
        list(pool.map(lambda ix: po.score(mean[ix], has[ix], q_sum, q_count, w.n_head,
                                          w.n_head_kv, w.d_head), parts))
    t_score = timed(score_all, 2) * (L / ls)
    scores = po.score(mean, has, q_sum, q_count, w.n_head, w.n_head_kv, w.d_head)
    # S6 + S7
    if use_ref:
        t_topk = timed(lambda: po.ref_pick_topk(scores, w.budget_blocks, w.sink_blocks), 5)
        rt = po.RefRuntime(T, w.budget_blocks, w.sink_blocks)
        rt.append(N * T)
        ids = po.ref_pick_topk(scores, w.budget_blocks, w.sink_blocks)
        t_plan = timed(lambda: rt.set_selection(ids), 5)
    else:
        t_topk = timed(lambda: po.pick_topk(scores, w.budget_blocks, w.sink_blocks), 5)
        st = po.Store(T)
        st.append(N * T)
        ids = po.pick_topk(scores, w.budget_blocks, w.sink_blocks)
        t_plan = timed(lambda: st.set_selection(ids), 5)
    # S11: staging memcpy of one block's units (all layers) into a host slab
    unit = T * E * 2 * 2
    s_np = np.ones(L * unit, np.uint8)
    d_np = np.zeros(L * unit, np.uint8)
    chunks = np.array_split(np.arange(L * unit // 4096), threads)

    def stage():
        list(pool.map(lambda ix: np.copyto(d_np[ix[0] * 4096:(ix[-1] + 1) * 4096],
                                           s_np[ix[0] * 4096:(ix[-1] + 1) * 4096]), chunks))
    t_stage = timed(stage, 3) * n_h2d
    # S12: RoPE of K block-layer units (f16 -> f32 -> rope -> f16)
    kb = rng.standard_normal((threads, T, w.n_head_kv, w.d_head)).astype(np.float16)

    def rope_unit(i):
        x = kb[i].astype(np.float32)
        if use_ref:
            y = po.ref_rope_neox(x, 4096 + i, w.freq_base)
        else:
            y = po.rope_neox(x, 4096 + i, w.freq_base)
        return y.astype(np.float16)

    t_rope = timed(lambda: list(pool.map(rope_unit, range(threads))), 2) / threads
    t_rope *= n_asm * L
    pool.shutdown()
    total = t_score + t_topk + t_plan + t_stage + t_rope
    parts_s = {"score": t_score, "topk": t_topk, "plan": t_plan, "stage_memcpy": t_stage,
               "rope": t_rope}
    return total, parts_s, ("reference" if use_ref else "port")


# ---------------------------------------------------------------------------
def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as po
    threads = os.cpu_count() or 1
    n_h2d, n_asm = args.churn_h2d, args.churn_asm
    vals = []
    for _ in range(args.warmup):
        cpu_sample(w, n_h2d, n_asm, threads, True)
    parts = None
    for _ in range(args.steps):
        t, parts, kind = cpu_sample(w, n_h2d, n_asm, threads, True)
        vals.append(t)
    us = sum(vals) / len(vals) * 1e6
    sample = (f"per step: restated score_retrieval on 2 of {w.n_layer} layers x {w.n_blocks} "
              f"blocks (x{w.n_layer // 2}), pick_topk + set_selection on all blocks, memcpy "
              f"staging of one block's {w.n_layer} layers (x{n_h2d} new blocks/step), "
              f"rope_neox_apply of {threads} block-layers (x{n_asm} moved blocks x "
              f"{w.n_layer} layers); "
              f"{'libkvmem from reference sources' if po.ref is not None else 'oracle port'}")
    line = {"impl": "reference", "metric": METRIC, "value": round(us, 1), "unit": "us/step",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(us / 1e3, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": decode_workload(w)[1], "data": "synthetic",
            "config": {"workload": decode_workload(w)[0], "threads": threads},
            "cpu_baseline": {"value": round(us, 1), "unit": "us/step", "cores": threads,
                             "kind": kind, "sample": sample,
                             "parts_ms": {k: round(v * 1e3, 3) for k, v in parts.items()}},
            "e2e": {"value": round(us, 1), "unit": "us/step", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
def run_ours(args, w):
    import numpy as np
    import torch
    import torch.distributed as dist

    import kvmret
    from kvmret import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    if w.n_layer % world:
        raise SystemExit(f"{w.n_layer} layers do not split over {world} GPUs")
    Ll = w.n_layer // world
    layer0 = rank * Ll
    T = w.block_tokens

    cfg = kvmret.default_config(
        n_layer=Ll, n_head=w.n_head, n_head_kv=w.n_head_kv, d_head=w.d_head, block_tokens=T,
        max_blocks=w.n_blocks, budget_blocks=w.budget_blocks, reserve_blocks=w.reserve_blocks,
        sink_blocks=w.sink_blocks, k_type=w.k_type, v_type=w.v_type, n_rot=w.d_head,
        freq_base=w.freq_base, pool_cache=int(args.pool_cache), device=local)
    t_setup = time.perf_counter()
    r = kvmret.Retriever(cfg)
    hist = synth.TorchHistory(w, local, layer0=layer0, n_layer=Ll)
    chunk = 64 * T
    for t0 in range(0, w.n_tokens, chunk):
        m = min(chunk, w.n_tokens - t0)
        kc, vc = hist.chunk(t0, m)
        if w.k_type == kvmret.TYPE_F16:
            r.append(kc, vc, pos0=t0)
        else:  # config 3: q8_0 K rows, q4_0 V rows, summaries from the f16 capture
            kq = kvmret.quantize_f16(kc, w.k_type)
            vq = kvmret.quantize_f16(vc, w.v_type)
            r.append(kc, vq, k_rows=kq, pos0=t0)
            del kq, vq
        r.sync()
        del kc, vc
    torch.cuda.synchronize()
    t_setup = time.perf_counter() - t_setup
    link = link_gbps()
    link_d2h = link_gbps(d2h=True)

    stride = r.contrib_stride
    contrib_loc = torch.zeros(Ll * stride, dtype=torch.float64, device="cuda")
    contrib_all = contrib_loc if world == 1 else torch.zeros(w.n_layer * stride,
                                                              dtype=torch.float64, device="cuda")
    ext = torch.cuda.ExternalStream(r.stream_ptr)
    cur = torch.cuda.current_stream()

    marks = []  # (label, event) on the library stream, --timeline only

    def mark(label):
        if args.timeline:
            e = torch.cuda.Event(enable_timing=True)
            e.record(ext)
            marks.append((label, e))

    p2p = world > 1 and args.exchange == "p2p"
    if p2p:  # peer-memory exchange: IPC handles all-gathered once over the process group
        handles = [None] * world
        dist.all_gather_object(handles, r.exchange_export(world))
        r.exchange_import(rank, handles)

    def step(q_dev):
        mark("start")
        r.query_reset()
        r.query_add(q_dev)
        mark("query")
        if p2p:  # score + push rows to every rank + wait + reduce, all on the device
            r.score_exchange()
            mark("score")
            mark("exchange")
        else:
            r.score_layers(contrib_loc)
            mark("score")
            if world > 1:
                ev = torch.cuda.Event()
                ev.record(ext)
                cur.wait_event(ev)
                dist.all_gather_into_tensor(contrib_all, contrib_loc)
                ev2 = torch.cuda.Event()
                ev2.record(cur)
                ext.wait_event(ev2)
            mark("exchange")
            r.score_reduce(contrib_all, w.n_layer)
        r.select_apply_async()
        mark("apply_enqueued")

    def queries(n):
        out = []
        for _ in range(n):
            q = hist.next_query()[layer0:layer0 + Ll].contiguous()
            out.append(q)
        return out

    def barrier():
        if world > 1:
            dist.barrier()

    # clocks are sampled from before the warm-up until after the e2e loop
    clocks = Clocks(local)
    time.sleep(0.6)
    # warm-up (the first step stages the whole window from the host)
    warm_q = queries(args.warmup)
    step(warm_q[0])
    ids0 = r.step_collect()[0]

    def restart():
        """Untimed: the start state both measured loops begin from. An empty
        working set and pool (kvmret_clear_working_set), the first warm-up
        step's selection staged again, then the other warm-up steps; the state
        (window, pool contents and LRU order) is then a function of these
        queries alone, so the e2e loop repeats the timed loop's work exactly."""
        r.clear_working_set(drop_pool=True)
        r.apply(ids0)
        for q in warm_q[1:]:
            step(q)
            r.step_collect()
        r.sync()

    restart()

    # timed region: device time of exactly K steps on the library stream
    qs = queries(args.steps)
    qh = [q.cpu().pin_memory() for q in qs]  # the same K queries for the e2e loop
    torch.cuda.synchronize()
    r.prof_enable(True)
    barrier()
    r.sync()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stats = []
    ids_timed = []
    marks.clear()
    e0.record(ext)
    # the host enqueues step k+1 before collecting step k, so the device never
    # waits for the host between steps. The NVTX range lets a profiler keep
    # only these launches (ncu --nvtx --nvtx-include "timed_steps/").
    torch.cuda.nvtx.range_push("timed_steps")
    for i, q in enumerate(qs):
        step(q)
        if i > 0:
            ids_k, st_k = r.step_collect()
            ids_timed.append(ids_k)
            stats.append(st_k)
    torch.cuda.nvtx.range_pop()
    e1.record(ext)
    ids_k, st_k = r.step_collect()
    ids_timed.append(ids_k)
    stats.append(st_k)
    r.sync()
    torch.cuda.synchronize()
    barrier()
    if args.print_steps and rank == 0:
        # per timed step: what the window assembly of that step moved (the
        # algorithmic bytes of a launch a profiler captured)
        for i, st in enumerate(stats):
            print(f"step {i}: n_moved {st['n_moved']} n_h2d {st['n_h2d_blocks']} "
                  f"assemble_bytes {st['assemble_bytes']} h2d_bytes {st['h2d_bytes']}",
                  file=sys.stderr)
    prof = r.prof_read()
    r.prof_enable(False)
    timeline = None
    if args.timeline and marks:
        acc, cnt = {}, {}
        for (la, ea), (lb, eb) in zip(marks, marks[1:]):
            key = f"{la}->{lb}"
            acc[key] = acc.get(key, 0.0) + ea.elapsed_time(eb)
            cnt[key] = cnt.get(key, 0) + 1
        timeline = {k: round(acc[k] / cnt[k] * 1e3, 1) for k in acc}
        marks.clear()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps

    # e2e: the same K queries from pinned host memory -> device every step, ids
    # back on the host, from the same start state as the timed loop (its
    # selections and per-step work are checked against the timed loop's below)
    restart()
    qd = torch.empty_like(qs[0])
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_stats = []
    e2e_ids = []
    for i, q in enumerate(qh):
        qd.copy_(q, non_blocking=True)
        step(qd)
        if i > 0:
            ids_k, st_k = r.step_collect()  # the previous step's ids, read on the host
            e2e_ids.append(ids_k)
            e2e_stats.append(st_k)
    ids_k, st_k = r.step_collect()
    e2e_ids.append(ids_k)
    e2e_stats.append(st_k)
    r.sync()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_us = e2e_s / args.steps * 1e6

    def avg(key, ss):
        return sum(s[key] for s in ss) / len(ss)

    e2e_same = (len(e2e_ids) == len(ids_timed) and
                all(np.array_equal(a, b) for a, b in zip(e2e_ids, ids_timed)) and
                all(a["n_moved"] == b["n_moved"] and a["n_h2d_blocks"] == b["n_h2d_blocks"]
                    for a, b in zip(e2e_stats, stats)))

    n_h2d = avg("n_h2d_blocks", stats)
    n_moved = avg("n_moved", stats)
    n_asm = avg("n_assembled", stats)
    h2d_step = avg("h2d_bytes", stats)
    asm_step = avg("assemble_bytes", stats)
    score_step = prof["score_bytes"] / max(1, prof["n_score"])
    if prof["dropped"]:
        print(f"warning: {prof['dropped']} timing regions dropped", file=sys.stderr)
    hbm, peak_src = load_peaks()

    # roofline of the dominant kernel (window assembly), live event timing. One
    # launch rebuilds moved slots from the HBM pool and fresh slots from the host
    # repository, so its bound is the slower of its HBM bytes at the HBM peak and
    # its host-link bytes at the measured link bandwidth.
    n_launch = max(1, prof["n_asm"])
    asm_ms = prof["asm_ms"] / n_launch
    asm_hbm = prof["asm_hbm_bytes"] / n_launch
    asm_link = prof["asm_link_bytes"] / n_launch
    achieved = asm_hbm / (asm_ms / 1e3) / 1e9 if asm_ms > 0 else 0.0
    t_asm_roof = max(asm_hbm / (hbm * 1e9), asm_link / (link * 1e9))
    asm_frac = t_asm_roof / (asm_ms / 1e3) if asm_ms > 0 else 0.0
    score_ms = prof["score_ms"] / max(1, prof["n_score"])
    score_gbs = score_step / (score_ms / 1e3) / 1e9 if score_ms > 0 else 0.0
    # step roofline: T = B_sum/BW_hbm + max(B_link/BW_link, (B_link + B_asm)/BW_hbm)
    t_roof = score_step / (hbm * 1e9) + max(h2d_step / (link * 1e9),
                                             (h2d_step + asm_step) / (hbm * 1e9))
    kv_bytes = score_step + h2d_step + asm_step
    # DRAM traffic of one assembly launch: the ratio of ncu's dram read + write
    # bytes to the launch's algorithmic bytes, measured on an 8-layer cut of
    # the same workload (profiles/step_kernels_cfg2_l8.md: 1556.8 / 1585.4 MB;
    # profiles/assemble_quant_kernel_cfg3_l8.md: 793.3 / 824.7 MB), scaled to
    # this launch's algorithmic bytes (the traffic grows with the blocks moved).
    traffic_ratio = (1556.8 / 1585.4) if w.k_type == kvmret.TYPE_F16 else (793.3 / 824.7)
    asm_traffic = traffic_ratio * asm_hbm

    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(ms_step * 1e3, 1), "unit": "us/step",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": decode_workload(w)[1],
            "data": "synthetic: seeded N(0,1) x LogNormal(0,0.5) channel scale, "
                    f"{w.n_planted} planted blocks, query drift {w.drift}/step",
            "config": {
                "workload": decode_workload(w)[0],
                "layers_per_gpu": Ll, "parallelism": f"layer-sharded x{world}",
                "exchange": (args.exchange if world > 1 else None),
                "l2": "inputs larger than L2 (summaries "
                      f"{score_step / 2**20:.0f} MiB/step, window/pool GiB-scale)",
                "pool_cache": bool(args.pool_cache)},
            "roofline": {"kernel": ("assemble_kernel" if w.k_type == kvmret.TYPE_F16
                                    else "assemble_quant_kernel")
                                   + " (window assembly: moved slots from the HBM pool, "
                                     "fresh slots from the host repository)",
                         "bound": "hbm" if asm_hbm / hbm >= asm_link / link else "host link",
                         "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(asm_frac, 4), "traffic": int(asm_traffic),
                         "traffic_source": "ncu dram bytes / algorithmic bytes of an 8-layer "
                                           "capture, scaled to this launch",
                         "peak_source": peak_src,
                         "avg_launch_ms": round(asm_ms, 4),
                         "alg_hbm_bytes_per_launch": int(asm_hbm),
                         "alg_link_bytes_per_launch": int(asm_link),
                         "link_gbs_measured": round(link, 2)},
            "kernels": {
                "score": {"ms": round(score_ms, 4), "GB/s": round(score_gbs, 1),
                          "frac_hbm": round(score_gbs / hbm, 4)}},
            "step_roofline": {"t_roof_us": round(t_roof * 1e6, 1),
                              "t_meas_us": round(ms_step * 1e3, 1),
                              "frac": round(t_roof * 1e3 / ms_step, 4),
                              "link_gbs_measured": round(link, 2),
                              "link_d2h_gbs_measured": round(link_d2h, 2), "hbm_gbs": hbm,
                              "B_sum": int(score_step), "B_link": int(h2d_step),
                              "B_asm": int(asm_step)},
            "kv_gbps": round(kv_bytes / (ms_step / 1e3) / 1e9, 1),
            "churn": {"n_h2d_blocks": round(n_h2d, 2), "n_moved": round(n_moved, 2),
                      "n_assembled": round(n_asm, 2)},
            "e2e": {"value": round(e2e_us, 1), "unit": "us/step",
                    "h2d_bytes_per_step": int(qs[0].numel() * 2 + avg("h2d_bytes", e2e_stats)),
                    "d2h_bytes_per_step": int(w.n_blocks),
                    "same_steps_as_timed": e2e_same,
                    "churn": {"n_h2d_blocks": round(avg("n_h2d_blocks", e2e_stats), 2),
                              "n_moved": round(avg("n_moved", e2e_stats), 2)}},
            "gpu_launches": int(prof["launches"]),
            "timeline_us": timeline,
            "clocks": clk,
            "setup_s": round(t_setup, 1),
        }
        if world == 1 and not args.no_cpu_baseline:
            total, parts, kind = cpu_sample(w, max(1, round(n_h2d)), max(1, round(n_asm)), 1,
                                            False)
            line["cpu_baseline"] = {
                "value": round(total * 1e6, 1), "unit": "us/step", "cores": 1, "kind": kind,
                "sample": "restated score_retrieval on 2 layers x all blocks (scaled to "
                          f"{w.n_layer}), pick_topk + set_selection, memcpy staging of one "
                          f"block (x{round(n_h2d)}), host RoPE of 1 block-layer (x"
                          f"{round(n_asm)} x {w.n_layer})",
                "parts_ms": {k: round(v * 1e3, 3) for k, v in parts.items()}}
    r.close()
    if world > 1:
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


def run_prefill(args, w):
    """Config 4: one step = score a prefill chunk (every token against every block
    summary on the tensor cores, per-token top-k, union), then append the
    chunk's K/V (its completed blocks go to the pinned host repository, their
    summaries are recomputed). 1 GPU."""
    import numpy as np
    import torch

    import kvmret
    from kvmret import synth

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0 or int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("config 4 runs on one GPU")
    torch.cuda.set_device(0)
    T, P, K = w.block_tokens, w.prefill_tokens, w.prefill_topk
    n_steps = args.warmup + args.steps
    blocks_cap = w.n_blocks + (n_steps + 6) * ((P + T - 1) // T)  # + the e2e steps
    cfg = kvmret.default_config(
        n_layer=w.n_layer, n_head=w.n_head, n_head_kv=w.n_head_kv, d_head=w.d_head,
        block_tokens=T, max_blocks=blocks_cap, budget_blocks=w.budget_blocks,
        reserve_blocks=w.reserve_blocks, sink_blocks=w.sink_blocks, n_rot=w.d_head,
        freq_base=w.freq_base, device=0)
    t_setup = time.perf_counter()
    r = kvmret.Retriever(cfg)
    hist = synth.TorchHistory(w, 0)
    for t0 in range(0, w.n_tokens, 64 * T):
        kc, vc = hist.chunk(t0, min(64 * T, w.n_tokens - t0))
        r.append(kc, vc, pos0=t0)
        r.sync()
        del kc, vc
    # two prefill chunks resident in HBM: queries [L][P][Hq*D] (N(0,1) plus a
    # share of the planted direction) and the chunk's K / V rows
    g = torch.Generator(device="cuda").manual_seed(w.seed + 11)
    qs, kvs = [], []
    for i in range(2):
        q = torch.randn((w.n_layer, P, w.n_head * w.d_head), generator=g, device="cuda")
        q.add_(0.3 * hist.q0.float().reshape(w.n_layer, 1, -1))
        qs.append(q.half())
        kvs.append(hist.chunk(w.n_tokens + i * P, P))
        del q
    sel = torch.zeros(blocks_cap, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    t_setup = time.perf_counter() - t_setup
    lib, h = kvmret.lib, r.h
    ext = torch.cuda.ExternalStream(r.stream_ptr)
    pos = [w.n_tokens]

    def step(i, q_dev=None, k_dev=None, v_dev=None):
        q_dev = qs[i % 2] if q_dev is None else q_dev
        kc, vc = kvs[i % 2] if k_dev is None else (k_dev, v_dev)
        kvmret._check(lib.kvmret_prefill_score(h, q_dev.data_ptr(), P, K, sel.data_ptr(), None,
                                                None))
        kvmret._check(lib.kvmret_append(h, pos[0], P, kc.data_ptr(), None, vc.data_ptr()))
        pos[0] += P

    clocks = Clocks(0)
    time.sleep(0.6)
    for i in range(args.warmup):
        step(i)
    r.sync()
    r.prof_enable(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    for i in range(args.steps):
        step(i)
    e1.record(ext)
    r.sync()
    torch.cuda.synchronize()
    ms_step = e0.elapsed_time(e1) / args.steps
    prof = r.prof_read()
    r.prof_enable(False)
    n_union = int(sel[: int(lib.kvmret_n_blocks(h))].sum().item())
    # e2e: the chunk's queries and K / V copied from pinned host memory each
    # step, the union flags read back
    qh = qs[0].cpu().pin_memory()
    kh, vh = (x.cpu().pin_memory() for x in kvs[0])
    qd, kd, vd = torch.empty_like(qs[0]), torch.empty_like(kvs[0][0]), torch.empty_like(kvs[0][1])
    sel_h = torch.empty_like(sel, device="cpu").pin_memory()
    e2e_steps = max(1, min(args.steps, 5))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        qd.copy_(qh, non_blocking=True)
        kd.copy_(kh, non_blocking=True)
        vd.copy_(vh, non_blocking=True)
        with kvmret._Ordered(r.stream_ptr):
            step(i, qd, kd, vd)
        torch.cuda.current_stream().wait_stream(ext)
        sel_h.copy_(sel, non_blocking=True)
    torch.cuda.synchronize()
    e2e_us = (time.perf_counter() - t0) / e2e_steps * 1e6
    clk = clocks.stop()
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    tc_peak = float(peaks.get("bf16_tflops", 1590.0))
    gemm_ms = prof["gemm_ms"] / max(1, prof["n_gemm"])
    gemm_tf = prof["gemm_flops"] / max(1, prof["n_gemm"]) / (gemm_ms / 1e3) / 1e12 \
        if gemm_ms > 0 else 0.0
    link = link_gbps()
    append_bytes = w.n_layer * P * 2 * w.E * 2  # K and V rows of the chunk into the repository
    line = {
        "metric": "prefill scoring + harvest us/step (config 4: 2048-token chunk x 2048 block "
                  "summaries x 64 layers, per-token top-256 union, append of 16 blocks x 64 "
                  "layers)",
        "value": round(ms_step * 1e3, 1), "unit": "us/step", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16 operands, f32 accumulate",
        "data": "synthetic: seeded N(0,1) x LogNormal channel scale history with "
                f"{w.n_planted} planted blocks; N(0,1) + 0.3 q0 chunk queries",
        "config": {"workload": f"{w.name}: {w.n_layer} layers, {w.n_head}q/{w.n_head_kv}kv, "
                               f"d{w.d_head}, {w.n_blocks} blocks + {P}-token chunks, top-{K}",
                   "l2": "inputs larger than L2 (2 GiB of chunk queries per step)"},
        "roofline": {"kernel": "gemm_f16_nt_kernel (tcgen05, TMEM accumulator)",
                     "bound": "tensor", "achieved": round(gemm_tf, 1), "peak": tc_peak,
                     "unit": "TFLOP/s", "frac": round(gemm_tf / tc_peak, 4), "traffic": None,
                     "peak_source": "measured bf16_tflops (burst)" if peaks else "fallback",
                     "avg_launch_ms": round(gemm_ms, 4),
                     "alg_flops_per_launch": prof["gemm_flops"] / max(1, prof["n_gemm"])},
        "step_roofline": {"append_bytes": append_bytes, "link_gbs_measured": round(link, 2),
                          "t_append_link_us": round(append_bytes / (link * 1e9) * 1e6, 1),
                          "frac": round(append_bytes / (link * 1e9) / (ms_step / 1e3), 4)},
        "union_blocks_last_step": n_union,
        "e2e": {"value": round(e2e_us, 1), "unit": "us/step",
                "h2d_bytes_per_step": int(qs[0].numel() * 2 + 2 * kvs[0][0].numel() * 2),
                "d2h_bytes_per_step": int(sel.numel())},
        "gpu_launches": int(prof["launches"]), "clocks": clk,
        "setup_s": round(t_setup, 1),
    }
    r.close()
    print(json.dumps(line), flush=True)


def host_mem_available():
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def run_lanes(args, w):
    """Config 5: `w.lanes` session lanes per GPU, each its own history and
    queries, layers split over the ranks; one step = every lane's query scored,
    one exchange for all lanes (N > 1), then every lane's top-k, plan and window
    assembly. The pinned host repositories of all lanes must fit the box's host
    memory; the per-lane history is shortened to fit when it does not, and the
    JSON line says so."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import kvmret
    from kvmret import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    if w.n_layer % world:
        raise SystemExit(f"{w.n_layer} layers do not split over {world} GPUs")
    Ll = w.n_layer // world
    layer0 = rank * Ll
    T, NL = w.block_tokens, w.lanes
    E = w.E
    row = kvmret.row_bytes(w.k_type, E) + kvmret.row_bytes(w.v_type, E)
    per_block = Ll * T * row
    avail = host_mem_available() // max(1, local_world)
    fit_blocks = int(0.75 * avail / (NL * per_block)) if avail else w.n_blocks
    n_blocks = max(w.budget_blocks + w.reserve_blocks + 64, min(w.n_blocks, fit_blocks))
    if world > 1:  # every rank must hold the same history length
        t = torch.tensor([n_blocks], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        n_blocks = int(t.item())
    wl = synth.scaled(w, n_blocks=n_blocks)
    t_setup = time.perf_counter()
    rs, hists = [], []
    for lane in range(NL):
        lw = synth.scaled(wl, seed=w.seed + 101 * lane)
        cfg = kvmret.default_config(
            n_layer=Ll, n_head=w.n_head, n_head_kv=w.n_head_kv, d_head=w.d_head,
            block_tokens=T, max_blocks=n_blocks, budget_blocks=w.budget_blocks,
            reserve_blocks=w.reserve_blocks, sink_blocks=w.sink_blocks, k_type=w.k_type,
            v_type=w.v_type, n_rot=w.d_head, freq_base=w.freq_base,
            pool_cache=int(args.pool_cache), device=local)
        r = kvmret.Retriever(cfg)
        h = synth.TorchHistory(lw, local, layer0=layer0, n_layer=Ll)
        for t0 in range(0, lw.n_tokens, 64 * T):
            m = min(64 * T, lw.n_tokens - t0)
            kc, vc = h.chunk(t0, m)
            r.append(kc, kvmret.quantize_f16(vc, w.v_type), k_rows=kvmret.quantize_f16(
                kc, w.k_type), pos0=t0)
            r.sync()
            del kc, vc
        rs.append(r)
        hists.append(h)
    lanes = kvmret.Lanes(rs)
    torch.cuda.synchronize()
    t_setup = time.perf_counter() - t_setup
    rows = torch.zeros(lanes.rows_per_rank, dtype=torch.float64, device="cuda")
    rows_all = rows if world == 1 else torch.zeros(world * lanes.rows_per_rank,
                                                  dtype=torch.float64, device="cuda")
    cur = torch.cuda.current_stream()

    def queries(n):
        return [[h.next_query()[layer0:layer0 + Ll].contiguous() for h in hists]
                for _ in range(n)]

    def step(qs):
        for r, q in zip(rs, qs):
            r.query_reset()
            r.query_add(q)
        lanes.score_layers(rows, stream=cur.cuda_stream)
        if world > 1:
            dist.all_gather_into_tensor(rows_all, rows)
        lanes.select_apply_async(rows_all, world, stream=cur.cuda_stream)

    def barrier():
        if world > 1:
            dist.barrier()

    clocks = Clocks(local)
    time.sleep(0.6)
    warm = queries(args.warmup)
    step(warm[0])
    ids0 = [ids for ids, _ in lanes.collect()]

    def restart():
        """Untimed: every lane's working set and pool emptied, the first
        warm-up step's selection staged again, then the other warm-up steps;
        the timed and the e2e loops both start from this state."""
        for r, ids in zip(rs, ids0):
            r.clear_working_set(drop_pool=True)
            r.apply(ids)
        for qs in warm[1:]:
            step(qs)
            lanes.collect()
        torch.cuda.synchronize()

    restart()
    qs_all = queries(args.steps)
    for r in rs:
        r.prof_enable(True)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stats = []
    e0.record(cur)
    for i, qs in enumerate(qs_all):
        step(qs)
        if i > 0:
            stats.append(lanes.collect())
    e1.record(cur)
    stats.append(lanes.collect())
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    profs = [r.prof_read() for r in rs]
    # e2e: the same queries, every lane's copied from pinned host memory each
    # step, the ids of the previous step read back on the host, from the same
    # start state as the timed loop
    qh = [[q.cpu().pin_memory() for q in qs] for qs in qs_all]
    qd = [torch.empty_like(q) for q in qs_all[0]]
    restart()
    barrier()
    torch.cuda.synchronize()
    e2e_res = []
    t0 = time.perf_counter()
    for i, qs in enumerate(qh):
        for d, q in zip(qd, qs):
            d.copy_(q, non_blocking=True)
        step(qd)
        if i > 0:
            e2e_res.append(lanes.collect())
    e2e_res.append(lanes.collect())
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_same = len(e2e_res) == len(stats) and all(
        np.array_equal(ia, ib) and sa["n_moved"] == sb["n_moved"] and
        sa["n_h2d_blocks"] == sb["n_h2d_blocks"]
        for ra, rb in zip(e2e_res, stats) for (ia, sa), (ib, sb) in zip(ra, rb))
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    hbm, peak_src = load_peaks()
    link = link_gbps()
    n_asm = sum(p["n_asm"] for p in profs)
    asm_ms = sum(p["asm_ms"] for p in profs)
    asm_hbm = sum(p["asm_hbm_bytes"] for p in profs)
    asm_link = sum(p["asm_link_bytes"] for p in profs)
    score_bytes = sum(p["score_bytes"] for p in profs) / max(1, args.steps)
    asm_step = asm_hbm / max(1, args.steps)
    link_step = asm_link / max(1, args.steps)
    t_roof = score_bytes / (hbm * 1e9) + max(link_step / (link * 1e9),
                                             (link_step + asm_step) / (hbm * 1e9))
    line = None
    if rank == 0:
        line = {
            "metric": "multi-lane retrieval+stage-in us/step (config 5: all lanes per step)",
            "value": round(ms_step * 1e3, 1), "unit": "us/step", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "q8_0/q4_0", "data": "synthetic: per-lane seeded histories and drifting "
                                          "queries (config 2's distributions)",
            "config": {"workload": f"{w.name}: {NL} lanes x {w.n_layer} layers, "
                                   f"{w.n_head}q/{w.n_head_kv}kv, d{w.d_head}, budget "
                                   f"{w.budget_blocks}, reserve {w.reserve_blocks}",
                       "history_tokens_per_lane": n_blocks * T,
                       "history_note": None if n_blocks >= w.n_blocks else
                       f"shortened from {w.n_tokens} to fit the pinned repositories of "
                       f"{NL} lanes into this box's host memory",
                       "layers_per_gpu": Ll, "parallelism": f"layer-sharded x{world}, "
                                                            f"{NL} lanes per GPU"},
            "roofline": {"kernel": "assemble_quant_kernel, all lanes", "bound": "hbm",
                         "achieved": round(asm_hbm / (asm_ms / 1e3) / 1e9, 1) if asm_ms else 0,
                         "peak": hbm, "unit": "GB/s",
                         "frac": round(asm_hbm / (asm_ms / 1e3) / 1e9 / hbm, 4) if asm_ms
                         else 0, "traffic": None, "peak_source": peak_src,
                         "note": "per-lane launches overlap, so the summed launch time "
                                 "exceeds the step's device time"},
            "step_roofline": {"t_roof_us": round(t_roof * 1e6, 1),
                              "frac": round(t_roof * 1e3 / ms_step, 4),
                              "B_sum": int(score_bytes), "B_link": int(link_step),
                              "B_asm": int(asm_step), "link_gbs_measured": round(link, 2)},
            "e2e": {"value": round(e2e_s / args.steps * 1e6, 1), "unit": "us/step",
                    "h2d_bytes_per_step": int(sum(q.numel() * 2 for q in qd)),
                    "d2h_bytes_per_step": int(NL * 4 * (w.budget_blocks + w.reserve_blocks)),
                    "same_steps_as_timed": e2e_same},
            "gpu_launches": int(sum(p["launches"] for p in profs)),
            "clocks": clk, "setup_s": round(t_setup, 1),
        }
    lanes.close()
    for r in rs:
        r.close()
    if world > 1:
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-pool-cache", dest="pool_cache", action="store_false",
                    help="free a block's HBM pool slot as soon as it leaves the window (the "
                         "reference's residency model); by default evicted blocks stay cached "
                         "in otherwise idle pool slots")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="N > 1: score-row exchange through NVLink peer memory written by the "
                         "scoring kernel (default), or an NCCL all-gather")
    ap.add_argument("--print-steps", action="store_true",
                    help="print each timed step's window-assembly counts to stderr (diagnostic)")
    ap.add_argument("--timeline", action="store_true",
                    help="record device events between the phases of each timed step (diagnostic)")
    ap.add_argument("--layers", type=int, default=0, help="override layer count (dev only)")
    ap.add_argument("--budget", type=int, default=0, help="override budget blocks (dev only)")
    ap.add_argument("--reserve", type=int, default=-1, help="override reserve slots (dev only)")
    ap.add_argument("--churn-h2d", type=int, default=6,
                    help="reference arm: blocks staged from the host per step (config 2 churn "
                         "measured by this bench without the pool cache: 6.2)")
    ap.add_argument("--churn-asm", type=int, default=168,
                    help="reference arm: window slots rewritten per step (measured: 167.6)")
    args = ap.parse_args()
    wl = workloads()
    w = wl.CONFIGS[args.config]
    if args.layers:
        w = wl.scaled(w, n_layer=args.layers)
    if args.budget:
        w = wl.scaled(w, budget_blocks=args.budget)
    if args.reserve >= 0:
        w = wl.scaled(w, reserve_blocks=args.reserve)
    if args.impl == "reference":
        run_reference(args, w)
    elif w.prefill_tokens:
        run_prefill(args, w)
    elif w.lanes:
        run_lanes(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
