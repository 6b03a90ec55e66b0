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
def load_oracle():
    """The CPU oracle and, when built, the reference's own libkvmem (the
    checker of the parity pass and the CPU arms; never on the timed GPU path)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as po
    return po


def workload_config(w):
    """`config` of a decode-step line: the same keys and values in both arms."""
    sum_mib = w.n_layer * w.n_blocks * w.E * 4 / 2**20
    return {"workload": decode_workload(w)[0],
            "l2": f"inputs larger than L2: {sum_mib:.0f} MiB of block summaries read per step, "
                  "GiB-scale window and block repository"}


def _ptrs(addrs):
    import ctypes
    a = np.ascontiguousarray(addrs, np.uint64)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_void_p))


class CpuRetrieval:
    """One retrieval step of the workload on the host cores: the CPU arms
    (the `--impl reference` arm and the GPU arm's `cpu_baseline`).

    Per step, in full: the restated score_retrieval of every block on every
    layer (threads over blocks), the reference's pick_topk_blocks and
    KvMemRuntime set_selection (libkvmem compiled from the reference's
    sources; the oracle's restatement when it is not built), the staging
    memcpy of every stage-in block's K and V rows (all layers) from the host
    repository into a staging area, and for every block-layer the plan
    rebuilds (remap rows without skip) its K rotated by rope_neox_apply at
    the new window base (f16 in and out; q8_0 K: dequant -> RoPE -> FWHT ->
    requant) and its V rows copied into the window.

    Workload: the library arm's own history (TorchHistory, generated with
    torch on the GPU when one is present) with its block summaries computed by
    the library's arithmetic (token-order f32 sum x 1/T), and the same drifting
    query sequence, so both arms select the same blocks step by step; without
    a GPU, summaries drawn from the same distributions (N(0, 1/T) x channel
    scale, planted blocks +0.5 along the group query direction). With a decode
    tail the newest tail_blocks are this turn's decode blocks: each step
    appends one decode token and the top-k runs over the blocks before them
    (they stay in the window beyond the budget, as the library's gen mode
    keeps them). The host repository holds R distinct blocks (block b reads
    slot b mod R) and the window holds S slots (slot i writes i mod S): 1 GiB
    and 2 GiB, well above the host caches, so the copies and RoPE stream from
    and to DRAM as with the full-size arrays."""

    R, S = 32, 64

    def __init__(self, w, threads, use_ref=True, tail_blocks=0, source=None, decode=True):
        """source: (summaries [N][L][E] f32, next_query() -> [L][Hq*D] f16
        numpy); None: generate the workload here. decode: one decode token
        appended per step, the decode blocks (the newest tail_blocks and the
        token's block) kept beyond the budget."""
        import concurrent.futures as cf
        po = load_oracle()
        self.po, self.w = po, w
        self.use_ref = use_ref and po.ref is not None
        self.kind = "reference" if self.use_ref else "port"
        self.threads = threads
        self.pool = cf.ThreadPoolExecutor(max_workers=threads)
        TYPE_F16 = workloads().TYPE_F16
        self.f16 = w.k_type == TYPE_F16
        L, Hq, Hkv, D, N, T = w.n_layer, w.n_head, w.n_head_kv, w.d_head, w.n_blocks, \
            w.block_tokens
        rng = np.random.default_rng(w.seed)
        if source is None:
            source = cpu_workload(w, rng)
        self.mean, self._next_query = source
        self.has = np.ones(N, np.uint8)
        self.decode = decode
        self.gen_first = N - tail_blocks if decode else N
        E = w.E
        self.k_row = E * 2 if self.f16 else E // 32 * 34
        self.v_row = E * 2 if w.v_type == TYPE_F16 else (E // 32 * 34 if w.v_type == 8
                                                          else E // 32 * 18)
        self.kb, self.vb = T * self.k_row, T * self.v_row
        unit = self.kb + self.vb
        self.unit = unit
        # repository and window contents: N(0,1) f16 rows (quantised for q8_0 K)
        base = rng.standard_normal(T * E).astype(np.float32)
        if self.f16:
            kblk = base.astype(np.float16).view(np.uint8)
        else:
            kblk = po.quant_q8_0(base)
        vblk = (base.astype(np.float16).view(np.uint8) if w.v_type == TYPE_F16
                else (po.quant_q8_0(base) if w.v_type == 8 else po.quant_q4_0(base)))
        one = np.concatenate([kblk[:self.kb], vblk[:self.vb]])
        self.repo = np.empty((self.R, L, unit), np.uint8)
        self.repo[:] = one
        self.win = np.zeros((self.S, L, unit), np.uint8)
        self.slab = np.zeros((self.S, L, unit), np.uint8)  # staging area
        self.parts = [ix for ix in np.array_split(np.arange(N), threads) if len(ix)]
        if self.use_ref:
            self.rt = po.RefRuntime(T, w.budget_blocks, w.sink_blocks)
        else:
            self.rt = po.Store(T)
        self.rt.append(N * T)
        self.n_tok = N * T
        self.fwht_n = D if not self.f16 else 0

    def next_query(self):
        return self._next_query()

    def _score(self, q_sum):
        w, po = self.w, self.po
        q_count = np.ones(w.n_layer, np.uint32)
        out = list(self.pool.map(
            lambda ix: po.score(self.mean[ix[0]:ix[-1] + 1], self.has[ix[0]:ix[-1] + 1], q_sum,
                                q_count, w.n_head, w.n_head_kv, w.d_head), self.parts))
        return np.concatenate(out)

    def _split(self, n):
        k = max(1, min(self.threads, n))
        b = np.linspace(0, n, k + 1).astype(np.int64)
        return [(int(b[i]), int(b[i + 1])) for i in range(k) if b[i + 1] > b[i]]

    def step(self):
        """One full step; returns its counts."""
        w, po = self.w, self.po
        L = w.n_layer
        q_sum = self.next_query().astype(np.float32)
        scores = self._score(q_sum)
        g0 = self.gen_first
        if self.decode:  # one decode token per step
            self.rt.append(1)
            self.n_tok += 1
        nb = (self.n_tok + w.block_tokens - 1) // w.block_tokens
        if self.use_ref:
            ids = po.ref_pick_topk(scores[:g0], w.budget_blocks, w.sink_blocks)
        else:
            ids = po.pick_topk(scores[:g0], w.budget_blocks, w.sink_blocks)
        if g0 < nb:  # the decode blocks stay in the window beyond the budget
            ids = np.concatenate([ids, np.arange(g0, nb, dtype=ids.dtype)])
        si, so, rm, cnt = self.rt.set_selection(ids)
        # staging memcpy: every stage-in block's K and V rows of all layers
        import ctypes
        lyr = np.arange(L, dtype=np.uint64)
        rb, sb, wb = (np.uint64(a.ctypes.data) for a in (self.repo, self.slab, self.win))
        unit = np.uint64(self.unit)
        lib = po.ref if self.use_ref else po.orc
        si64 = np.asarray(si, np.uint64)
        if len(si64):
            src = rb + (((si64 % np.uint64(self.R))[:, None] * np.uint64(L) + lyr) * unit)
            dst = sb + (((np.arange(len(si64), dtype=np.uint64) % np.uint64(self.S))[:, None] *
                         np.uint64(L) + lyr) * unit)
            a_s, p_s = _ptrs(src.reshape(-1))
            a_d, p_d = _ptrs(dst.reshape(-1))
            a_n = np.full(a_s.size, self.unit, np.uint64)
            p_n = a_n.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))
            copy = lib.ref_copy_list if self.use_ref else lib.orc_copy_list
            list(self.pool.map(lambda r_: copy(p_s, p_d, p_n, r_[0], r_[1]),
                               self._split(a_s.size)))
        # window rebuild: every remapped block-layer (skip == 0)
        sel = np.nonzero(rm[:, 5] == 0)[0] if len(rm) else np.zeros(0, np.int64)
        moved = sel
        if len(sel):
            blk = rm[sel, 0].astype(np.uint64)
            o_src = ((blk % np.uint64(self.R))[:, None] * np.uint64(L) + lyr) * unit
            o_dst = ((sel.astype(np.uint64) % np.uint64(self.S))[:, None] * np.uint64(L) +
                     lyr) * unit
            a1, p1 = _ptrs((rb + o_src).reshape(-1))
            a2, p2 = _ptrs((wb + o_dst).reshape(-1))
            a3, p3 = _ptrs((rb + o_src + np.uint64(self.kb)).reshape(-1))
            a4, p4 = _ptrs((wb + o_dst + np.uint64(self.kb)).reshape(-1))
            pa = np.ascontiguousarray(np.repeat(rm[sel, 3], L), np.int32)
            pp = pa.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
            T, H, D = w.block_tokens, w.n_head_kv, w.d_head
            n_units = a1.size
            if self.f16:
                fn = lib.ref_rope_units_f16 if self.use_ref else lib.orc_rope_units_f16
                list(self.pool.map(lambda r_: fn(p1, p2, p3, p4, self.vb, pp, r_[0], r_[1], T, H,
                                                 D, w.freq_base, 1.0), self._split(n_units)))
            else:  # quantised K: the restated stage-in kernels (no host code in the reference)
                fn = po.orc.orc_rope_units_q8_0
                list(self.pool.map(lambda r_: fn(p1, p2, p3, p4, self.vb, pp, r_[0], r_[1], T, H,
                                                 D, w.freq_base, 1.0, self.fwht_n),
                                   self._split(n_units)))
        return {"n_stage_in": len(si), "n_rebuilt": len(moved), "ids": ids}

    def close(self):
        self.pool.shutdown()


def cpu_workload(w, rng):
    """(summaries [N][L][E] f32, next_query) of the workload: the library arm's
    own TorchHistory and query sequence when a GPU is present, else draws from
    the same distributions."""
    try:
        import torch
        gpu = torch.cuda.is_available()
    except ImportError:
        gpu = False
    if gpu:
        mean, h = workloads().torch_block_summaries(w, 0)
        return mean, lambda: h.next_query().reshape(w.n_layer, -1).cpu().numpy()
    L, Hq, Hkv, D, N, T = w.n_layer, w.n_head, w.n_head_kv, w.d_head, w.n_blocks, \
        w.block_tokens
    scale = np.exp(rng.normal(0.0, 0.5, size=(L, Hkv, D))).astype(np.float32)
    q0 = rng.standard_normal((L, Hq, D)).astype(np.float16)
    planted = workloads().planted_ids(w, rng)
    qg = q0.astype(np.float32).reshape(L, Hkv, Hq // Hkv, D).sum(axis=2)
    u = qg / np.linalg.norm(qg, axis=-1, keepdims=True)
    mean = rng.standard_normal((N, L, Hkv, D), dtype=np.float32)
    mean *= scale[None] / np.float32(np.sqrt(T))
    mean[planted] += np.float32(0.5) * u[None]
    state = {"q": q0.astype(np.float32), "rng": np.random.default_rng(w.seed + 7)}

    def next_query():
        q16 = state["q"].astype(np.float16)
        state["q"] = state["q"] + np.float32(w.drift) * state["rng"].standard_normal(
            q0.shape).astype(np.float32)
        return q16.reshape(L, -1)
    return mean.reshape(N, L, Hkv * D), next_query


def cpu_steps(w, steps, warmup, threads, use_ref=True, tail_blocks=0, source=None,
              decode=True):
    """Mean seconds per full CPU step over `steps` timed steps after `warmup`."""
    cpu = CpuRetrieval(w, threads, use_ref, tail_blocks, source, decode)
    for _ in range(warmup):
        cpu.step()
    times, stats = [], []
    for _ in range(steps):
        t0 = time.perf_counter()
        st = cpu.step()
        times.append(time.perf_counter() - t0)
        stats.append(st)
    cpu.close()
    churn = {"n_stage_in": round(sum(s["n_stage_in"] for s in stats) / len(stats), 2),
             "n_rebuilt": round(sum(s["n_rebuilt"] for s in stats) / len(stats), 2)}
    return sum(times) / len(times), cpu.kind, churn


def cpu_sample_text(w, kind, steps, warmup, threads):
    src = ("libkvmem from the reference's sources (pick_topk_blocks, KvMemRuntime "
           "set_selection, rope_neox_apply) + restated score_retrieval"
           if kind == "reference" else "the oracle's restatement of the path")
    return (f"{steps} timed steps (after {warmup} warm-up) of the full workload on "
            f"{threads} host threads, each step in full: score all {w.n_layer} layers x "
            f"{w.n_blocks} blocks, top-k, plan, staging memcpy of every stage-in block, "
            f"RoPE + V copy of every rebuilt block-layer; {src}")


# ---------------------------------------------------------------------------
def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    sec, kind, churn = cpu_steps(w, args.steps, args.warmup, threads, True,
                                 decode_tail(args, w), decode=not args.no_decode)
    us = sec * 1e6
    line = {"impl": "reference", "metric": METRIC, "value": round(us, 1), "unit": "us/step",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(us / 1e3, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": decode_workload(w)[1],
            "data": "synthetic: seeded N(0,1) x LogNormal(0,0.5) channel-scale summaries, "
                    f"{w.n_planted} planted blocks, query drift {w.drift}/step",
            "config": workload_config(w),
            "churn": churn,
            "cpu_baseline": {"value": round(us, 1), "unit": "us/step", "cores": threads,
                             "kind": kind,
                             "sample": cpu_sample_text(w, kind, args.steps, args.warmup,
                                                       threads)},
            "e2e": {"value": round(us, 1), "unit": "us/step", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# DRAM traffic of the window-assembly kernels per algorithmic byte: ncu's
# dram__bytes_read.sum + dram__bytes_write.sum over one captured launch divided
# by that launch's algorithmic bytes (8-layer cut of the same workload:
#   ncu --section MemoryWorkloadAnalysis --clock-control none -k regex:assemble
#       -s 20 -c 1 python bench.py --layers 8 --steps 5 --warmup 3 --config C
# ). The traffic grows with the blocks a launch moves, so a launch's traffic is
# this ratio times its algorithmic bytes.
NCU_TRAFFIC_RATIO = {"assemble_kernel": 1588.2 / 1619.0,
                     "assemble_quant_tma_kernel": 675.3 / 695.2}


class OracleCheck:
    """The checker of the parity pass (outside every timed region): the
    oracle's restated score_retrieval over host copies of this rank's block
    summaries, the per-layer terms of all ranks reduced in global layer order,
    pick_topk, and the set_selection plan replayed over every host-table
    operation of the run, plus the oracle RoPE / requantisation of sampled
    window slots from the pinned repository's bytes."""

    def __init__(self, po, w, r, Ll, world, threads, dist, gen_first):
        import concurrent.futures as cf
        self.po, self.w, self.r, self.Ll, self.world, self.dist = po, w, r, Ll, world, dist
        # the top-k candidates: the blocks before the decode blocks
        self.g0 = gen_first
        self.mean = np.ascontiguousarray(r.summaries()[:gen_first])  # [g0][Ll][E]
        N = self.mean.shape[0]
        self.N = N
        self.pool = cf.ThreadPoolExecutor(max_workers=max(1, threads))
        self.parts = [ix for ix in np.array_split(np.arange(N), max(1, threads)) if len(ix)]
        self.store = po.Store(w.block_tokens)  # replays the run's table log from empty
        self.tie_high = bool(r.cfg.tie_higher_id)

    def ids(self, q_host, n_blocks):
        """Oracle selection of one step's query ([Ll][1][qdim] f16, this rank's
        layers) over a store of n_blocks blocks: the top-k of the blocks before
        the decode blocks, plus the decode blocks."""
        import torch
        po, w = self.po, self.w
        q_sum = q_host.numpy().reshape(self.Ll, -1).astype(np.float32)
        q_count = np.ones(self.Ll, np.uint32)
        res = list(self.pool.map(
            lambda ix: po.score_terms(self.mean[ix[0]:ix[-1] + 1], q_sum, q_count, w.n_head,
                                      w.n_head_kv, w.d_head), self.parts))
        terms = np.concatenate([t for t, _ in res], axis=1)
        act = res[0][1]
        if self.world > 1:
            t = torch.from_numpy(np.ascontiguousarray(terms)).cuda().reshape(-1)
            t_all = torch.empty(self.world * t.numel(), dtype=t.dtype, device="cuda")
            self.dist.all_gather_into_tensor(t_all, t)
            a = torch.from_numpy(act.astype(np.uint8)).cuda()
            a_all = torch.empty(self.world * a.numel(), dtype=a.dtype, device="cuda")
            self.dist.all_gather_into_tensor(a_all, a)
            terms = t_all.cpu().numpy().reshape(-1, self.N)
            act = a_all.cpu().numpy()
        scores = po.score_reduce(terms, act, np.ones(self.N, np.uint8))
        ids = po.pick_topk(scores, w.budget_blocks, w.sink_blocks, tie_higher_id=self.tie_high)
        if n_blocks > self.g0:
            ids = np.concatenate([ids, np.arange(self.g0, n_blocks, dtype=ids.dtype)])
        return ids

    def replay(self, op):
        """One host-table operation of the run, in the oracle's store."""
        kind = op[0]
        if kind == "clear":
            self.store.clear_working_set(op[1])
        elif kind == "append":
            self.store.append(op[1])
        elif kind == "truncate":
            self.store.truncate(op[1])
        else:
            return self.store.set_selection(op[1])
        return None

    def summaries_exact(self):
        """Device summaries of sampled blocks against the oracle's token-order
        mean of the repository's unrotated f16 K rows (f16 K only)."""
        po, w, r = self.po, self.w, self.r
        repo = r.repo_view()
        unit = int(kvmret_lib().kvmret_repo_unit_bytes(r.h))
        T, E = w.block_tokens, w.E
        ok = True
        for b in sorted({0, self.N // 3, 2 * self.N // 3, self.N - 1}):
            for l in range(self.Ll):
                o = (b * self.Ll + l) * unit
                k = repo[o:o + T * E * 2].view(np.float16).reshape(1, T, E)
                ok &= bool(np.array_equal(po.mean_k(k)[0].view(np.uint32),
                                          self.mean[b, l].view(np.uint32)))
        return ok

    def window_slot(self, layer, slot, block, n_tok, base):
        """(K difference, V equal) of one window slot of one layer: f16 K in
        ulps; q8_0 K as (max |q| LSB, max scale ulp)."""
        po, w, r = self.po, self.w, self.r
        repo = r.repo_view()
        unit = int(kvmret_lib().kvmret_repo_unit_bytes(r.h))
        kbytes = int(kvmret_lib().kvmret_repo_k_bytes(r.h))
        o = (block * self.Ll + layer) * unit
        kr, vr = r.k_row, r.v_row
        src_k = np.array(repo[o:o + n_tok * kr])
        src_v = np.array(repo[o + kbytes:o + kbytes + n_tok * vr])
        win_k = r.window_read(layer, False, slot, 1)[:n_tok * kr]
        win_v = r.window_read(layer, True, slot, 1)[:n_tok * vr]
        H, D = w.n_head_kv, w.d_head
        if r.cfg.k_type == 1:
            want = po.rope_block_f16(src_k.view(np.uint16).reshape(n_tok, H, D), base,
                                     w.freq_base).reshape(-1)
            kd = int(f16_ulps(win_k.view(np.uint16), want).max(initial=0))
            kdiff = (kd, 0)
        else:
            want = po.rope_block_q8_0(src_k, n_tok, H, D, base, w.freq_base, fwht_n=D)
            kdiff = q8_diff(win_k, want)
        return kdiff, bool(np.array_equal(win_v, src_v))

    def close(self):
        self.pool.shutdown()


def kvmret_lib():
    import kvmret
    return kvmret.lib


def f16_ulps(a_bits, b_bits):
    a = np.asarray(a_bits, np.uint16).astype(np.int32)
    b = np.asarray(b_bits, np.uint16).astype(np.int32)
    oa = np.where(a & 0x8000, 0x8000 - a, a)
    ob = np.where(b & 0x8000, 0x8000 - b, b)
    return np.abs(oa - ob)


def q8_diff(a, b):
    a = np.asarray(a, np.uint8).reshape(-1, 34)
    b = np.asarray(b, np.uint8).reshape(-1, 34)
    qa = a[:, 2:].view(np.int8).astype(np.int32)
    qb = b[:, 2:].view(np.int8).astype(np.int32)
    da = a[:, :2].copy().view(np.uint16).reshape(-1)
    db = b[:, :2].copy().view(np.uint16).reshape(-1)
    return int(np.abs(qa - qb).max(initial=0)), int(f16_ulps(da, db).max(initial=0))


def decode_tail(args, w):
    """Decode blocks at the end of the history: at most what the gen reserve
    holds next to the loop's own decode block."""
    if args.no_decode:
        return 0
    spare = w.reserve_blocks - 1 - (args.warmup + args.steps + w.block_tokens - 1) // \
        w.block_tokens
    return max(0, min(args.decode_tail, spare, w.n_blocks - w.budget_blocks - 1))


def run_ours(args, w):
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
    T = w.block_tokens
    # decode: the newest `tail` blocks of the history are this turn's decode
    # blocks (appended in gen mode, pinned in reserve slots), and every step
    # appends one more decode token before its retrieval
    decoding = not args.no_decode
    tail = decode_tail(args, w)
    n_dec = args.warmup + args.steps  # decode tokens of one loop
    H0 = w.n_tokens                   # the history every loop starts from
    quant = w.k_type != kvmret.TYPE_F16

    max_blocks = w.n_blocks + (n_dec + T - 1) // T + 1
    # --hbm-resident: a pool with a slot for every block (the history is
    # copied into it before every measured loop)
    pool_blocks = min(8192, max_blocks + w.reserve_blocks) if args.hbm_resident else 0
    cfg = kvmret.default_config(
        n_layer=Ll, n_head=w.n_head, n_head_kv=w.n_head_kv, d_head=w.d_head, block_tokens=T,
        max_blocks=max_blocks, budget_blocks=w.budget_blocks,
        reserve_blocks=w.reserve_blocks, sink_blocks=w.sink_blocks, k_type=w.k_type,
        v_type=w.v_type, n_rot=w.d_head, freq_base=w.freq_base,
        pool_cache=int(args.pool_cache), pool_blocks=pool_blocks, device=local)
    t_setup = time.perf_counter()
    r = kvmret.Retriever(cfg)
    hist = synth.TorchHistory(w, local, layer0=layer0, n_layer=Ll)
    table_log = []  # every host-table operation of the run, in order

    def append(kc, vc, t0):
        if quant:  # config 3: q8_0 K rows, q4_0 V rows, summaries from the f16 capture
            r.append(kc, kvmret.quantize_f16(vc, w.v_type).view(Ll, kc.shape[1], -1),
                     k_rows=kvmret.quantize_f16(kc, w.k_type).view(Ll, kc.shape[1], -1), pos0=t0)
        else:
            r.append(kc, vc, pos0=t0)
        table_log.append(("append", int(kc.shape[1])))

    g0_tok = (w.n_blocks - tail) * T
    chunk = 64 * T  # the chunks torch_block_summaries generates, same random stream
    for t0 in range(0, w.n_tokens, chunk):
        m = min(chunk, w.n_tokens - t0)
        kc, vc = hist.chunk(t0, m)
        cut = min(max(g0_tok - t0, 0), m)  # tokens before the decode tail
        if cut:
            append(kc[:, :cut].contiguous(), vc[:, :cut].contiguous(), t0)
        if cut < m:
            if r.gen_first_block is None:
                r.gen_begin()
            append(kc[:, cut:].contiguous(), vc[:, cut:].contiguous(), t0 + cut)
        r.sync()
        del kc, vc
    if decoding and r.gen_first_block is None:
        r.gen_begin()
    # the decode tokens of one loop, one [Ll][1][row] tensor set per token
    dk, dv = hist.chunk(H0, n_dec)
    dec = []
    for i in range(n_dec):
        kc = dk[:, i:i + 1].contiguous()
        vc = dv[:, i:i + 1].contiguous()
        if quant:
            dec.append((kc, kvmret.quantize_f16(kc, w.k_type).view(Ll, 1, -1),
                        kvmret.quantize_f16(vc, w.v_type).view(Ll, 1, -1)))
        else:
            dec.append((kc, None, vc))
    del dk, dv
    torch.cuda.synchronize()
    t_setup = time.perf_counter() - t_setup
    if world > 1:  # every rank copies at once, as every rank's step reads the host at once
        dist.barrier()
    link = link_gbps()
    if world > 1:
        dist.barrier()
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

    def step(q_dev, d=None):
        mark("start")
        if d is not None:  # the decode token of this step (gen mode: into its reserve slot)
            r.append(d[0], d[2], k_rows=d[1])
            table_log.append(("append", 1))
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

    def collect():
        ids_k, st_k = r.step_collect()
        table_log.append(("sel", ids_k))
        return ids_k, st_k

    def queries(n):
        return [hist.next_query()[layer0:layer0 + Ll].contiguous() for _ in range(n)]

    def barrier():
        if world > 1:
            dist.barrier()

    # clocks are sampled from before the warm-up until after the last timed loop
    clocks = Clocks(local)
    time.sleep(0.6)
    warm_q = queries(args.warmup)
    warm_ids = []
    r_cache = [bool(args.pool_cache)]  # the pool's caching mode for the next loop

    def restart():
        """Untimed: the start state every measured loop begins from. The
        history cut back to its H0 tokens (the previous loop's decode tokens
        leave), an empty working set and pool (kvmret_clear_working_set), then
        the warm-up steps, each with its decode token (the first one stages
        the whole window from the host); the state (history, window, pool
        contents and LRU order) is then a function of these inputs alone, so
        every loop repeats the same work."""
        r.truncate(H0)
        table_log.append(("truncate", H0))
        r.clear_working_set(drop_pool=True)
        table_log.append(("clear", True))
        if args.hbm_resident and r_cache[0]:
            r.pool_prefetch(0, (H0 + T - 1) // T)
        warm_ids.clear()
        for j, q in enumerate(warm_q):
            step(q, dec[j] if decoding else None)
            warm_ids.append(collect()[0])
        r.sync()

    def timed_loop(qs):
        """Device time of exactly len(qs) steps on the library stream (max over
        ranks), with each step's ids and stats and the kernel timings."""
        restart()
        torch.cuda.synchronize()
        r.prof_enable(True)
        barrier()
        r.sync()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stats, ids_l = [], []
        marks.clear()
        e0.record(ext)
        # the host enqueues step k+1 before collecting step k, so the device never
        # waits for the host between steps. The NVTX range lets a profiler keep
        # only these launches (ncu --nvtx --nvtx-include "timed_steps/").
        torch.cuda.nvtx.range_push("timed_steps")
        W = len(warm_q)
        for i, q in enumerate(qs):
            step(q, dec[W + i] if decoding else None)
            if i > 0:
                ids_k, st_k = collect()
                ids_l.append(ids_k)
                stats.append(st_k)
        torch.cuda.nvtx.range_pop()
        e1.record(ext)
        ids_k, st_k = collect()
        ids_l.append(ids_k)
        stats.append(st_k)
        r.sync()
        torch.cuda.synchronize()
        barrier()
        prof = r.prof_read()
        r.prof_enable(False)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms / len(qs), ids_l, stats, prof

    def avg(key, ss):
        return sum(s[key] for s in ss) / len(ss)

    hbm, peak_src = load_peaks()
    asm_name = "assemble_kernel" if w.k_type == kvmret.TYPE_F16 else "assemble_quant_tma_kernel"

    def figures(ms_step, stats, prof):
        """Per-step byte counts, the assembly kernel's live roofline and the step roofline."""
        n_launch = max(1, prof["n_asm"])
        asm_ms = prof["asm_ms"] / n_launch
        asm_hbm = prof["asm_hbm_bytes"] / n_launch
        asm_link = prof["asm_link_bytes"] / n_launch
        achieved = asm_hbm / (asm_ms / 1e3) / 1e9 if asm_ms > 0 else 0.0
        t_asm_roof = max(asm_hbm / (hbm * 1e9), asm_link / (link * 1e9))
        h2d_step = avg("h2d_bytes", stats)
        asm_step = avg("assemble_bytes", stats)
        score_step = prof["score_bytes"] / max(1, prof["n_score"])
        score_ms = prof["score_ms"] / max(1, prof["n_score"])
        t_roof = score_step / (hbm * 1e9) + max(h2d_step / (link * 1e9),
                                                 (h2d_step + asm_step) / (hbm * 1e9))
        # the simple max form: every byte of the step at its link's peak, no
        # dependency between scoring and stage-in
        t_roof_max = max((score_step + h2d_step + asm_step) / (hbm * 1e9),
                         h2d_step / (link * 1e9))
        return {"asm_ms": asm_ms, "asm_hbm": asm_hbm, "asm_link": asm_link,
                "t_roof_max": t_roof_max,
                "achieved": achieved,
                "asm_frac": t_asm_roof / (asm_ms / 1e3) if asm_ms > 0 else 0.0,
                "h2d_step": h2d_step, "asm_step": asm_step, "score_step": score_step,
                "score_ms": score_ms,
                "score_gbs": score_step / (score_ms / 1e3) / 1e9 if score_ms > 0 else 0.0,
                "t_roof": t_roof, "step_frac": t_roof * 1e3 / ms_step,
                "churn": {"n_h2d_blocks": round(avg("n_h2d_blocks", stats), 2),
                          "n_moved": round(avg("n_moved", stats), 2),
                          "n_assembled": round(avg("n_assembled", stats), 2)}}

    # --- timed region: device time of exactly K steps on the library stream
    qs = queries(args.steps)
    qh = [q.cpu().pin_memory() for q in qs]  # the same K queries for the e2e loop
    ms_step, ids_timed, stats, prof = timed_loop(qs)
    timeline = None
    if args.timeline and marks:
        acc, cnt = {}, {}
        for (la, ea), (lb, eb) in zip(marks, marks[1:]):
            key = f"{la}->{lb}"
            acc[key] = acc.get(key, 0.0) + ea.elapsed_time(eb)
            cnt[key] = cnt.get(key, 0) + 1
        timeline = {k: round(acc[k] / cnt[k] * 1e3, 1) for k in acc}
        marks.clear()
    if args.print_steps and rank == 0:
        # per timed step: what the window assembly of that step moved (the
        # algorithmic bytes of a launch a profiler captured)
        for i, st in enumerate(stats):
            print(f"step {i}: n_moved {st['n_moved']} n_h2d {st['n_h2d_blocks']} "
                  f"assemble_bytes {st['assemble_bytes']} h2d_bytes {st['h2d_bytes']}",
                  file=sys.stderr)

    # --- e2e: the same K queries from pinned host memory -> device every step,
    # ids back on the host, from the same start state as the timed loop (its
    # selections and per-step work are checked against the timed loop's below)
    restart()
    qd = torch.empty_like(qs[0])
    W = len(warm_q)
    # this loop's decode rows in pinned host memory, and their device staging
    dec_h = [tuple(x.cpu().pin_memory() if x is not None else None for x in d)
             for d in dec[W:]] if decoding else []
    dec_d = tuple(torch.empty_like(x) if x is not None else None for x in dec[0]) if decoding \
        else None
    dec_bytes = sum(x.numel() * x.element_size() for x in dec[0] if x is not None) if decoding \
        else 0
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_stats, e2e_ids = [], []
    for i, q in enumerate(qh):
        qd.copy_(q, non_blocking=True)
        if decoding:
            for dst, src in zip(dec_d, dec_h[i]):
                if dst is not None:
                    dst.copy_(src, non_blocking=True)
        step(qd, dec_d)
        if i > 0:
            ids_k, st_k = collect()  # the previous step's ids, read on the host
            e2e_ids.append(ids_k)
            e2e_stats.append(st_k)
    ids_k, st_k = collect()
    e2e_ids.append(ids_k)
    e2e_stats.append(st_k)
    r.sync()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_us = e2e_s / args.steps * 1e6
    e2e_same = (len(e2e_ids) == len(ids_timed) and
                all(np.array_equal(a, b) for a, b in zip(e2e_ids, ids_timed)) and
                all(a["n_moved"] == b["n_moved"] and a["n_h2d_blocks"] == b["n_h2d_blocks"]
                    for a, b in zip(e2e_stats, stats)))

    # --- the other residency, same queries and start state (a sub-result)
    other = None
    if not args.no_residency_variant:
        r.set_pool_cache(not args.pool_cache)
        r_cache[0] = not args.pool_cache
        ms_o, ids_o, stats_o, prof_o = timed_loop(qs)
        r.set_pool_cache(args.pool_cache)
        r_cache[0] = args.pool_cache
        fo = figures(ms_o, stats_o, prof_o)
        other = {"pool_cache": not args.pool_cache,
                 "residency": ("HBM pool keeps evicted blocks in idle slots" if not
                               args.pool_cache else "only the working set on the GPU (the "
                                                    "reference's residency)"),
                 "value": round(ms_o * 1e3, 1), "unit": "us/step",
                 "same_ids_as_timed": all(np.array_equal(a, b) for a, b in zip(ids_o, ids_timed)),
                 "churn": fo["churn"],
                 "step_roofline": {"t_roof_us": round(fo["t_roof"] * 1e6, 1),
                                   "frac": round(fo["step_frac"], 4)},
                 "assembly": {"avg_launch_ms": round(fo["asm_ms"], 4),
                              "frac": round(fo["asm_frac"], 4),
                              "bound": "hbm" if fo["asm_hbm"] / hbm >= fo["asm_link"] / link
                              else "host link"}}

    # --- parity pass (untimed): the same steps once more from the same start
    # state, one at a time, each checked against the oracle
    parity = None
    if not args.no_parity:
        po = load_oracle()
        threads = max(1, (os.cpu_count() or 1) // max(1, local_world))
        chk = OracleCheck(po, w, r, Ll, world, threads, dist, w.n_blocks - tail)
        restart()
        for op in table_log:
            chk.replay(op)
        nb_at = lambda j: (H0 + (j + 1 if decoding else 0) + T - 1) // T  # noqa: E731
        oracle_warm = [chk.ids(q.cpu(), nb_at(j)) for j, q in enumerate(warm_q)]
        ok_ids = all(np.array_equal(a, b) for a, b in zip(warm_ids, oracle_warm))
        ok_plan = ok_layout = ok_v = ok_timed = True
        k_max, k_scale_max, n_slots = 0, 0, 0
        pass_ids = []
        for i, q in enumerate(qs):
            step(q, dec[W + i] if decoding else None)
            if decoding:
                chk.replay(("append", 1))
            ids_d, _ = collect()
            plan = r.last_plan()
            lay, bases = r.window_layout()
            want = chk.ids(qh[i], nb_at(W + i))
            si, so, rm, _ = chk.store.set_selection(want)
            pass_ids.append(ids_d)
            ok_ids &= bool(np.array_equal(ids_d, want))
            ok_timed &= bool(np.array_equal(ids_d, ids_timed[i]))
            ok_plan &= bool(np.array_equal(plan.remaps, rm) and np.array_equal(plan.stage_in, si)
                            and np.array_equal(plan.stage_out, so))
            ok_layout &= bool(np.array_equal(lay, rm[:, 0].astype(np.uint32)) and
                              np.array_equal(bases, rm[:, 3]))
            n = len(rm)
            rebuilt = np.nonzero(rm[:, 5] == 0)[0]
            slots = {n - 1, (i * 37) % n}
            if len(rebuilt):
                slots.add(int(rebuilt[(i * 13) % len(rebuilt)]))
            for sl in sorted(slots):
                for layer in sorted({0, Ll - 1}):
                    (kd, ksd), v_eq = chk.window_slot(layer, sl, int(rm[sl, 0]), int(rm[sl, 1]),
                                                      int(rm[sl, 3]))
                    k_max, k_scale_max = max(k_max, kd), max(k_scale_max, ksd)
                    ok_v &= v_eq
                    n_slots += 1
        summ_ok = chk.summaries_exact() if w.k_type == kvmret.TYPE_F16 else None
        chk.close()
        flags = torch.tensor([ok_ids, ok_plan, ok_layout, ok_v, ok_timed, e2e_same,
                              summ_ok is not False], dtype=torch.int32, device="cuda")
        mx = torch.tensor([k_max, k_scale_max], dtype=torch.int32, device="cuda")
        across = True
        if world > 1:
            dist.all_reduce(flags, op=dist.ReduceOp.MIN)
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            mine = b"".join(a.astype(np.uint32).tobytes() for a in pass_ids)
            allr = [None] * world
            dist.all_gather_object(allr, mine)
            across = all(x == allr[0] for x in allr)
        f = [bool(x) for x in flags.tolist()]
        kx = mx.tolist()
        parity = {
            "checker": "oracle/kvmret_oracle.cpp: restated score_retrieval (terms reduced over "
                       "all layers in layer order), pick_topk, set_selection replayed over "
                       "every host-table operation of the run, RoPE / dequant-RoPE-FWHT-requant "
                       "of window slots from the pinned repository's bytes",
            "steps_checked": len(warm_q) + len(qs),
            "ids_bit_exact": f[0], "timed_ids_equal_checked_ids": f[4],
            "plan_rows_exact": f[1], "window_layout_exact": f[2],
            "window_slots_checked": n_slots * (world if world > 1 else 1),
            "window_v_exact": f[3],
            "summaries_bit_exact": (f[6] if summ_ok is not None else None),
        }
        if w.k_type == kvmret.TYPE_F16:
            parity["window_k_max_ulp"] = kx[0]
        else:
            parity["window_k_max_lsb"] = kx[0]
            parity["window_k_scale_max_ulp"] = kx[1]
            parity["summaries_note"] = ("quantised K: the repository holds q8_0 rows, the "
                                        "summaries come from the f16 capture")
        if world > 1:
            parity["ids_equal_across_ranks"] = across

    clk = clocks.stop()
    fg = figures(ms_step, stats, prof)
    kv_bytes = fg["score_step"] + fg["h2d_step"] + fg["asm_step"]
    asm_traffic = NCU_TRAFFIC_RATIO[asm_name] * fg["asm_hbm"]

    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(ms_step * 1e3, 1), "unit": "us/step",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": decode_workload(w)[1],
            "data": "synthetic: seeded N(0,1) x LogNormal(0,0.5) channel scale, "
                    f"{w.n_planted} planted blocks, query drift {w.drift}/step",
            "config": workload_config(w),
            "setup": {"layers_per_gpu": Ll, "parallelism": f"layer-sharded x{world}",
                      "exchange": (args.exchange if world > 1 else None),
                      "pool_cache": bool(args.pool_cache),
                      "pool_slots": int(pool_blocks or (w.budget_blocks + w.reserve_blocks)),
                      "residency": ("hbm-resident: a pool slot for every block, the whole "
                                    "history copied into the HBM pool before each measured "
                                    "loop (kvmret_pool_prefetch)" if args.hbm_resident else
                                    "pool of the window's size (budget + reserve slots), "
                                    "caching evicted blocks in idle slots" if args.pool_cache
                                    else "only the working set on the GPU"),
                      "decode": ({"tail_blocks": tail, "tokens_per_step": 1,
                                  "note": "the newest tail blocks are this turn's decode "
                                          "blocks, pinned in gen-reserve window slots "
                                          "(kvmret_gen_begin); every step first appends "
                                          "one decode token into its reserve slot"}
                                 if decoding else None)},
            "roofline": {"kernel": asm_name + " (window assembly: moved slots from the HBM "
                                              "pool, fresh slots from the host repository)",
                         "bound": "hbm" if fg["asm_hbm"] / hbm >= fg["asm_link"] / link
                         else "host link",
                         "achieved": round(fg["achieved"], 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(fg["asm_frac"], 4), "traffic": int(asm_traffic),
                         "traffic_source": "ncu dram read + write bytes per algorithmic byte "
                                           "of an 8-layer capture, times this launch's "
                                           "algorithmic bytes",
                         "peak_source": peak_src,
                         "avg_launch_ms": round(fg["asm_ms"], 4),
                         "alg_hbm_bytes_per_launch": int(fg["asm_hbm"]),
                         "alg_link_bytes_per_launch": int(fg["asm_link"]),
                         "link_gbs_measured": round(link, 2)},
            "kernels": {
                "score": {"ms": round(fg["score_ms"], 4), "GB/s": round(fg["score_gbs"], 1),
                          "frac_hbm": round(fg["score_gbs"] / hbm, 4)}},
            "step_roofline": {"t_roof_us": round(fg["t_roof"] * 1e6, 1),
                              "t_meas_us": round(ms_step * 1e3, 1),
                              "frac": round(fg["step_frac"], 4),
                              "t_roof_max_form_us": round(fg["t_roof_max"] * 1e6, 1),
                              "frac_max_form": round(fg["t_roof_max"] * 1e3 / ms_step, 4),
                              "link_gbs_measured": round(link, 2),
                              "link_d2h_gbs_measured": round(link_d2h, 2), "hbm_gbs": hbm,
                              "B_sum": int(fg["score_step"]), "B_link": int(fg["h2d_step"]),
                              "B_asm": int(fg["asm_step"])},
            "kv_gbps": round(kv_bytes / (ms_step / 1e3) / 1e9, 1),
            "churn": fg["churn"],
            "other_residency": other,
            "parity": parity,
            "e2e": {"value": round(e2e_us, 1), "unit": "us/step",
                    "h2d_bytes_per_step": int(qs[0].numel() * 2 + dec_bytes +
                                              avg("h2d_bytes", e2e_stats)),
                    # per step the readback ring returns 8 counts and the window's ids
                    "d2h_bytes_per_step": int(4 * (8 + w.budget_blocks + w.reserve_blocks)),
                    "same_steps_as_timed": e2e_same,
                    "churn": {"n_h2d_blocks": round(avg("n_h2d_blocks", e2e_stats), 2),
                              "n_moved": round(avg("n_moved", e2e_stats), 2)}},
            "gpu_launches": int(prof["launches"]),
            "timeline_us": timeline,
            "clocks": clk,
            "setup_s": round(t_setup, 1),
        }
    summ_host = r.summaries()[:w.n_blocks] if line is not None and world == 1 else None
    r.close()
    if world > 1:
        dist.destroy_process_group()
    if line is not None and world == 1 and not args.no_cpu_baseline:
        # the same workload on the host cores: this run's summaries and the
        # same query sequence (a fresh generator of it)
        threads = os.cpu_count() or 1
        qgen = synth.TorchHistory(w, local)
        src = (summ_host, lambda: qgen.next_query().reshape(w.n_layer, -1).cpu().numpy())
        sec, kind, churn = cpu_steps(w, 3, 1, threads, True, tail, src, decoding)
        line["cpu_baseline"] = {"value": round(sec * 1e6, 1), "unit": "us/step",
                                "cores": threads, "kind": kind,
                                "sample": cpu_sample_text(w, kind, 3, 1, threads),
                                "churn": churn}
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
    if world > 1:  # every rank copies at once, as in the step
        dist.barrier()
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
            "roofline": {"kernel": "assemble_quant_tma_kernel, all lanes", "bound": "hbm",
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
    ap.add_argument("--hbm-resident", action="store_true",
                    help="a pool slot for every block, the whole history copied into the HBM "
                         "pool before each measured loop (kvmret_pool_prefetch); the default "
                         "keeps the pool at the window's size")
    ap.add_argument("--decode-tail", type=int, default=64,
                    help="blocks at the end of the history generated in this turn (decode "
                         "blocks pinned in gen-reserve slots)")
    ap.add_argument("--no-decode", action="store_true",
                    help="retrieval steps only: no decode token per step, no gen-reserve "
                         "placement")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the untimed parity pass against the CPU oracle")
    ap.add_argument("--no-residency-variant", action="store_true",
                    help="skip the timed loop under the other pool residency")
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
