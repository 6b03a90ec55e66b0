"""Layer sharding of the global block score (N > 1 without a GPU).

The reference's score is one mean over all layers (score_retrieval,
src/adapter/llama-memory-kvmem.cpp:4149-4196), so shards must exchange their
per-(layer, block) terms and every rank reduces them in global layer order.
Two `gloo` ranks each own half of the layers, compute their terms with the
oracle, all-gather them and reduce: the scores and the selected block ids must
equal the single-process oracle bit for bit.
"""
import os
import socket

import numpy as np
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case():
    rng = np.random.default_rng(42)
    N, L, Hq, Hkv, D = 96, 6, 16, 4, 64
    mean = rng.standard_normal((N, L, Hkv * D)).astype(np.float32)
    q_sum = rng.standard_normal((L, Hq * D)).astype(np.float32)
    q_count = np.array([1, 2, 0, 1, 3, 1], np.uint32)  # layer 2 carries no query
    has = np.ones(N, np.uint8)
    has[[5, 50]] = 0
    return mean, q_sum, q_count, has, (Hq, Hkv, D)


def _rank(rank, world, port, out):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "oracle"))
    import torch
    import torch.distributed as dist
    import pyoracle as po
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    mean, q_sum, q_count, has, (Hq, Hkv, D) = _case()
    L = mean.shape[1]
    per = L // world
    sl = slice(rank * per, (rank + 1) * per)
    terms, active = po.score_terms(mean[:, sl], q_sum[sl], q_count[sl], Hq, Hkv, D)
    t_all = [torch.zeros(per, mean.shape[0], dtype=torch.float64) for _ in range(world)]
    a_all = [torch.zeros(per, dtype=torch.uint8) for _ in range(world)]
    dist.all_gather(t_all, torch.from_numpy(terms))
    dist.all_gather(a_all, torch.from_numpy(active))
    scores = po.score_reduce(torch.cat(t_all).numpy(), torch.cat(a_all).numpy(), has)
    ids = po.pick_topk(scores, 12, 1)
    out[rank] = (scores.tobytes(), ids.tobytes())
    dist.destroy_process_group()


def test_two_gloo_ranks_reproduce_global_scores_and_selection():
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "oracle"))
    import pyoracle as po
    mean, q_sum, q_count, has, (Hq, Hkv, D) = _case()
    want = po.score(mean, has, q_sum, q_count, Hq, Hkv, D)
    want_ids = po.pick_topk(want, 12, 1)
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        scores = np.frombuffer(out[r][0], np.float64)
        ids = np.frombuffer(out[r][1], np.uint32)
        assert np.array_equal(scores, want)
        assert np.array_equal(ids, want_ids)


# ---------------------------------------------------------------------------
# Session lanes (config 5): each rank's exchange buffer is lane-major,
# [lane][local layer][block]; one all-gather for all lanes gives
# [rank][lane][local layer][block], and lane i's global rows are the
# [rank][i] slices in rank order (what kvmret_lanes_select_apply_async gathers
# with one strided copy per lane).

def _lane_case(lane):
    rng = np.random.default_rng(100 + lane)
    N, L, Hq, Hkv, D = 64, 4, 8, 2, 64
    mean = rng.standard_normal((N, L, Hkv * D)).astype(np.float32)
    q_sum = rng.standard_normal((L, Hq * D)).astype(np.float32)
    q_count = np.ones(L, np.uint32)
    has = np.ones(N, np.uint8)
    return mean, q_sum, q_count, has, (Hq, Hkv, D)


N_LANES = 3


def _lanes_rank(rank, world, port, out):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "oracle"))
    import torch
    import torch.distributed as dist
    import pyoracle as po
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rows, acts = [], []
    for lane in range(N_LANES):
        mean, q_sum, q_count, has, (Hq, Hkv, D) = _lane_case(lane)
        per = mean.shape[1] // world
        sl = slice(rank * per, (rank + 1) * per)
        t, a = po.score_terms(mean[:, sl], q_sum[sl], q_count[sl], Hq, Hkv, D)
        rows.append(torch.from_numpy(t))
        acts.append(torch.from_numpy(a))
    local = torch.stack(rows)                       # [lane][per][N]
    gathered = [torch.zeros_like(local) for _ in range(world)]
    dist.all_gather(gathered, local)                # one collective for every lane
    a_local = torch.stack(acts)
    a_gathered = [torch.zeros_like(a_local) for _ in range(world)]
    dist.all_gather(a_gathered, a_local)
    allr = torch.stack(gathered)                    # [rank][lane][per][N]
    alla = torch.stack(a_gathered)
    res = []
    for lane in range(N_LANES):
        terms = allr[:, lane].reshape(-1, allr.shape[-1]).numpy()   # [rank * per][N]
        active = alla[:, lane].reshape(-1).numpy()
        has = _lane_case(lane)[3]
        scores = po.score_reduce(terms, active, has)
        res.append(po.pick_topk(scores, 10, 1).tobytes())
    out[rank] = res
    dist.destroy_process_group()


def test_two_gloo_ranks_three_lanes_share_one_exchange():
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "oracle"))
    import pyoracle as po
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_lanes_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for lane in range(N_LANES):
        mean, q_sum, q_count, has, (Hq, Hkv, D) = _lane_case(lane)
        want = po.pick_topk(po.score(mean, has, q_sum, q_count, Hq, Hkv, D), 10, 1)
        for r in range(2):
            assert np.array_equal(np.frombuffer(out[r][lane], np.uint32), want)
