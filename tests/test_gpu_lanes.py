"""Session lanes (config 5 at test scale): several conversations on one GPU
stepped together through kvmret_lanes_* — each lane with its own seeded
history and queries, q8_0 K / q4_0 V — must select exactly the blocks the
oracle selects for that lane alone and build the same window layout; and on 2
GPUs with the layers split, one NCCL all-gather carries every lane's terms.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import kvmret
import pyoracle as po
from kvm_helpers import append_history, config_for, oracle_scores, q8_blocks_diff
from kvmret import synth

pytestmark = pytest.mark.gpu

N_LANES = 3


def _lane_workload(lane, n_layer=2):
    return synth.scaled(synth.CONFIGS[3], n_layer=n_layer, n_blocks=40, budget_blocks=10,
                        reserve_blocks=3, n_planted=4, n_head=16, seed=500 + lane)


def _quant_rows(fn, row_bytes):
    def f(x):
        L, n, E = x.shape
        return fn(x.astype(np.float32)).reshape(L, n, row_bytes)
    return f


KQ = _quant_rows(po.quant_q8_0, 1088)
VQ = _quant_rows(po.quant_q4_0, 576)


def test_lanes_on_one_gpu_match_per_lane_oracle():
    ws = [_lane_workload(i) for i in range(N_LANES)]
    hists = [synth.NumpyHistory(w) for w in ws]
    rs = [kvmret.Retriever(config_for(w)) for w in ws]
    for r, h in zip(rs, hists):
        append_history(r, h, cuts=[700], k_rows_fn=KQ, v_rows_fn=VQ)
    lanes = kvmret.Lanes(rs)
    w0 = ws[0]
    rows = torch.zeros(lanes.rows_per_rank, dtype=torch.float64, device="cuda")
    qs = [h.queries(3) for h in hists]
    stores = []
    for w in ws:
        st = po.Store(w.block_tokens)
        st.append(w.n_tokens)
        stores.append(st)
    for s in range(3):
        for r, w, q in zip(rs, ws, qs):
            r.query_reset()
            r.query_add(torch.from_numpy(q[s].reshape(w.n_layer, 1, -1)).cuda())
        lanes.score_layers(rows)
        lanes.select_apply_async(rows, 1, mandatory=[[], [w0.n_blocks - 1], []])
        got = lanes.collect()
        for i, (r, w, h, q) in enumerate(zip(rs, ws, hists, qs)):
            want, _ = oracle_scores(h, q[s].reshape(w.n_layer, -1).astype(np.float32),
                                    np.ones(w.n_layer, np.uint32))
            mand = [w.n_blocks - 1] if i == 1 else []
            want_ids = po.pick_topk(want, w.budget_blocks, w.sink_blocks, 0, mand)
            assert list(got[i][0]) == list(want_ids), (s, i)
            _, _, rm, _ = stores[i].set_selection(want_ids)
            lay, bases = r.window_layout()
            assert list(lay) == list(rm[:, 0]) and list(bases) == list(rm[:, 3])
    # windows of the last step: requantised K within 1 LSB, V exact
    for r, w, h in zip(rs, ws, hists):
        L, n, E = w.n_layer, w.n_tokens, w.E
        kq = KQ(h.k.reshape(L, n, E)).reshape(L, w.n_blocks, -1)
        vq = VQ(h.v.reshape(L, n, E)).reshape(L, w.n_blocks, -1)
        lay, bases = r.window_layout()
        for l in range(L):
            wk = r.window_read(l, False, 0, len(lay)).reshape(len(lay), -1)
            wv = r.window_read(l, True, 0, len(lay)).reshape(len(lay), -1)
            for j, (b, base) in enumerate(zip(lay, bases)):
                want_k = po.rope_block_q8_0(kq[l, b], w.block_tokens, w.n_head_kv, w.d_head,
                                            int(base), w.freq_base, fwht_n=128)
                dq, dd = q8_blocks_diff(wk[j], want_k)
                assert dq <= 1 and dd <= 1
                assert np.array_equal(wv[j], vq[l, b])
    lanes.close()
    for r in rs:
        r.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, out):
    import sys
    from datetime import timedelta
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (here, os.path.join(root, "kvmem-llama.cpp_b200"), os.path.join(root, "oracle")):
        sys.path.insert(0, p)
    import torch.distributed as dist
    import kvmret
    from kvm_helpers import config_for
    from kvmret import synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ws = [_lane_workload(i, n_layer=4) for i in range(2)]
    hists = [synth.NumpyHistory(w) for w in ws]
    Ll = 4 // world
    sl = slice(rank * Ll, (rank + 1) * Ll)
    rs = []
    for w, h in zip(ws, hists):
        r = kvmret.Retriever(config_for(w, n_layer=Ll, device=rank))
        n = w.n_tokens
        k = np.ascontiguousarray(h.k.reshape(w.n_layer, n, w.E)[sl])
        v = np.ascontiguousarray(h.v.reshape(w.n_layer, n, w.E)[sl])
        r.append(torch.from_numpy(k).cuda(), torch.from_numpy(VQ(v)).cuda(),
                 k_rows=torch.from_numpy(KQ(k)).cuda())
        r.sync()
        rs.append(r)
    lanes = kvmret.Lanes(rs)
    local = torch.zeros(lanes.rows_per_rank, dtype=torch.float64, device="cuda")
    allr = torch.zeros(world * lanes.rows_per_rank, dtype=torch.float64, device="cuda")
    qs = [h.queries(2) for h in hists]
    res = []
    for s in range(2):
        for r, w, q in zip(rs, ws, qs):
            r.query_reset()
            r.query_add(torch.from_numpy(np.ascontiguousarray(
                q[s].reshape(w.n_layer, 1, -1)[sl])).cuda())
        lanes.score_layers(local)
        dist.all_gather_into_tensor(allr, local)  # one collective for every lane
        lanes.select_apply_async(allr, world)
        res.append([ids.tobytes() for ids, _ in lanes.collect()])
    out[rank] = res
    lanes.close()
    for r in rs:
        r.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_lanes_layer_sharded_over_two_gpus():
    ws = [_lane_workload(i, n_layer=4) for i in range(2)]
    hists = [synth.NumpyHistory(w) for w in ws]
    qs = [h.queries(2) for h in hists]
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for s in range(2):
        for i, (w, h, q) in enumerate(zip(ws, hists, qs)):
            want, _ = oracle_scores(h, q[s].reshape(w.n_layer, -1).astype(np.float32),
                                    np.ones(w.n_layer, np.uint32))
            want_ids = po.pick_topk(want, w.budget_blocks, w.sink_blocks)
            for rank in range(2):
                assert np.array_equal(np.frombuffer(out[rank][s][i], np.uint32), want_ids)
