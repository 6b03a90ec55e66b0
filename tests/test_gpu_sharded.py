"""Layer-sharded retrieval on 2 GPUs: each rank's context owns half of the
layers; the per-(layer, block) score terms, with each layer's query flag in
the last column of its row, are exchanged (an NCCL all-gather, or peer
memory: each rank's rows in its own region, read by every rank's reduction
over NVLink after the rank's step flag) and reduced in global layer order,
so every rank
selects the same blocks as the single-context oracle, bit for bit, and
assembles its own layers' windows (skipped with fewer than 2 GPUs). On one
GPU: the peer-memory exchange's bounded wait when a rank never writes.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, out, exchange="nccl", quant=False):
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
    w = synth.scaled(synth.CONFIGS[1], n_layer=4, n_blocks=96, budget_blocks=12, n_planted=4)
    if quant:
        w = synth.scaled(w, k_type=kvmret.TYPE_Q8_0, v_type=kvmret.TYPE_Q4_0)
    hist = synth.NumpyHistory(w)
    Ll = w.n_layer // world
    sl = slice(rank * Ll, (rank + 1) * Ll)
    r = kvmret.Retriever(config_for(w, n_layer=Ll, device=rank))
    n = w.n_tokens
    k = torch.from_numpy(np.ascontiguousarray(hist.k.reshape(w.n_layer, n, w.E)[sl])).cuda()
    v = torch.from_numpy(np.ascontiguousarray(hist.v.reshape(w.n_layer, n, w.E)[sl])).cuda()
    if quant:  # q8_0 K rows, q4_0 V rows, summaries from the f16 capture
        r.append(k, kvmret.quantize_f16(v, w.v_type).view(Ll, n, -1),
                 k_rows=kvmret.quantize_f16(k, w.k_type).view(Ll, n, -1))
    else:
        r.append(k, v)
    stride = r.contrib_stride
    c_loc = torch.zeros(Ll * stride, dtype=torch.float64, device="cuda")
    c_all = torch.zeros(w.n_layer * stride, dtype=torch.float64, device="cuda")
    if exchange == "p2p":
        handles = [None] * world
        dist.all_gather_object(handles, r.exchange_export(world))
        r.exchange_import(rank, handles)
    q = hist.queries(3)
    res = []
    # the same three queries twice: through select + apply, then through the
    # GPU-resident step (select_apply_async + step_collect)
    for s in range(6):
        r.query_reset()
        r.query_add(torch.from_numpy(np.ascontiguousarray(
            q[s % 3].reshape(w.n_layer, 1, -1)[sl])).cuda())
        if exchange == "p2p":
            r.score_exchange()
        else:
            r.score_layers(c_loc)
            r.sync()
            dist.all_gather_into_tensor(c_all, c_loc)
            torch.cuda.synchronize()
            r.score_reduce(c_all, w.n_layer)
        if s < 3:
            ids = r.select()
            r.apply(ids)
        else:
            r.select_apply_async()
            ids = r.step_collect()[0]
        lay, bases = r.window_layout()
        res.append((ids.tobytes(), lay.tobytes(), bases.tobytes()))
    out[rank] = res
    r.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange,quant", [("nccl", False), ("p2p", False), ("p2p", True)])
def test_two_gpu_layer_sharded_selection_matches_oracle(exchange, quant):
    import pyoracle as po
    from kvm_helpers import oracle_scores
    from kvmret import synth
    w = synth.scaled(synth.CONFIGS[1], n_layer=4, n_blocks=96, budget_blocks=12, n_planted=4)
    hist = synth.NumpyHistory(w)
    q = hist.queries(3)
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out, exchange, quant))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    store = po.Store(w.block_tokens)
    store.append(w.n_tokens)
    for s in range(6):
        want, _ = oracle_scores(hist, q[s % 3].reshape(w.n_layer, -1).astype(np.float32),
                                np.ones(w.n_layer, np.uint32))
        want_ids = po.pick_topk(want, w.budget_blocks, w.sink_blocks)
        _, _, rm, _ = store.set_selection(want_ids)
        for rank in range(2):
            ids, lay, bases = (np.frombuffer(b, t) for b, t in
                               zip(out[rank][s], (np.uint32, np.uint32, np.int32)))
            assert np.array_equal(ids, want_ids)
            assert np.array_equal(lay, rm[:, 0].astype(np.uint32))
            assert np.array_equal(bases, rm[:, 3])


def _silent_rank(w_kwargs, q_handle, q_done):
    """Rank 1 of a 2-rank exchange that exports its region (same geometry as
    rank 0's) and then never scores: its flag is never set."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (here, os.path.join(root, "kvmem-llama.cpp_b200")):
        sys.path.insert(0, p)
    import kvmret
    from kvm_helpers import config_for
    from kvmret import synth
    r = kvmret.Retriever(config_for(synth.Workload(**w_kwargs)))
    q_handle.put(r.exchange_export(2))
    q_done.get(timeout=300)
    r.close()


def test_exchange_wait_gives_up_when_a_rank_never_writes():
    """The reduce's wait on a peer's flag is bounded (2 s): the step then fails
    with plan error 0x100, the window stays as it was, and the context keeps
    working. One GPU: the silent rank is a second process that only exports."""
    import time
    import kvmret
    import pyoracle as po
    from kvm_helpers import append_history, config_for, oracle_scores
    from kvmret import synth
    wk = dict(name="ex", n_layer=2, n_head=8, n_head_kv=2, d_head=128, block_tokens=64,
              n_blocks=32, budget_blocks=6, sink_blocks=1, reserve_blocks=0, n_planted=2,
              seed=61)
    ctx = mp.get_context("spawn")
    q_handle, q_done = ctx.Queue(), ctx.Queue()
    p = ctx.Process(target=_silent_rank, args=(wk, q_handle, q_done))
    p.start()
    try:
        w = synth.Workload(**wk)
        hist = synth.NumpyHistory(w)
        r = kvmret.Retriever(config_for(w))
        append_history(r, hist, cuts=[])
        before = r.apply([0, 5, 9])
        assert before["n_selected"] == 3
        h0 = r.exchange_export(2)
        h1 = q_handle.get(timeout=300)
        r.exchange_import(0, [h0, h1])
        q = hist.queries(1)[0]
        r.query_reset()
        r.query_add(torch.from_numpy(q.reshape(w.n_layer, 1, -1)).cuda())
        t0 = time.monotonic()
        r.score_exchange()
        r.select_apply_async()
        with pytest.raises(kvmret.KvmretError, match="0x100"):
            r.step_collect()
        assert 1.5 < time.monotonic() - t0 < 60
        assert list(r.window_layout()[0]) == [0, 5, 9]  # the failed step changed nothing
        # a local step on the same context afterwards selects the oracle's blocks
        got = r.score()
        want, _ = oracle_scores(hist, q.reshape(w.n_layer, -1).astype(np.float32),
                                np.ones(w.n_layer, np.uint32))
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64))
        ids = r.select()
        assert list(ids) == list(po.pick_topk(want, w.budget_blocks, w.sink_blocks))
        st = r.apply(ids)
        assert list(r.window_layout()[0]) == sorted(ids.tolist()) and st["n_selected"] == len(ids)
        r.close()
    finally:
        q_done.put(1)
        p.join(timeout=120)
    assert p.exitcode == 0


def _empty_rank(w_kwargs, q_handle, q_peer, q_done):
    """Rank 1 of a 2-rank exchange whose history holds no block: it scores
    once (no query rows), which must still publish its step flag to rank 0;
    its own wait for rank 0 (which has not scored yet) gives up after 2 s."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (here, os.path.join(root, "kvmem-llama.cpp_b200")):
        sys.path.insert(0, p)
    import kvmret
    from kvm_helpers import config_for
    from kvmret import synth
    r = kvmret.Retriever(config_for(synth.Workload(**w_kwargs)))
    h1 = r.exchange_export(2)
    q_handle.put(h1)
    h0 = q_peer.get(timeout=300)
    r.exchange_import(1, [h0, h1])
    r.query_reset()
    r.score_exchange()
    r.select_apply_async()
    try:
        r.step_collect()
        status = "ok"
    except kvmret.KvmretError as e:
        status = str(e)
    r.sync()
    q_done.put(status)
    q_peer.get(timeout=300)  # rank 0 finished with this rank's region
    r.close()


def test_exchange_rank_with_empty_history_still_signals():
    """A rank with no blocks yet takes part in the step protocol: rank 0 (with
    a history) completes its exchange step at once, with the oracle's
    selection over its own layers (rank 1 contributes no query rows), instead
    of timing out. The ranks' steps run one after the other, never as two
    waiting kernels at the same time."""
    import time
    import kvmret
    import pyoracle as po
    from kvm_helpers import append_history, config_for, oracle_scores
    from kvmret import synth
    wk = dict(name="ex0", n_layer=2, n_head=8, n_head_kv=2, d_head=128, block_tokens=64,
              n_blocks=32, budget_blocks=6, sink_blocks=1, reserve_blocks=0, n_planted=2,
              seed=62)
    ctx = mp.get_context("spawn")
    q_handle, q_peer, q_done = ctx.Queue(), ctx.Queue(), ctx.Queue()
    p = ctx.Process(target=_empty_rank, args=(wk, q_handle, q_peer, q_done))
    p.start()
    try:
        w = synth.Workload(**wk)
        hist = synth.NumpyHistory(w)
        r = kvmret.Retriever(config_for(w))
        append_history(r, hist, cuts=[])
        h0 = r.exchange_export(2)
        h1 = q_handle.get(timeout=300)
        q_peer.put(h0)
        r.exchange_import(0, [h0, h1])
        # rank 1 scores first and gives up waiting for rank 0 (bounded, 2 s)
        assert "0x100" in q_done.get(timeout=300)
        q = hist.queries(1)[0]
        r.query_reset()
        r.query_add(torch.from_numpy(q.reshape(w.n_layer, 1, -1)).cuda())
        t0 = time.monotonic()
        r.score_exchange()
        r.select_apply_async()
        ids, _ = r.step_collect()
        assert time.monotonic() - t0 < 1.5  # rank 1's flag was already there
        want, _ = oracle_scores(hist, q.reshape(w.n_layer, -1).astype(np.float32),
                                np.ones(w.n_layer, np.uint32))
        assert list(ids) == list(po.pick_topk(want, w.budget_blocks, w.sink_blocks))
        r.close()
    finally:
        q_peer.put(1)
        p.join(timeout=120)
    assert p.exitcode == 0
