"""kvmret_clear_working_set (KvMemStore::clear_working_set,
kvmem/src/host/kvmem_store.cpp:897-901) on the GPU context:

- after a clear that keeps the pool, the next selection is rebuilt entirely
  from the HBM pool (no host reads) and the window equals the oracle's;
- after a clear that drops the pool, the whole selection is staged from the
  host repository, as on a fresh context;
- the same start state (clear + the same selection) and the same queries
  replay the same selections and the same per-step work, pool cache on.
"""
import numpy as np
import pytest
import torch

import kvmret
import pyoracle as po
from kvm_helpers import append_history, config_for, f16_ulp_diff, history_units
from kvmret import synth

pytestmark = pytest.mark.gpu


def _workload():
    return synth.Workload("ws", n_layer=2, n_head=8, n_head_kv=2, d_head=128, block_tokens=64,
                          n_blocks=40, budget_blocks=8, sink_blocks=1, reserve_blocks=2,
                          n_planted=3, seed=91)


def _check_window(r, hist):
    w = hist.w
    k, v = history_units(hist)  # [N][L][T][E] f16 bits
    lay, bases = r.window_layout()
    T = w.block_tokens
    for l in range(w.n_layer):
        wk = r.window_read(l, False, 0, len(lay)).view(np.uint16).reshape(
            len(lay), T, w.n_head_kv, w.d_head)
        wv = r.window_read(l, True, 0, len(lay)).view(np.uint16).reshape(len(lay), T, -1)
        for j, (b, base) in enumerate(zip(lay, bases)):
            want = po.rope_block_f16(k[b, l].view(np.uint16).reshape(T, w.n_head_kv, w.d_head),
                                     int(base), w.freq_base)
            assert f16_ulp_diff(wk[j], want).max() <= 2
            assert np.array_equal(wv[j], v[b, l].view(np.uint16))


def test_clear_keeps_or_drops_the_pool():
    w = _workload()
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w, pool_cache=1))
    append_history(r, hist, cuts=[])
    ids1 = [0, 3, 5, 7, 9, 11, 13, 15]
    ids2 = [0, 3, 6, 8, 10, 12, 14, 16]
    st = r.apply(ids1)
    assert st["n_h2d_blocks"] == 8
    st = r.apply(ids2)
    assert st["n_h2d_blocks"] == 6  # 0 and 3 stay pooled
    _check_window(r, hist)

    r.clear_working_set(drop_pool=False)
    st = r.apply(ids2)
    assert st["n_h2d_blocks"] == 0 and st["n_moved"] == 8
    assert st["n_stage_in"] == 8  # the host table: every block enters the working set
    assert list(r.window_layout()[0]) == ids2
    _check_window(r, hist)

    r.clear_working_set(drop_pool=True)
    st = r.apply(ids1)
    assert st["n_h2d_blocks"] == 8 and st["n_moved"] == 0
    assert list(r.window_layout()[0]) == ids1
    _check_window(r, hist)
    r.close()


def test_same_start_state_replays_the_same_steps():
    w = _workload()
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w, pool_cache=1))
    append_history(r, hist, cuts=[])
    rng = np.random.default_rng(3)
    qs = [(hist.q0 + 0.6 * rng.standard_normal(hist.q0.shape)).astype(np.float16)
          for _ in range(6)]
    start = [0, 2, 4, 6, 8, 10, 12, 14]

    def run():
        r.clear_working_set(drop_pool=True)
        r.apply(start)
        out = []
        for q in qs:
            r.query_reset()
            r.query_add(torch.from_numpy(q.reshape(w.n_layer, 1, -1)).cuda())
            r.score()
            r.select_apply_async()
            ids, st = r.step_collect()
            out.append((ids.tolist(), st["n_h2d_blocks"], st["n_moved"]))
        return out

    a = run()
    b = run()
    assert a == b
    assert sum(x[1] for x in a) > 0  # the queries did change the selection
    _check_window(r, hist)
    r.close()


def test_clear_with_steps_in_flight_collects_them_first():
    w = _workload()
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w))
    append_history(r, hist, cuts=[])
    r.query_reset()
    r.query_add(torch.from_numpy(hist.q0.reshape(w.n_layer, 1, -1)).cuda())
    r.score()
    r.select_apply_async()
    r.select_apply_async()
    r.clear_working_set(drop_pool=True)  # drains both readbacks
    with pytest.raises(kvmret.KvmretError):
        r.step_collect()  # nothing left to collect
    st = r.apply([0, 1, 2])
    assert st["n_h2d_blocks"] == 3
    _check_window(r, hist)
    r.close()


@pytest.mark.parametrize("pool_cache", [0, 1])
def test_full_pool_frees_before_it_allocates(pool_cache):
    """Every release precedes the new allocations (the ordering invariant of
    kvmem/tests/kvmem_runtime_test.cpp:51-80): with a pool exactly as large as
    the selection, a disjoint selection fits only if the departing blocks'
    slots are released first."""
    w = synth.Workload("fp", n_layer=2, n_head=8, n_head_kv=2, d_head=128, block_tokens=64,
                       n_blocks=24, budget_blocks=6, sink_blocks=1, reserve_blocks=0,
                       n_planted=1, seed=13)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w, pool_cache=pool_cache, pool_blocks=6))
    append_history(r, hist, cuts=[])
    a, b = [1, 3, 5, 7, 9, 11], [0, 2, 4, 6, 8, 10]
    assert r.apply(a)["n_h2d_blocks"] == 6
    st = r.apply(b)
    assert st["n_h2d_blocks"] == 6 and st["n_stage_out"] == 6
    assert list(r.window_layout()[0]) == b
    _check_window(r, hist)
    st = r.apply(a)  # b's blocks took every slot: a is staged again from the host
    assert st["n_h2d_blocks"] == 6
    assert list(r.window_layout()[0]) == a
    _check_window(r, hist)
    r.close()
