"""Edge cases of the retrieval step the reference's own tests cover for the
selection (kvmem_store_test: empty store, everything fits), run through the
GPU context:

- no history at all: every entry point selects nothing and leaves the window
  empty;
- fewer blocks than the budget: every block is selected, in order, and the
  window holds them at consecutive bases;
- more blocks than the selector stages in shared memory (16,384): the radix
  selection reading the scores from global memory picks exactly the oracle's
  top-k.
"""
import numpy as np
import pytest
import torch

import kvmret
import pyoracle as po
from kvm_helpers import append_history, config_for, f16_ulp_diff, oracle_scores
from kvmret import synth

pytestmark = pytest.mark.gpu


def _query(w, seed=0):
    q = np.random.default_rng(seed).standard_normal((w.n_layer, 1, w.n_head * w.d_head))
    return torch.from_numpy(q.astype(np.float16)).cuda()


def test_empty_history_selects_nothing():
    w = synth.Workload("e0", n_layer=2, n_head=8, n_head_kv=2, d_head=128, block_tokens=64,
                       n_blocks=8, budget_blocks=4, sink_blocks=1, reserve_blocks=1,
                       n_planted=0, seed=3)
    r = kvmret.Retriever(config_for(w))
    r.query_reset()
    r.query_add(_query(w))
    assert len(r.score()) == 0
    assert len(r.select()) == 0
    st = r.apply([])
    assert st["n_selected"] == 0 and st["n_h2d_blocks"] == 0
    r.select_apply_async()
    ids, st = r.step_collect()
    assert len(ids) == 0 and st["n_selected"] == 0
    lay, _ = r.window_layout()
    assert len(lay) == 0
    r.close()


def test_fewer_blocks_than_budget_selects_all():
    w = synth.Workload("e1", n_layer=2, n_head=8, n_head_kv=2, d_head=128, block_tokens=64,
                       n_blocks=5, budget_blocks=8, sink_blocks=1, reserve_blocks=0,
                       n_planted=1, seed=5)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w))
    append_history(r, hist, cuts=[130])
    r.query_reset()
    r.query_add(_query(w, 1))
    r.score()
    ids = r.select()
    assert list(ids) == [0, 1, 2, 3, 4]
    st = r.apply(ids)
    assert st["n_selected"] == 5
    lay, bases = r.window_layout()
    assert list(lay) == [0, 1, 2, 3, 4]
    assert list(bases) == [64 * i for i in range(5)]
    T, L, E = w.block_tokens, w.n_layer, w.E
    k = hist.k.reshape(L, -1, E)
    for l in range(L):
        wk = r.window_read(l, False, 0, 5).view(np.uint16).reshape(5 * T, w.n_head_kv, w.d_head)
        want = po.rope_block_f16(k[l, :5 * T].view(np.uint16).reshape(
            5 * T, w.n_head_kv, w.d_head), 0, w.freq_base)
        assert f16_ulp_diff(wk, want).max() <= 2
    r.close()


def test_block_count_beyond_the_shared_memory_selector():
    n_blocks = 20000  # beyond the 16,384 blocks staged in shared memory
    w = synth.Workload("e2", n_layer=1, n_head=2, n_head_kv=1, d_head=64, block_tokens=16,
                       n_blocks=n_blocks, budget_blocks=64, sink_blocks=1, reserve_blocks=0,
                       n_planted=6, seed=9)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w))
    append_history(r, hist, cuts=[w.n_tokens // 2])
    q = hist.queries(2)
    for s in range(2):
        r.query_reset()
        r.query_add(torch.from_numpy(q[s].reshape(w.n_layer, 1, -1)).cuda())
        got = r.score()
        want, _ = oracle_scores(hist, q[s].reshape(w.n_layer, -1).astype(np.float32),
                                np.ones(w.n_layer, np.uint32))
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64))
        ids = r.select(mandatory=[n_blocks - 1])
        assert list(ids) == list(po.pick_topk(want, w.budget_blocks, w.sink_blocks, 0,
                                              [n_blocks - 1]))
        r.select_apply_async(mandatory=[n_blocks - 1])
        ids2, _ = r.step_collect()
        assert np.array_equal(ids, ids2)
    r.close()
