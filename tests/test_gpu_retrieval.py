"""GPU parity of the full retrieval step on BASELINE config 1 (2 layers,
32 q / 8 kv heads, 256 blocks of 128 f16 tokens, budget 32, sink 1,
gen-reserve 8 slots) against the CPU oracle, through the C ABI.

Bars: summaries and selected ids bit-exact, scores within 1e-3 relative (the
scorer reproduces the reference's float/double order, so they are expected to
be bit-exact too), plan rows bit-exact, window K within 2 f16 ulps of the
oracle's RoPE at the window base, window V bytes exact.
"""
import numpy as np
import pytest
import torch

import kvmret
import pyoracle as po
from kvm_helpers import (append_history, config_for, f16_ulp_diff, history_units,
                         oracle_scores)
from kvmret import synth

pytestmark = pytest.mark.gpu

W1 = synth.CONFIGS[1]


@pytest.fixture(scope="module")
def hist1():
    return synth.NumpyHistory(W1)


@pytest.fixture(scope="module")
def ctx1(hist1):
    r = kvmret.Retriever(config_for(W1))
    # ragged chunks: partial blocks are continued across appends
    append_history(r, hist1, cuts=[1, 200, 5000, 5001, 20000])
    yield r
    r.close()


def test_summaries_bit_exact(ctx1, hist1):
    got = ctx1.summaries()
    k, _ = history_units(hist1)
    w = W1
    want = po.mean_k(k.reshape(w.n_blocks * w.n_layer, w.block_tokens, w.E)).reshape(
        w.n_blocks, w.n_layer, w.E)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_repository_bytes(ctx1, hist1):
    w = W1
    repo = ctx1.repo_view()
    unit = int(kvmret.lib.kvmret_repo_unit_bytes(ctx1.h))
    kpart = int(kvmret.lib.kvmret_repo_k_bytes(ctx1.h))
    k, v = history_units(hist1)
    for b in (0, 1, 77, w.n_blocks - 1):
        for l in range(w.n_layer):
            u = repo[(b * w.n_layer + l) * unit:(b * w.n_layer + l + 1) * unit]
            kb = k[b, l].reshape(-1).view(np.uint8)
            vb = v[b, l].reshape(-1).view(np.uint8)
            assert np.array_equal(u[:kb.size], kb)
            assert np.array_equal(u[kpart:kpart + vb.size], vb)


def _step_and_check(r, hist, q, store, tie_higher=True):
    w = hist.w
    r.query_reset()
    r.query_add(torch.from_numpy(q.reshape(w.n_layer, 1, -1)).cuda())
    got_scores = r.score()
    q_sum = q.reshape(w.n_layer, -1).astype(np.float32)
    q_count = np.ones(w.n_layer, np.uint32)
    want_scores, _ = oracle_scores(hist, q_sum, q_count)
    rel = np.abs(got_scores - want_scores) / np.maximum(np.abs(want_scores), 1e-30)
    assert rel.max() <= 1e-3
    n_exact = int(np.sum(got_scores.view(np.uint64) == want_scores.view(np.uint64)))
    ids = r.select()
    want_ids = po.pick_topk(want_scores, w.budget_blocks, w.sink_blocks, 0, (), tie_higher)
    assert list(ids) == list(want_ids)
    stats = r.apply(ids)
    plan = r.last_plan()
    si, so, rm, c = store.set_selection(ids)
    assert np.array_equal(plan.remaps, rm)
    assert np.array_equal(plan.stage_in, si) and np.array_equal(plan.stage_out, so)
    lay_ids, lay_bases = r.window_layout()
    assert list(lay_ids) == list(rm[:, 0]) and list(lay_bases) == list(rm[:, 3])
    return stats, n_exact


def _check_window(r, hist, layers=None):
    w = hist.w
    k, v = history_units(hist)
    ids, bases = r.window_layout()
    worst = 0
    for l in (range(w.n_layer) if layers is None else layers):
        wk = r.window_read(l, False, 0, len(ids)).view(np.uint16).reshape(
            len(ids), w.block_tokens, w.n_head_kv, w.d_head)
        wv = r.window_read(l, True, 0, len(ids)).view(np.uint16).reshape(
            len(ids), w.block_tokens, w.n_head_kv, w.d_head)
        for i, (b, base) in enumerate(zip(ids, bases)):
            src = k[b, l].view(np.uint16).reshape(w.block_tokens, w.n_head_kv, w.d_head)
            want = po.rope_block_f16(src, int(base), w.freq_base)
            d = f16_ulp_diff(wk[i], want)
            worst = max(worst, int(d.max()))
            assert np.array_equal(wv[i], v[b, l].view(np.uint16).reshape(wv[i].shape))
    assert worst <= 2
    return worst


def test_retrieval_steps_match_oracle(ctx1, hist1):
    w = W1
    qs = hist1.queries(6)
    store = po.Store(w.block_tokens)
    store.append(w.n_tokens)
    exact = 0
    for s in range(len(qs)):
        stats, n_exact = _step_and_check(ctx1, hist1, qs[s], store)
        exact += n_exact
        assert stats["n_selected"] == w.budget_blocks
        if s == 0:
            assert stats["n_h2d_blocks"] == w.budget_blocks
        _check_window(ctx1, hist1)
    # the planted blocks dominate the selection
    ids, _ = ctx1.window_layout()
    assert set(hist1.planted.tolist()) <= set(ids.tolist())
    # every score reproduced bit for bit
    assert exact == len(qs) * w.n_blocks


def test_apply_retrieval_entry_point(hist1):
    w = W1
    r = kvmret.Retriever(config_for(w, pool_cache=1))
    append_history(r, hist1, cuts=[])
    q = hist1.queries(2)
    for s in range(2):
        r.query_reset()
        r.query_add(torch.from_numpy(q[s].reshape(w.n_layer, 1, -1)).cuda())
        ids, stats = r.apply_retrieval(mandatory=[w.n_blocks - 1])
        assert w.n_blocks - 1 in ids.tolist()
        assert len(ids) == w.budget_blocks
    _check_window(r, hist1, layers=[1])
    r.close()


@pytest.mark.parametrize("pool_cache", [0, 1])
def test_async_step_matches_preview_apply(hist1, pool_cache):
    """score -> select_apply_async with the collect lagging one step behind (the
    bench's loop) gives the same selections and byte-identical windows as
    preview -> apply_selection."""
    w = W1
    a = kvmret.Retriever(config_for(w, pool_cache=pool_cache))
    b = kvmret.Retriever(config_for(w, pool_cache=pool_cache))
    append_history(a, hist1, cuts=[3000])
    append_history(b, hist1, cuts=[])
    qs = hist1.queries(8)
    got_b = []
    for s in range(len(qs)):
        q = torch.from_numpy(qs[s].reshape(w.n_layer, 1, -1)).cuda()
        a.query_reset()
        a.query_add(q)
        ids_a = a.preview()
        a.apply(ids_a)
        b.query_reset()
        b.query_add(q)
        b.score_layers()
        kvmret._check(kvmret.lib.kvmret_score_reduce(b.h, kvmret.lib.kvmret_contrib_dev(b.h),
                                                      w.n_layer))
        b.select_apply_async()
        if s > 0:
            got_b.append(b.step_collect()[0])
        got_a = ids_a
        if s > 0:
            assert list(got_b[-1]) == list(prev_a)
        prev_a = got_a
    got_b.append(b.step_collect()[0])
    assert list(got_b[-1]) == list(prev_a)
    la, ba = a.window_layout()
    lb, bb = b.window_layout()
    assert np.array_equal(la, lb) and np.array_equal(ba, bb)
    for l in range(w.n_layer):
        for is_v in (False, True):
            assert np.array_equal(a.window_read(l, is_v, 0, len(la)),
                                  b.window_read(l, is_v, 0, len(lb)))
    assert np.array_equal(a.last_plan().remaps, b.last_plan().remaps)
    a.close()
    b.close()
