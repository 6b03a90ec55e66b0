"""Gen-reserve placement of decode blocks (the adapter's prepare_working_set
after a retrieval, src/adapter/llama-memory-kvmem.cpp:2314-2365; alloc_slot
:1720-1741; kvmem_fill_slot_info, src/adapter/llama-kvmem-batch.cpp:5-58),
truncation (KvMemRuntime::truncate_to) and the stream order of the host block
table, on the GPU through the C ABI, against the CPU oracle:

- decoding token by token across block boundaries in gen mode: every token
  has a cache cell at once; the window holds every selected block and every
  decode block, chronologically, K rotated at its window base (within 2 f16
  ulp / 1 q8_0 LSB of the oracle), V exact; later steps keep the decode
  blocks beyond the budget and select the oracle's top-k over the others;
- a decode block that needs a slot when none is free fails cleanly and
  changes nothing;
- truncation into a partial block rebuilds its summary bit-exactly;
- an append made while a step is in flight reaches the host table's plan
  after that step's selection, as in the reference's call order.
"""
import numpy as np
import pytest
import torch

import kvmret
import pyoracle as po
from kvm_helpers import append_history, check_window as _check_window, config_for
from kvm_helpers import oracle_ids_tokens as _oracle_ids, oracle_mean_tokens as _oracle_mean
from kvmret import synth

pytestmark = pytest.mark.gpu


def _w(**kw):
    base = dict(name="gen", n_layer=2, n_head=8, n_head_kv=2, d_head=128, block_tokens=32,
                n_blocks=24, budget_blocks=5, sink_blocks=1, reserve_blocks=3, n_planted=3,
                seed=71)
    base.update(kw)
    return synth.Workload(**base)


def _append_tokens(r, hist, t0, t1, quant=False):
    w = hist.w
    L, E = w.n_layer, w.E
    k = torch.from_numpy(np.ascontiguousarray(hist.k.reshape(L, w.n_tokens, E)[:, t0:t1])).cuda()
    v = torch.from_numpy(np.ascontiguousarray(hist.v.reshape(L, w.n_tokens, E)[:, t0:t1])).cuda()
    if quant:
        r.append(k, kvmret.quantize_f16(v, w.v_type), k_rows=kvmret.quantize_f16(k, w.k_type),
                 pos0=t0)
    else:
        r.append(k, v, pos0=t0)


@pytest.mark.parametrize("selected_before", [True, False])
def test_decode_across_block_boundaries_in_reserve_slots(selected_before):
    w = _w()
    hist = synth.NumpyHistory(w)
    T = w.block_tokens
    n0 = 20 * T - 7  # block 19 holds 25 tokens
    r = kvmret.Retriever(config_for(w))
    append_history(r, hist, cuts=[300], stop=n0)
    q = hist.queries(6)
    r.query_reset()
    r.query_add(torch.from_numpy(q[0].reshape(w.n_layer, 1, -1)).cuda())
    mand = [19] if selected_before else []
    ids = r.preview(mand)
    assert (19 in ids) == selected_before
    r.apply(ids)
    s1 = list(ids)
    r.gen_begin()
    assert r.gen_first_block == 19
    n_tok, step = n0, 1
    for t in range(n0, n0 + 50):  # fills block 19, all of block 20, starts block 21
        _append_tokens(r, hist, t, t + 1)
        n_tok = t + 1
        cell = int(r.cells(t, 1)[0])
        lay, _ = r.window_layout()
        b = t // T
        assert cell == list(lay).index(b) * T + (t - b * T)
        if t % 12 == 0:  # a retrieval step: decode blocks pinned beyond the budget
            r.query_reset()
            r.query_add(torch.from_numpy(q[step].reshape(w.n_layer, 1, -1)).cuda())
            r.score()
            r.select_apply_async()
            got, _ = r.step_collect()
            want = _oracle_ids(hist, n_tok, q[step], gen_first=19)
            assert list(got) == want
            s1 = [x for x in want if x < 19]
            step += 1
        if t % 7 == 0 or t == n0 + 49:
            gen = list(range(19, n_tok // T + (1 if n_tok % T else 0)))
            _check_window(r, hist, n_tok, sorted(set(s1) | set(gen)))
    r.gen_end()
    # after the turn the decode blocks are ordinary candidates again
    r.query_reset()
    r.query_add(torch.from_numpy(q[step].reshape(w.n_layer, 1, -1)).cuda())
    ids, _ = r.apply_retrieval()
    want = _oracle_ids(hist, n_tok, q[step])
    assert list(ids) == want
    _check_window(r, hist, n_tok, want)
    r.close()


def test_decode_blocks_quantised_k():
    w = _w(k_type=kvmret.TYPE_Q8_0, v_type=kvmret.TYPE_Q4_0, seed=72)
    hist = synth.NumpyHistory(w)
    T = w.block_tokens
    n0 = 20 * T - 5
    r = kvmret.Retriever(config_for(w))
    qk = lambda k: po.quant_q8_0(k.astype(np.float32)).reshape(k.shape[0], k.shape[1], -1)  # noqa: E731
    qv = lambda v: po.quant_q4_0(v.astype(np.float32)).reshape(v.shape[0], v.shape[1], -1)  # noqa: E731
    append_history(r, hist, cuts=[400], stop=n0, k_rows_fn=qk, v_rows_fn=qv)
    q = hist.queries(3)
    r.query_reset()
    r.query_add(torch.from_numpy(q[0].reshape(w.n_layer, 1, -1)).cuda())
    s1 = list(r.preview())
    r.apply(s1)
    r.gen_begin()
    n_tok = n0
    for t in range(n0, n0 + 40):
        _append_tokens(r, hist, t, t + 1, quant=True)
        n_tok = t + 1
        if t in (n0, n0 + 4, n0 + 5, n0 + 39):
            gen = list(range(19, (n_tok + T - 1) // T))
            _check_window(r, hist, n_tok, sorted(set(s1) - set(gen) | set(gen)), quant=True)
    r.query_reset()
    r.query_add(torch.from_numpy(q[1].reshape(w.n_layer, 1, -1)).cuda())
    r.score()
    r.select_apply_async()
    got, _ = r.step_collect()
    assert list(got) == _oracle_ids(hist, n_tok, q[1], gen_first=19)
    _check_window(r, hist, n_tok, list(got), quant=True)
    r.gen_end()
    r.close()


def test_no_free_reserve_slot_fails_cleanly():
    w = _w(reserve_blocks=1, seed=73)
    hist = synth.NumpyHistory(w)
    T = w.block_tokens
    n0 = 20 * T - 3
    r = kvmret.Retriever(config_for(w))
    append_history(r, hist, cuts=[], stop=n0)
    r.apply([0, 3, 5, 7, 9])  # the budget's five blocks; block 19 outside the window
    r.gen_begin()
    _append_tokens(r, hist, n0, n0 + 3)  # block 19 takes the one reserve slot
    lay0, bases0 = r.window_layout()
    with pytest.raises(kvmret.KvmretError, match="no free GPU slot for block 20"):
        _append_tokens(r, hist, n0 + 3, n0 + 4)  # block 20 finds none
    assert r.n_tokens == n0 + 3
    lay1, bases1 = r.window_layout()
    assert np.array_equal(lay0, lay1) and np.array_equal(bases0, bases1)
    _check_window(r, hist, n0 + 3, list(lay0))
    r.gen_end()
    _append_tokens(r, hist, n0 + 3, n0 + 4)  # outside gen mode the append goes through
    assert r.n_tokens == n0 + 4
    r.close()


def test_truncate_rebuilds_partial_block_summary():
    w = _w(seed=74)
    hist = synth.NumpyHistory(w)
    T = w.block_tokens
    r = kvmret.Retriever(config_for(w))
    append_history(r, hist, cuts=[200], stop=20 * T - 7)
    q = hist.queries(2)
    r.query_reset()
    r.query_add(torch.from_numpy(q[0].reshape(w.n_layer, 1, -1)).cuda())
    r.apply(r.preview([19]))
    r.truncate(18 * T + 24)  # block 18 keeps 24 tokens, block 19 leaves
    assert r.n_tokens == 18 * T + 24 and r.n_blocks == 19
    got = r.summaries()
    want = _oracle_mean(hist, 18 * T + 24)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert all(b < 19 for b in r.window_layout()[0])
    # appending again continues the partial block's running sum
    _append_tokens(r, hist, 18 * T + 24, 21 * T + 5)
    got = r.summaries()
    want = _oracle_mean(hist, 21 * T + 5)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    r.query_reset()
    r.query_add(torch.from_numpy(q[1].reshape(w.n_layer, 1, -1)).cuda())
    ids, _ = r.apply_retrieval()
    want_ids = _oracle_ids(hist, 21 * T + 5, q[1])
    assert list(ids) == want_ids
    _check_window(r, hist, 21 * T + 5, want_ids)
    r.close()


def test_truncate_quantised_k_block_boundaries_only():
    w = _w(k_type=kvmret.TYPE_Q8_0, v_type=kvmret.TYPE_Q4_0, seed=75)
    hist = synth.NumpyHistory(w)
    T = w.block_tokens
    r = kvmret.Retriever(config_for(w))
    qk = lambda k: po.quant_q8_0(k.astype(np.float32)).reshape(k.shape[0], k.shape[1], -1)  # noqa: E731
    qv = lambda v: po.quant_q4_0(v.astype(np.float32)).reshape(v.shape[0], v.shape[1], -1)  # noqa: E731
    append_history(r, hist, cuts=[], stop=10 * T, k_rows_fn=qk, v_rows_fn=qv)
    with pytest.raises(kvmret.KvmretError, match="block boundary"):
        r.truncate(9 * T + 3)
    r.truncate(8 * T)
    assert r.n_blocks == 8
    got = r.summaries()
    assert np.array_equal(got.view(np.uint32), _oracle_mean(hist, 8 * T).view(np.uint32))
    r.close()


def test_append_while_step_in_flight_replays_in_call_order():
    """A step is enqueued, then tokens are appended (a new block), then the
    step is collected: its plan is the oracle's set_selection before the
    append; the next step's plan includes the new block."""
    w = _w(seed=76)
    hist = synth.NumpyHistory(w)
    T = w.block_tokens
    r = kvmret.Retriever(config_for(w))
    append_history(r, hist, cuts=[], stop=18 * T)
    store = po.Store(T)
    store.append(18 * T)
    q = hist.queries(2)
    r.query_reset()
    r.query_add(torch.from_numpy(q[0].reshape(w.n_layer, 1, -1)).cuda())
    r.score()
    r.select_apply_async()
    _append_tokens(r, hist, 18 * T, 19 * T + 9)  # while the step is in flight
    ids, _ = r.step_collect()
    want = _oracle_ids(hist, 18 * T, q[0])
    assert list(ids) == want
    si, so, rm, _ = store.set_selection(want)
    p = r.last_plan()
    assert np.array_equal(p.remaps, rm) and np.array_equal(p.stage_in, si)
    store.append(T + 9)
    r.query_reset()
    r.query_add(torch.from_numpy(q[1].reshape(w.n_layer, 1, -1)).cuda())
    ids, _ = r.apply_retrieval()
    want = _oracle_ids(hist, 19 * T + 9, q[1])
    assert list(ids) == want
    si, so, rm, _ = store.set_selection(want)
    p = r.last_plan()
    assert np.array_equal(p.remaps, rm) and np.array_equal(p.stage_out, so)
    _check_window(r, hist, 19 * T + 9, want)
    r.close()
