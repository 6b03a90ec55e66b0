"""Conversation stores (llama_kvmem_store_create / _switch, the reference's
swap_conv, src/adapter/llama-memory-kvmem.cpp:1624-1714) on the GPU through
the C ABI: two conversations with different histories take turns on one
context's window and HBM pool. After every swap the incoming conversation's
working set is back in the window (same blocks, same bases, K within 2 f16
ulp of the oracle, V exact) and its next steps select the oracle's blocks; a
new store starts empty; a parked store keeps its rows."""
import numpy as np
import pytest
import torch

import kvmret
from kvm_helpers import append_history, check_window, config_for, oracle_ids_tokens
from kvmret import synth

pytestmark = pytest.mark.gpu


def _w(**kw):
    base = dict(name="conv", n_layer=2, n_head=8, n_head_kv=2, d_head=128, block_tokens=32,
                n_blocks=24, budget_blocks=5, sink_blocks=1, reserve_blocks=2, n_planted=3,
                seed=81)
    base.update(kw)
    return synth.Workload(**base)


@pytest.mark.parametrize("quant", [False, True])
def test_two_conversations_take_turns_on_one_window(quant):
    kw = dict(k_type=kvmret.TYPE_Q8_0, v_type=kvmret.TYPE_Q4_0) if quant else {}
    wa, wb = _w(**kw), _w(seed=82, **kw)
    ha, hb = synth.NumpyHistory(wa), synth.NumpyHistory(wb)
    T = wa.block_tokens
    na, nb = 24 * T - 9, 17 * T + 5
    r = kvmret.Retriever(config_for(wa))
    kwa = {}
    if quant:
        import pyoracle as po
        kwa = dict(k_rows_fn=lambda k: po.quant_q8_0(k.astype(np.float32)).reshape(
            k.shape[0], k.shape[1], -1),
            v_rows_fn=lambda v: po.quant_q4_0(v.astype(np.float32)).reshape(
                v.shape[0], v.shape[1], -1))
    append_history(r, ha, cuts=[300], stop=na, **kwa)
    qa, qb = ha.queries(3), hb.queries(3)

    def step(hist, q, n):
        w = hist.w
        r.query_reset()
        r.query_add(torch.from_numpy(q.reshape(w.n_layer, 1, -1)).cuda())
        r.score()
        r.select_apply_async()
        ids, _ = r.step_collect()
        want = oracle_ids_tokens(hist, n, q)
        assert list(ids) == want
        check_window(r, hist, n, want, quant=quant)
        return want

    sel_a = step(ha, qa[0], na)
    store = r.store_create()
    assert store.rows == 0 and store.host_bytes > 0
    assert r.store_swap(store) is False  # the new conversation is empty
    assert store.rows == na and r.n_tokens == 0
    assert len(r.window_layout()[0]) == 0
    append_history(r, hb, cuts=[100], stop=nb, **kwa)
    sel_b = step(hb, qb[0], nb)
    for turn in range(2):
        # A comes back: its working set is rebuilt, then it steps on
        assert r.store_swap(store) is True
        assert r.n_tokens == na and store.rows == nb
        check_window(r, ha, na, sel_a, quant=quant)
        sel_a = step(ha, qa[1 + turn], na)
        # and B again
        assert r.store_swap(store) is True
        assert r.n_tokens == nb and store.rows == na
        check_window(r, hb, nb, sel_b, quant=quant)
        sel_b = step(hb, qb[1 + turn], nb)
    store.close()
    r.close()


def test_store_appends_continue_after_swaps():
    """Appends to a swapped-in conversation continue its partial block's
    running sum: its summaries stay the oracle's token-order means."""
    wa, wb = _w(seed=83), _w(seed=84)
    ha, hb = synth.NumpyHistory(wa), synth.NumpyHistory(wb)
    T = wa.block_tokens
    r = kvmret.Retriever(config_for(wa))
    append_history(r, ha, cuts=[], stop=10 * T + 7)
    store = r.store_create()
    r.store_swap(store)
    append_history(r, hb, cuts=[], stop=6 * T + 30)
    r.store_swap(store)  # A again
    append_history(r, ha, cuts=[], start=10 * T + 7, stop=12 * T + 3)
    from kvm_helpers import oracle_mean_tokens
    got = r.summaries()
    assert np.array_equal(got.view(np.uint32), oracle_mean_tokens(ha, 12 * T + 3).view(np.uint32))
    r.store_swap(store)  # B again
    append_history(r, hb, cuts=[], start=6 * T + 30, stop=8 * T)
    got = r.summaries()
    assert np.array_equal(got.view(np.uint32), oracle_mean_tokens(hb, 8 * T).view(np.uint32))
    store.close()
    r.close()
