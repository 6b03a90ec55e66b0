"""HBM-resident history (kvmret_pool_prefetch), on the GPU through the C ABI,
against the CPU oracle:

- with a pool that holds the whole history, every block is placed; the
  GPU-resident steps that follow copy nothing from the host, and each window
  matches the oracle's selection, layout and bytes (f16 and q8_0 K);
- with a smaller pool, prefetch fills the free slots and stops; the steps
  evict the prefetched blocks first (they count as least recently used) and
  stay correct;
- a block that grows after it was prefetched is restaged from the host;
- without pool caching the call fails and changes nothing.
"""
import numpy as np
import pytest
import torch

import kvmret
from kvm_helpers import append_history, check_window, config_for, oracle_ids_tokens
from kvmret import synth

pytestmark = pytest.mark.gpu


def _w(**kw):
    base = dict(name="pf", n_layer=2, n_head=8, n_head_kv=2, d_head=128, block_tokens=32,
                n_blocks=40, budget_blocks=6, sink_blocks=1, reserve_blocks=2, n_planted=4,
                seed=91)
    base.update(kw)
    return synth.Workload(**base)


def _q8(x):
    return kvmret.quantize_f16(torch.from_numpy(np.ascontiguousarray(x)).cuda(),
                               kvmret.TYPE_Q8_0).cpu().numpy()


def _q4(x):
    return kvmret.quantize_f16(torch.from_numpy(np.ascontiguousarray(x)).cuda(),
                               kvmret.TYPE_Q4_0).cpu().numpy()


def _steps(r, hist, n_tok, qs, quant):
    stats = []
    for q in qs:
        r.query_reset()
        r.query_add(torch.from_numpy(q.reshape(hist.w.n_layer, 1, -1)).cuda())
        r.score()
        r.select_apply_async()
        ids, st = r.step_collect()
        assert list(ids) == oracle_ids_tokens(hist, n_tok, q)
        check_window(r, hist, n_tok, list(ids), quant=quant)
        stats.append(st)
    return stats


@pytest.mark.parametrize("quant", [False, True])
def test_whole_history_in_the_pool_reads_nothing_from_the_host(quant):
    w = _w(k_type=kvmret.TYPE_Q8_0, v_type=kvmret.TYPE_Q4_0) if quant else _w()
    hist = synth.NumpyHistory(w)
    cfg = config_for(w, pool_cache=1, pool_blocks=w.n_blocks + w.reserve_blocks)
    r = kvmret.Retriever(cfg)
    append_history(r, hist, cuts=[333], k_rows_fn=_q8 if quant else None,
                   v_rows_fn=_q4 if quant else None)
    assert r.pool_prefetch() == w.n_blocks
    assert r.pool_prefetch() == 0  # every block already holds a slot
    stats = _steps(r, hist, w.n_tokens, hist.queries(5), quant)
    assert all(st["n_h2d_blocks"] == 0 for st in stats)
    r.close()


def test_small_pool_fills_and_evicts_prefetched_blocks_first():
    w = _w()
    hist = synth.NumpyHistory(w)
    P = w.budget_blocks + w.reserve_blocks + 10
    r = kvmret.Retriever(config_for(w, pool_cache=1, pool_blocks=P))
    append_history(r, hist, cuts=[])
    assert r.pool_prefetch(3, 1000) == P  # blocks 3 .. 3 + P - 1
    qs = hist.queries(4)
    stats = _steps(r, hist, w.n_tokens, qs, False)
    # the first window's blocks in 3 .. 3 + P - 1 came from the pool, the
    # others from the host
    ids0 = oracle_ids_tokens(hist, w.n_tokens, qs[0])
    assert stats[0]["n_h2d_blocks"] == sum(1 for b in ids0 if not 3 <= b < 3 + P)
    r.close()


def test_block_grown_after_prefetch_is_restaged():
    w = _w()
    hist = synth.NumpyHistory(w)
    T = w.block_tokens
    n0 = w.n_tokens - T // 2  # the newest block is half full
    r = kvmret.Retriever(config_for(w, pool_cache=1, pool_blocks=w.n_blocks + w.reserve_blocks))
    append_history(r, hist, cuts=[], stop=n0)
    assert r.pool_prefetch() == w.n_blocks
    append_history(r, hist, cuts=[], start=n0)  # fills it
    q = hist.queries(1)[0]
    r.query_reset()
    r.query_add(torch.from_numpy(q.reshape(w.n_layer, 1, -1)).cuda())
    ids = r.preview([w.n_blocks - 1])
    st = r.apply(ids)
    assert st["n_h2d_blocks"] == 1  # only the grown block
    check_window(r, hist, w.n_tokens, list(ids))
    r.close()


def test_prefetch_needs_pool_caching():
    w = _w()
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w, pool_cache=0))
    append_history(r, hist, cuts=[])
    with pytest.raises(kvmret.KvmretError):
        r.pool_prefetch()
    r.close()
