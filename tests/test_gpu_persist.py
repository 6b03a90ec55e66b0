"""Persistence of a conversation on the GPU through the C ABI:

- the snapshot archive of an f16 conversation is byte-identical to the
  reference's own RawKvStore::snapshot_write of the same rows (reference
  library built from its sources), hash included;
- snapshot -> fresh context -> restore gives bit-identical summaries and
  repository rows, the same selection and window as the oracle, and appends
  continue the partial block's running sum (f16 and q8_0 / q4_0);
- repository blocks spilled to the NVMe raw tier and read back (O_DIRECT
  where the file system allows) are byte-identical, and a step staging them
  matches the oracle.
"""
import numpy as np
import pytest
import torch

import kvmret
import pyoracle as po
from kvm_helpers import (append_history, check_window, config_for, oracle_ids_tokens,
                         oracle_mean_tokens)
from kvmret import synth

pytestmark = pytest.mark.gpu


def _w(**kw):
    base = dict(name="persist", n_layer=2, n_head=8, n_head_kv=2, d_head=128, block_tokens=32,
                n_blocks=24, budget_blocks=5, sink_blocks=1, reserve_blocks=2, n_planted=3,
                seed=91)
    base.update(kw)
    return synth.Workload(**base)


def _quant_fns():
    return dict(k_rows_fn=lambda k: po.quant_q8_0(k.astype(np.float32)).reshape(
        k.shape[0], k.shape[1], -1),
        v_rows_fn=lambda v: po.quant_q4_0(v.astype(np.float32)).reshape(
            v.shape[0], v.shape[1], -1))


@pytest.mark.skipif(po.ref is None, reason="oracle/_ref not built")
def test_snapshot_bytes_equal_the_reference_writer():
    w = _w()
    h = synth.NumpyHistory(w)
    n = 20 * w.block_tokens - 7
    r = kvmret.Retriever(config_for(w))
    append_history(r, h, cuts=[100], stop=n)
    arc, hsh = r.snapshot()
    L, E = w.n_layer, w.E
    k = np.ascontiguousarray(h.k.reshape(L, w.n_tokens, E)[:, :n])
    v = np.ascontiguousarray(h.v.reshape(L, w.n_tokens, E)[:, :n])
    ref, ref_h = po.ref_snapshot_rows(L, E, w.block_tokens, 0, 2 * E,
                                      k.view(np.uint8).reshape(L, n, 2 * E),
                                      k.astype(np.float32), v.view(np.uint8).reshape(L, n, 2 * E))
    assert arc.size == ref.size and np.array_equal(arc, ref)
    assert hsh == ref_h
    r.close()


@pytest.mark.parametrize("quant", [False, True])
def test_snapshot_round_trip(quant):
    kw = dict(k_type=kvmret.TYPE_Q8_0, v_type=kvmret.TYPE_Q4_0) if quant else {}
    w = _w(seed=92, **kw)
    h = synth.NumpyHistory(w)
    T = w.block_tokens
    n = 19 * T + 11
    fns = _quant_fns() if quant else {}
    a = kvmret.Retriever(config_for(w))
    append_history(a, h, cuts=[200], stop=n, **fns)
    arc, hsh = a.snapshot()
    b = kvmret.Retriever(config_for(w))
    assert b.restore(arc) == hsh
    assert b.n_tokens == n and b.n_blocks == a.n_blocks
    sa, sb = a.summaries(), b.summaries()
    assert np.array_equal(sa.view(np.uint32), sb.view(np.uint32))
    unit = int(kvmret.lib.kvmret_repo_unit_bytes(a.h))
    kb = int(kvmret.lib.kvmret_repo_k_bytes(a.h))
    ra, rb = a.repo_view(), b.repo_view()
    for blk in range(b.n_blocks):
        nt = min(T, n - blk * T)
        for l in range(w.n_layer):
            o = (blk * w.n_layer + l) * unit
            assert np.array_equal(ra[o:o + nt * a.k_row], rb[o:o + nt * b.k_row])
            assert np.array_equal(ra[o + kb:o + kb + nt * a.v_row], rb[o + kb:o + kb + nt * b.v_row])
    q = h.queries(2)
    for r in (a, b):
        r.query_reset()
        r.query_add(torch.from_numpy(q[0].reshape(w.n_layer, 1, -1)).cuda())
        ids, _ = r.apply_retrieval()
        assert list(ids) == oracle_ids_tokens(h, n, q[0])
        check_window(r, h, n, list(ids), quant=quant)
    # the restored partial block continues its running sum
    append_history(b, h, cuts=[], start=n, stop=21 * T + 3, **fns)
    if not quant:
        got = b.summaries()
        assert np.array_equal(got.view(np.uint32), oracle_mean_tokens(h, 21 * T + 3).view(np.uint32))
    append_history(a, h, cuts=[], start=n, stop=21 * T + 3, **fns)
    assert np.array_equal(a.summaries().view(np.uint32), b.summaries().view(np.uint32))
    with pytest.raises(kvmret.KvmretError, match="empty context"):
        b.restore(arc)
    bad = arc.copy()
    bad[0] ^= 1
    c = kvmret.Retriever(config_for(w))
    with pytest.raises(kvmret.KvmretError, match="geometry"):
        c.restore(bad)
    with pytest.raises(kvmret.KvmretError, match="truncated|size"):
        c.restore(arc[:-5])
    assert c.n_tokens == 0
    for r in (a, b, c):
        r.close()


def test_repository_blocks_through_the_nvme_tier(tmp_path):
    w = _w(seed=93)
    h = synth.NumpyHistory(w)
    T = w.block_tokens
    n = 22 * T
    r = kvmret.Retriever(config_for(w))
    append_history(r, h, cuts=[], stop=n)
    slot = int(kvmret.lib.kvmret_repo_unit_bytes(r.h)) * w.n_layer
    tier = kvmret.Nvme(str(tmp_path), total_bytes=3 * slot, slot_bytes=slot, direct_read=True)
    repo = r.repo_view()
    blocks = [3, 7, 8, 9]
    before = {b: repo[b * slot:(b + 1) * slot].copy() for b in blocks}
    st = r.repo_spill(tier, blocks)  # 4 blocks into 3 slots: block 3 is evicted
    assert st["bytes"] == 4 * slot
    assert tier.block_slot(3) == -1 and tier.block_slot(9) >= 0
    for b in blocks:
        repo[b * slot:(b + 1) * slot] = 0
    with pytest.raises(kvmret.KvmretError, match="not on the NVMe tier"):
        r.repo_fill(tier, [3])
    st = r.repo_fill(tier, [7, 8, 9])
    assert st["bytes"] == 3 * slot
    for b in (7, 8, 9):
        assert np.array_equal(repo[b * slot:(b + 1) * slot], before[b])
    repo[3 * slot:4 * slot] = before[3]
    q = h.queries(1)[0]
    r.query_reset()
    r.query_add(torch.from_numpy(q.reshape(w.n_layer, 1, -1)).cuda())
    ids, _ = r.apply_retrieval(mandatory=[7, 8, 9])
    assert {7, 8, 9} <= set(ids.tolist())
    check_window(r, h, n, list(ids))
    tier.close()
    r.close()
