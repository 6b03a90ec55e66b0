"""The product's host block table (libkvmret, no GPU needed) against the
reference's libkvmem and the oracle: the always-kept part of a selection and
the plan diff (stage-in / stage-out / remaps) must be bit-identical."""
import numpy as np
import pytest

import kvmret
import pyoracle as po

needs_ref = pytest.mark.skipif(po.ref is None, reason="oracle/_ref not built")


def _table(bt, budget, sink=1, recent=0, immutable=False):
    c = kvmret.default_config(block_tokens=bt, budget_blocks=budget, sink_blocks=sink,
                              recent_blocks=recent, immutable_source_k=int(immutable))
    return kvmret.Table(c)


@pytest.mark.parametrize("seed", range(30))
def test_keep_plus_rank_fill_equals_oracle_topk(seed):
    """keep() + the score fill the GPU runs (emulated here by an exact rank) == pick_topk."""
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 400))
    budget = int(rng.integers(1, 64))
    sink = int(rng.integers(0, 3))
    recent = int(rng.integers(0, 3))
    t = _table(16, budget, sink, recent)
    t.append(n * 16)
    scores = rng.standard_normal(n)
    if seed % 2:
        scores = np.round(scores)
    mand = list(rng.integers(0, n, size=int(rng.integers(0, 5))))
    kept, kc, need = t.keep(mand)
    cand = [i for i in range(n) if not kept[i]]
    order = sorted(cand, key=lambda i: (-scores[i], -i))
    sel = sorted(set(np.nonzero(kept)[0].tolist()) | set(order[:need]))
    assert sel == list(po.pick_topk(scores, budget, sink, recent, mand, tie_higher_id=True))


@pytest.mark.parametrize("immutable", [False, True])
@pytest.mark.parametrize("seed", range(6))
def test_plan_equals_oracle(seed, immutable):
    rng = np.random.default_rng(200 + seed)
    bt = 16
    t = _table(bt, 1 << 20, immutable=immutable)
    o = po.Store(bt, immutable)
    n_tok = int(rng.integers(bt, bt * 80))
    t.append(n_tok)
    o.append(n_tok)
    for step in range(15):
        if rng.random() < 0.25:
            extra = int(rng.integers(1, 2 * bt))
            t.append(extra)
            o.append(extra)
            n_tok += extra
        nb = (n_tok + bt - 1) // bt
        ids = rng.choice(nb + 3, size=int(rng.integers(0, nb + 1)), replace=True)
        force = bool(rng.random() < 0.1)
        a = t.set_selection(ids, force)
        b = o.set_selection(ids, force)
        for x, y in zip(a, b):
            assert np.array_equal(x, y)


@needs_ref
@pytest.mark.parametrize("seed", range(6))
def test_plan_equals_reference_runtime(seed):
    rng = np.random.default_rng(300 + seed)
    bt = 128
    t = _table(bt, 1 << 20)
    r = po.RefRuntime(bt, 1 << 20, 1, False)
    t.append(bt * 300)
    r.append(bt * 300)
    for _ in range(10):
        ids = rng.choice(300, size=int(rng.integers(1, 64)), replace=False)
        a = t.set_selection(ids)
        b = r.set_selection(ids)
        for x, y in zip(a, b):
            assert np.array_equal(x, y)


def test_keep_all_fit_and_empty():
    t = _table(128, 8)
    kept, kc, need = t.keep()
    assert len(kept) == 0 and kc == 0 and need == 0
    t.append(128 * 3)
    kept, kc, need = t.keep()
    assert list(kept) == [1, 1, 1] and need == 0


@pytest.mark.parametrize("immutable", [False, True])
@pytest.mark.parametrize("seed", range(4))
def test_clear_working_set_equals_oracle(seed, immutable):
    """clear_working_set between selections (with and without dropping the GPU
    tier): the next plans stay identical to the oracle's."""
    rng = np.random.default_rng(400 + seed)
    bt = 16
    t = _table(bt, 1 << 20, immutable=immutable)
    o = po.Store(bt, immutable)
    t.append(bt * 60)
    o.append(bt * 60)
    for step in range(12):
        if step % 3 == 2:
            drop = bool(rng.random() < 0.5)
            t.clear_working_set(drop)
            o.clear_working_set(drop)
        ids = rng.choice(60, size=int(rng.integers(1, 40)), replace=False)
        for x, y in zip(t.set_selection(ids), o.set_selection(ids)):
            assert np.array_equal(x, y)


@needs_ref
@pytest.mark.parametrize("seed", range(4))
def test_clear_working_set_equals_reference_runtime(seed):
    """The reference store's clear_working_set (kvmem_store.cpp:897-901): after
    it every selected block is staged in again, resident ones as resident."""
    rng = np.random.default_rng(500 + seed)
    bt = 128
    t = _table(bt, 1 << 20)
    r = po.RefRuntime(bt, 1 << 20, 1, False)
    t.append(bt * 200)
    r.append(bt * 200)
    for step in range(9):
        if step % 3 == 1:
            t.clear_working_set()
            r.clear_working_set()
        ids = rng.choice(200, size=int(rng.integers(1, 48)), replace=False)
        a = t.set_selection(ids)
        b = r.set_selection(ids)
        for x, y in zip(a, b):
            assert np.array_equal(x, y)
        if step % 3 == 1:  # right after the clear: every selected block stages in
            assert a[3][0] == len(set(ids.tolist()))


try:
    from hypothesis import given, settings, strategies as hs
except ImportError:  # pragma: no cover - hypothesis is part of the test image
    hs = None

if hs is not None:
    _op = hs.one_of(
        hs.tuples(hs.just("append"), hs.integers(1, 80)),
        hs.tuples(hs.just("clear"), hs.booleans()),
        hs.tuples(hs.just("select"), hs.lists(hs.integers(0, 70), max_size=40), hs.booleans()),
        hs.tuples(hs.just("truncate"), hs.floats(0.0, 1.0)),
        hs.tuples(hs.just("tier_gpu"), hs.integers(0, 70)),
    )

    @needs_ref
    @settings(max_examples=60, deadline=None, derandomize=True)
    @given(first=hs.integers(1, 600), ops=hs.lists(_op, min_size=1, max_size=14),
           immutable=hs.booleans())
    def test_random_op_sequences_match_oracle_and_reference(first, ops, immutable):
        """Any sequence of appends, truncations, tier changes to GPU, working-set
        clears (keeping the GPU tier, the reference's form; or dropping it) and
        selections, with forced refreshes: the host table, the oracle and the
        reference runtime give
        the same plans (the reference only for clears that keep the tier)."""
        bt = 16
        t = _table(bt, 1 << 20, immutable=immutable)
        o = po.Store(bt, immutable)
        r = po.RefRuntime(bt, 1 << 20, 1, immutable)
        ref_ok = True
        for x in (t, o, r):
            x.append(first)
        n_tok = first
        for op in ops:
            if op[0] == "append":
                for x in (t, o, r):
                    x.append(op[1])
                n_tok += op[1]
            elif op[0] == "truncate":  # KvMemStore::truncate_to
                n_tok = int(op[1] * n_tok)
                for x in (t, o, r):
                    x.truncate(n_tok)
            elif op[0] == "tier_gpu":  # a decode block given a reserve slot
                for x in (t, o, r):
                    x.set_tier_gpu(op[1])
            elif op[0] == "clear":
                t.clear_working_set(op[1])
                o.clear_working_set(op[1])
                if op[1]:
                    ref_ok = False  # the reference store has no tier drop
                else:
                    r.clear_working_set()
            else:
                ids = np.asarray(op[1], np.uint32)
                a, b = t.set_selection(ids, op[2]), o.set_selection(ids, op[2])
                for x, y in zip(a, b):
                    assert np.array_equal(x, y)
                if ref_ok:
                    for x, y in zip(a, r.set_selection(ids, op[2])):
                        assert np.array_equal(x, y)
