"""The control kernels at sizes beyond the headline configuration.

- `kvmret_topk_select` (the radix top-k behind every retrieval step) against
  the rank rule it restates (kvmem_store.cpp:600-616: score desc, ties by id,
  nth_element's set for that strict total order), from 1 to 100,000 blocks,
  with heavy ties, all-equal scores, mixed -0.0 / +0.0, kept blocks and
  `need` from 0 to beyond the candidates, under both tie rules. Sizes on both
  sides of the shared-memory staging limit (16,384) are covered.
- the plan kernel's least-recently-used eviction (a radix selection over
  (last use, slot)) against a host model of the pool, with pools of up to
  8192 slots: the blocks copied from the host at each step and the window
  contents must match.
"""
import numpy as np
import pytest
import torch

import kvmret
from kvm_helpers import append_history, check_window, config_for
from kvmret import synth

pytestmark = pytest.mark.gpu


def _want(scores, kept, need, tie_high):
    """Rank rule on the host: kept blocks plus the `need` best others."""
    n = len(scores)
    ids = np.arange(n)
    cand = ids[kept == 0]
    sc = scores[cand]
    # lexsort: last key primary; -0.0 and +0.0 compare equal
    order = np.lexsort(((-cand if tie_high else cand), -sc))
    out = kept.astype(np.uint8).copy()
    out[cand[order[:need]]] = 1
    return out


def _scores(rng, n, kind):
    if kind == "gauss":
        return rng.normal(0.0, 0.01, n)
    if kind == "ties":
        return np.round(rng.normal(0.0, 1.0, n), 1)
    if kind == "equal":
        return np.full(n, 0.25)
    if kind == "zeros":
        return np.where(rng.random(n) < 0.5, 0.0, -0.0)
    return rng.uniform(-1.0, 1.0, n)


@pytest.mark.parametrize("n", [1, 2, 31, 2048, 8192, 16384, 16385, 100_000])
@pytest.mark.parametrize("kind", ["gauss", "ties", "equal", "zeros", "uniform"])
def test_topk_select_matches_rank_rule(n, kind):
    rng = np.random.default_rng(n * 7 + len(kind))
    scores = _scores(rng, n, kind)
    kept = (rng.random(n) < 0.05).astype(np.uint8)
    n_cand = int(n - kept.sum())
    d_sc = torch.from_numpy(scores).cuda()
    d_kept = torch.from_numpy(kept).cuda()
    for need in sorted({0, 1, n_cand // 3, max(0, n_cand - 1), n_cand, n_cand + 5}):
        for tie_high in (True, False):
            got = kvmret.topk_select(d_sc, d_kept, need, tie_high).cpu().numpy()
            want = _want(scores, kept, need, tie_high)
            assert np.array_equal(got, want), (n, kind, need, tie_high)


class _PoolModel:
    """The pool as the plan kernel keeps it with caching on: free slots taken
    in ascending order, then blocks outside the new window evicted by
    (last use, slot), the k-th slot to the k-th block that needs one in
    window order."""

    def __init__(self, P):
        self.P = P
        self.slot_blk = [-1] * P
        self.blk_slot = {}
        self.used = [0] * P
        self.step = 0

    def plan(self, ids):
        self.step += 1
        sel = set(ids)
        need = [b for b in ids if b not in self.blk_slot]
        free = [s for s in range(self.P) if self.slot_blk[s] < 0]
        if len(need) > len(free):
            cand = sorted((self.used[s], s) for s in range(self.P)
                          if self.slot_blk[s] >= 0 and self.slot_blk[s] not in sel)
            for _, s in cand[:len(need) - len(free)]:
                del self.blk_slot[self.slot_blk[s]]
                self.slot_blk[s] = -1
                free.append(s)
        assert len(need) <= len(free)
        for b, s in zip(need, free):
            self.slot_blk[s] = b
            self.blk_slot[b] = s
        for b in ids:
            self.used[self.blk_slot[b]] = self.step
        return len(need)


@pytest.mark.parametrize("pool,budget,n_blocks,steps", [
    (96, 32, 400, 60),       # deficits of many blocks per step, ties in last use
    (8192, 64, 12000, 120),  # the largest pool: 8k candidates per eviction
])
def test_lru_eviction_matches_pool_model(pool, budget, n_blocks, steps):
    w = synth.Workload("lru", n_layer=1, n_head=2, n_head_kv=1, d_head=64, block_tokens=16,
                       n_blocks=n_blocks, budget_blocks=budget, sink_blocks=0,
                       reserve_blocks=0, n_planted=0, seed=21)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w, pool_cache=1, pool_blocks=pool))
    append_history(r, hist, cuts=[w.n_tokens // 2])
    model = _PoolModel(pool)
    rng = np.random.default_rng(pool)
    hot = rng.choice(n_blocks, size=min(n_blocks, pool + pool // 2), replace=False)
    for s in range(steps):
        # mostly a hot set slightly larger than the pool, sometimes anything
        src = hot if rng.random() < 0.8 else np.arange(n_blocks)
        k = int(rng.integers(1, budget + 1))
        ids = sorted(int(x) for x in rng.choice(src, size=k, replace=False))
        st = r.apply(ids)
        assert st["n_h2d_blocks"] == model.plan(ids), s
        if s % 20 == 19 or s == steps - 1:
            check_window(r, hist, w.n_tokens, ids)
    r.close()
