"""Prefill scoring on the tensor cores (config 4's path; an extension of the
reference, which scores the mean query of a span — parity is against the
stated semantics, not a reference output).

- the tcgen05 GEMM against a float64 product of the same f16 operands;
- the per-token scores against a float64 restatement (unit-length group
  queries and summaries, mean cosine over layers and KV heads), within the
  f16-operand tolerance;
- the union of the per-token top-k exactly equal to the host's top-k of the
  returned scores under the tie rule, and consistent with the float64 scores
  up to the tolerance band at each token's cut;
- the unit summaries kept current across appends.
"""
import numpy as np
import pytest
import torch

import kvmret
from kvm_helpers import append_history, config_for
from kvmret import synth

pytestmark = pytest.mark.gpu

SCORE_TOL = 3e-3  # f16 unit-length operands: |cos error| <= ~2 * 2^-11 per term


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 1024), (128, 768, 8192),
                                   (128, 256, 65536), (128, 272, 128), (2048, 2048, 1024),
                                   (1280, 2000, 512)])
def test_gemm_matches_float64(m, n, k):
    """Whole 256-wide tiles (the first four and 2048 x 2048) and partial last
    tiles: 128 x 272 (a 16-column last tile) and 1280 x 2000 (a 208-column
    last tile, so one 32-column chunk of the epilogue is cut at 16)."""
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = (torch.randn(m, k, device="cuda", generator=g) * 0.5).half()
    b = (torch.randn(n, k, device="cuda", generator=g) * 0.5).half()
    c, err = kvmret.gemm_f16_nt(a, b, alpha=0.25)
    torch.cuda.synchronize()
    assert int(err[0]) == 0
    a64, b64 = a.double().cpu(), b.double().cpu()
    ref = 0.25 * (a64 @ b64.T)
    bound = 0.25 * (a64.abs() @ b64.abs().T) * 2e-6 + 1e-6  # f32 accumulation over k
    assert torch.all((c.double().cpu() - ref).abs() <= bound)


@pytest.mark.parametrize("m,n,k", [(128, 768, 8192), (512, 2048, 4096), (256, 512, 64),
                                   (2048, 2048, 1024), (256, 272, 4096)])
def test_split_gemm_matches_float64(m, n, k):
    """The workspace form: with few tiles (3, 32, 4) one CTA per SM runs (a
    lockstep CTA per tile for the first k-steps, helpers on the k tails, the
    pieces added by the fix-up launch; 256 x 272 with 16-column last tiles);
    with a single k-step per tile (256 x 512 x 64) or 128 tiles, where the
    split would not pay, a tile per CTA. Same bound as the plain form, and
    the same result on a second run."""
    g = torch.Generator(device="cuda").manual_seed(m * 3 + n + k)
    a = (torch.randn(m, k, device="cuda", generator=g) * 0.5).half()
    b = (torch.randn(n, k, device="cuda", generator=g) * 0.5).half()
    c, err = kvmret.gemm_f16_nt_split(a, b, alpha=0.5)
    c2, err2 = kvmret.gemm_f16_nt_split(a, b, alpha=0.5)
    torch.cuda.synchronize()
    assert int(err[0]) == 0 and int(err2[0]) == 0
    assert torch.equal(c, c2)
    a64, b64 = a.double().cpu(), b.double().cpu()
    ref = 0.5 * (a64 @ b64.T)
    bound = 0.5 * (a64.abs() @ b64.abs().T) * 2e-6 + 1e-6
    assert torch.all((c.double().cpu() - ref).abs() <= bound)


def _oracle_scores(hist, q, w, n_tokens):
    """float64: mean over (layer, KV head) of cos(group query of token t, summary of b),
    the summary being the mean key of the block's appended tokens."""
    L, Hq, Hkv, D, T = w.n_layer, w.n_head, w.n_head_kv, w.d_head, w.block_tokens
    n_tok = q.shape[1]
    n_blocks = (n_tokens + T - 1) // T
    qg = q.astype(np.float64).reshape(L, n_tok, Hkv, Hq // Hkv, D).sum(axis=3)
    qn = qg / np.maximum(np.linalg.norm(qg, axis=-1, keepdims=True), 1e-300)
    k = hist.k.reshape(L, -1, Hkv, D)[:, :n_tokens].astype(np.float64)
    m = np.stack([k[:, b * T:min((b + 1) * T, n_tokens)].mean(axis=1)
                  for b in range(n_blocks)], axis=1)  # [L][b][g][D]
    mn = m / np.maximum(np.linalg.norm(m, axis=-1, keepdims=True), 1e-300)
    return np.einsum("ltgd,lbgd->tb", qn, mn) / (L * Hkv)


def _host_topk_union(s, top_k, tie_high):
    n_tok, nb = s.shape
    sel = np.zeros(nb, np.uint8)
    ids = np.arange(nb)
    for t in range(n_tok):
        key = -ids if tie_high else ids
        order = np.lexsort((key, -s[t].astype(np.float64)))
        sel[order[:top_k]] = 1
    return sel


@pytest.mark.parametrize("tie_high", [1, 0])
def test_prefill_scores_and_union(tie_high):
    w = synth.Workload("pf", n_layer=4, n_head=16, n_head_kv=4, d_head=128, block_tokens=64,
                       n_blocks=300, budget_blocks=32, sink_blocks=1, reserve_blocks=4,
                       n_planted=6, seed=41)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w, tie_higher_id=tie_high))
    n_first = 250 * w.block_tokens + 17  # a partial block at the end
    append_history(r, hist, cuts=[n_first], stop=n_first)
    top_k = 24
    rng = np.random.default_rng(5)
    for rnd, n_tok in enumerate((200, 384)):
        nb = int(kvmret.lib.kvmret_n_blocks(r.h))
        n_app = int(kvmret.lib.kvmret_n_tokens(r.h))
        q = (rng.standard_normal((w.n_layer, n_tok, w.n_head * w.d_head)) +
             hist.q0.reshape(w.n_layer, 1, -1) * 0.3).astype(np.float16)
        sel, n_sel, s = r.prefill_score(torch.from_numpy(q).cuda(), top_k, scores=True)
        assert s.shape == (n_tok, nb)
        want = _oracle_scores(hist, q, w, n_app)
        assert np.abs(s - want).max() <= SCORE_TOL
        # union: exactly the host top-k of the returned scores
        assert np.array_equal(sel, _host_topk_union(s, top_k, tie_high))
        assert n_sel == int(sel.sum())
        # consistent with the float64 scores outside each token's tolerance band
        kth = np.sort(want, axis=1)[:, -top_k]
        certain = (want >= kth[:, None] + 2 * SCORE_TOL).any(axis=0)
        possible = (want >= kth[:, None] - 2 * SCORE_TOL).any(axis=0)
        assert np.all(sel[certain] == 1) and np.all(possible[sel == 1])
        if rnd == 0:  # append the rest: the stale unit summaries must be refreshed
            append_history(r, hist, cuts=[], start=n_first)
    r.close()


def test_prefill_top_k_above_block_count_selects_all():
    w = synth.Workload("pf2", n_layer=2, n_head=8, n_head_kv=8, d_head=64, block_tokens=32,
                       n_blocks=20, budget_blocks=8, sink_blocks=1, reserve_blocks=0,
                       n_planted=2, seed=43)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w))
    append_history(r, hist, cuts=[])
    q = np.random.default_rng(1).standard_normal(
        (w.n_layer, 130, w.n_head * w.d_head)).astype(np.float16)
    sel, n_sel, _ = r.prefill_score(torch.from_numpy(q).cuda(), 64)
    assert n_sel == w.n_blocks and sel.all()
    r.close()
