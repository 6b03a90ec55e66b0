"""Decode-time append (the reference's running mean-K with block-full flush,
llama-kvmem-stagein.cu:270-320 and llama-memory-kvmem.cpp:3855-3998): tokens
arrive one per decode step; the newest block's summary is the token-order f32
running sum times 1/tokens after every token, bit-exact against the oracle,
across block boundaries, and the tokens land in the pinned repository. A
retrieval step then stages the partial newest block as a mandatory block.
"""
import numpy as np
import pytest
import torch

import kvmret
import pyoracle as po
from kvm_helpers import append_history, config_for, f16_ulp_diff
from kvmret import synth

pytestmark = pytest.mark.gpu


def _want_summaries(hist, n_app):
    w = hist.w
    L, T, E = w.n_layer, w.block_tokens, w.E
    k = hist.k.reshape(L, -1, E)[:, :n_app]
    out = []
    for b in range((n_app + T - 1) // T):
        t1 = min((b + 1) * T, n_app)
        out.append(po.mean_k(np.ascontiguousarray(k[:, b * T:t1])))  # [L][E]
    return np.stack(out)  # [b][L][E]


def test_single_token_appends_keep_running_summaries_exact():
    w = synth.Workload("dec", n_layer=2, n_head=8, n_head_kv=2, d_head=128, block_tokens=64,
                       n_blocks=20, budget_blocks=6, sink_blocks=1, reserve_blocks=2,
                       n_planted=2, seed=77)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w))
    T, L, E = w.block_tokens, w.n_layer, w.E
    n0 = 10 * T + 5
    append_history(r, hist, cuts=[], stop=n0)
    k = hist.k.reshape(L, -1, E)
    v = hist.v.reshape(L, -1, E)
    n_app = n0
    checkpoints = {n0 + 1, 11 * T - 1, 11 * T, 11 * T + 1, 12 * T, 13 * T + 20}
    while n_app < 13 * T + 20:
        kc = torch.from_numpy(np.ascontiguousarray(k[:, n_app:n_app + 1])).cuda()
        vc = torch.from_numpy(np.ascontiguousarray(v[:, n_app:n_app + 1])).cuda()
        r.append(kc, vc, pos0=n_app)
        n_app += 1
        if n_app in checkpoints:
            r.sync()
            got = r.summaries()
            want = _want_summaries(hist, n_app)
            assert got.shape == want.shape
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), n_app
    # the repository holds every appended token's K and V rows
    repo = r.repo_view()
    unit = int(kvmret.lib.kvmret_repo_unit_bytes(r.h))
    kpart = int(kvmret.lib.kvmret_repo_k_bytes(r.h))
    for b in (10, 11, 12, 13):
        n_b = min(T, n_app - b * T)
        for l in range(L):
            u = repo[(b * L + l) * unit:(b * L + l + 1) * unit]
            kb = k[l, b * T:b * T + n_b].reshape(-1).view(np.uint8)
            vb = v[l, b * T:b * T + n_b].reshape(-1).view(np.uint8)
            assert np.array_equal(u[:kb.size], kb)
            assert np.array_equal(u[kpart:kpart + vb.size], vb)
    # a retrieval step with the partial newest block pinned
    newest = n_app // T
    r.query_reset()
    r.query_add(torch.from_numpy(hist.q0.reshape(L, 1, -1)).cuda())
    ids, _ = r.apply_retrieval(mandatory=[newest])
    assert newest in ids.tolist()
    lay, bases = r.window_layout()
    i = list(lay).index(newest)
    n_b = n_app - newest * T
    wk = r.window_read(0, False, i, 1).view(np.uint16).reshape(T, w.n_head_kv, w.d_head)[:n_b]
    want = po.rope_block_f16(k[0, newest * T:n_app].view(np.uint16).reshape(
        n_b, w.n_head_kv, w.d_head), int(bases[i]), w.freq_base)
    assert f16_ulp_diff(wk, want).max() <= 2
    r.close()
