"""kvmret_score_noalloc — the scorer for callers that cannot allocate device
memory (allocator hooks, memory managers that own the whole device, serving
paths where cudaMalloc is forbidden).

Called through the C ABI on caller-owned buffers, twice in a row (with two
different queries, so the second call must overwrite the first call's scratch),
its scores must match those of the existing entry point kvmret_score within
the scorer tolerance of the other tests (1e-3 relative; bit-exact expected).
Collected last so that a failure here leaves every other test already run;
it also passes alone in a fresh process.
"""
import numpy as np
import pytest
import torch

import kvmret
from kvm_helpers import append_history, config_for
from kvmret import synth

pytestmark = pytest.mark.gpu


def test_noalloc_scores_match_existing_entry_point_twice():
    w = synth.scaled(synth.CONFIGS[1], n_blocks=100, budget_blocks=12, n_planted=4)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w))
    append_history(r, hist, cuts=[700])
    L, E, N = w.n_layer, w.E, w.n_blocks
    stride = r.contrib_stride
    assert stride % 64 == 0 and stride >= N
    # padding columns between n_blocks and the stride must never reach a score
    summ = np.full((L, E, stride), np.nan, np.float32)
    summ[:, :, :N] = r.summaries().transpose(1, 2, 0)
    summ_d = torch.from_numpy(summ).cuda()
    has_d = torch.ones(N, dtype=torch.uint8, device="cuda")
    out = torch.empty(N, dtype=torch.float64, device="cuda")
    q = hist.queries(2)
    for s in range(2):
        r.query_reset()
        r.query_add(torch.from_numpy(q[s].reshape(L, 1, -1)).cuda())
        want = r.score()
        q_sum, q_count = r.query_get()
        qs_d = torch.from_numpy(q_sum).cuda()
        qc_d = torch.from_numpy(q_count.astype(np.int32)).cuda()
        out.fill_(float("nan"))
        torch.cuda.synchronize()
        rc = kvmret.lib.kvmret_score_noalloc(
            summ_d.data_ptr(), stride, qs_d.data_ptr(), qc_d.data_ptr(), has_d.data_ptr(), N, L,
            w.n_head, w.n_head_kv, w.d_head, out.data_ptr(), None)
        assert rc == 0, kvmret.lib.kvmret_last_error()
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        rel = np.abs(got - want) / np.maximum(np.abs(want), 1e-30)
        assert rel.max() <= 1e-3
        assert np.array_equal(got, want)
    r.close()


@pytest.mark.parametrize("d_head,n_blocks", [(64, 700), (256, 300), (128, 12000)])
def test_noalloc_matches_oracle_across_head_dims_and_tile_forms(d_head, n_blocks):
    """d_head 64 / 256, and 12000 blocks x 8 layers: enough 64-block tiles
    that the scorer takes its wide-tile form. Padding columns hold NaN; blocks
    without data score 0. Two calls in a row with different queries."""
    import pyoracle as po
    rng = np.random.default_rng(d_head + n_blocks)
    L, Hq, Hkv = 8, 8, 2
    E = Hkv * d_head
    stride = (n_blocks + 63) // 64 * 64 + 64
    mean = rng.standard_normal((n_blocks, L, E)).astype(np.float32)
    has = (rng.random(n_blocks) > 0.05).astype(np.uint8)
    summ = np.full((L, E, stride), np.nan, np.float32)
    summ[:, :, :n_blocks] = mean.transpose(1, 2, 0)
    summ_d = torch.from_numpy(summ).cuda()
    has_d = torch.from_numpy(has).cuda()
    out = torch.empty(n_blocks, dtype=torch.float64, device="cuda")
    for call in range(2):
        q_sum = rng.standard_normal((L, Hq * d_head)).astype(np.float32)
        q_count = np.full(L, 1 + call, np.uint32)
        q_count[3] = 0  # a layer without query rows
        want = po.score(mean, has, q_sum, q_count, Hq, Hkv, d_head)
        qs_d = torch.from_numpy(q_sum).cuda()
        qc_d = torch.from_numpy(q_count.astype(np.int32)).cuda()
        out.fill_(float("nan"))
        torch.cuda.synchronize()
        rc = kvmret.lib.kvmret_score_noalloc(
            summ_d.data_ptr(), stride, qs_d.data_ptr(), qc_d.data_ptr(), has_d.data_ptr(),
            n_blocks, L, Hq, Hkv, d_head, out.data_ptr(), None)
        assert rc == 0, kvmret.lib.kvmret_last_error()
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.array_equal(got, want)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    dummy = torch.zeros(64, dtype=torch.float32, device="cuda")
    out = torch.zeros(64, dtype=torch.float64, device="cuda")
    # 64 layers x 32768-block stride needs 16 MiB of score terms: over the 8 MiB limit
    rc = kvmret.lib.kvmret_score_noalloc(dummy.data_ptr(), 32768, dummy.data_ptr(),
                                         dummy.data_ptr(), dummy.data_ptr(), 64, 64, 64, 8, 128,
                                         out.data_ptr(), None)
    assert rc == -1  # KVMRET_ERR_ARG
    assert b"exceeds" in kvmret.lib.kvmret_last_error()
