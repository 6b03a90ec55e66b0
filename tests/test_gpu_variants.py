"""GPU parity beyond config 1: quantised K windows (q8_0 / q4_0 K, dequant ->
RoPE -> FWHT -> requant within 1 LSB), other head geometries (d_head 64 / 256, no
GQA, odd group sizes), layers without a query, ties under both tie rules,
mandatory pinning, the stateless RoPE entry points and batched copies."""
import ctypes

import numpy as np
import pytest
import torch

import kvmret
import pyoracle as po
from kvm_helpers import (append_history, config_for, f16_ulp_diff, history_units,
                         oracle_scores, q4_blocks_diff, q8_blocks_diff)
from kvmret import synth

pytestmark = pytest.mark.gpu


def _quant_rows(fn, row_bytes):
    def f(x):  # x [L][n][E] f16 -> [L][n][row_bytes] u8
        L, n, E = x.shape
        return fn(x.astype(np.float32)).reshape(L, n, row_bytes)
    return f


_QROW = {kvmret.TYPE_Q8_0: (po.quant_q8_0, 34), kvmret.TYPE_Q4_0: (po.quant_q4_0, 18),
         kvmret.TYPE_F16: (None, 64)}


def _rows_fn(t, E):
    fn, per = _QROW[t]
    if fn is None:
        return None, E * 2
    return _quant_rows(fn, E // 32 * per), E // 32 * per


@pytest.mark.parametrize("kt,vt", [(kvmret.TYPE_Q8_0, kvmret.TYPE_Q4_0),
                                   (kvmret.TYPE_Q4_0, kvmret.TYPE_Q8_0),
                                   (kvmret.TYPE_Q8_0, kvmret.TYPE_F16)])
def test_quant_k_window(kt, vt):
    """Window K for quantised K (dequant -> RoPE -> FWHT -> requant) within
    1 LSB of the oracle, V bytes exact, over fresh and moved blocks."""
    w = synth.scaled(synth.CONFIGS[3], n_layer=2, n_blocks=48, budget_blocks=12,
                     reserve_blocks=4, n_planted=4, n_head=16, k_type=kt, v_type=vt)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w))
    L, n, E = w.n_layer, w.n_tokens, w.E
    kq, krow = _rows_fn(kt, E)
    vq, vrow = _rows_fn(vt, E)
    append_history(r, hist, cuts=[130, 3000], k_rows_fn=kq, v_rows_fn=vq)
    k_q = kq(hist.k.reshape(L, n, E)).reshape(L, w.n_blocks, w.block_tokens * krow)
    if vq is None:
        v_b = hist.v.reshape(L, w.n_blocks, -1).view(np.uint8)
    else:
        v_b = vq(hist.v.reshape(L, n, E)).reshape(L, w.n_blocks, w.block_tokens * vrow)
    rope = po.rope_block_q8_0 if kt == kvmret.TYPE_Q8_0 else po.rope_block_q4_0
    diff = q8_blocks_diff if kt == kvmret.TYPE_Q8_0 else q4_blocks_diff
    q = hist.queries(3)
    worst_q, worst_d = 0, 0
    for s in range(3):
        r.query_reset()
        r.query_add(torch.from_numpy(q[s].reshape(L, 1, -1)).cuda())
        got = r.score()
        want, _ = oracle_scores(hist, q[s].reshape(L, -1).astype(np.float32),
                                np.ones(L, np.uint32))
        assert np.array_equal(got, want)  # summaries come from the f16 capture (F5)
        ids = r.select()
        assert list(ids) == list(po.pick_topk(want, w.budget_blocks, w.sink_blocks))
        r.apply(ids)
        lay_ids, bases = r.window_layout()
        for l in range(L):
            wk = r.window_read(l, False, 0, len(lay_ids)).reshape(len(lay_ids), -1)
            wv = r.window_read(l, True, 0, len(lay_ids)).reshape(len(lay_ids), -1)
            for i, (b, base) in enumerate(zip(lay_ids, bases)):
                want_k = rope(k_q[l, b], w.block_tokens, w.n_head_kv, w.d_head, int(base),
                              w.freq_base, fwht_n=128)
                dq, dd = diff(wk[i], want_k)
                worst_q, worst_d = max(worst_q, dq), max(worst_d, dd)
                assert np.array_equal(wv[i], v_b[l, b])
    assert worst_q <= 1 and worst_d <= 1
    r.close()


@pytest.mark.parametrize("hq,hkv,d,t", [(8, 8, 64, 64), (32, 4, 256, 32), (12, 4, 128, 128),
                                        (16, 2, 128, 16)])
def test_geometries(hq, hkv, d, t):
    w = synth.Workload("geo", n_layer=3, n_head=hq, n_head_kv=hkv, d_head=d, block_tokens=t,
                       n_blocks=70, budget_blocks=9, sink_blocks=2, reserve_blocks=3,
                       n_planted=3, seed=11)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w))
    append_history(r, hist, cuts=[t // 2, 5 * t + 3])
    L = w.n_layer
    q = hist.queries(2)
    store = po.Store(t)
    store.append(w.n_tokens)
    for s in range(2):
        # layer 1 carries no query rows this step: it must be skipped (q_count == 0)
        q_sum = q[s].reshape(L, -1).astype(np.float32)
        q_count = np.array([1, 0, 2], np.uint32)
        q_sum[2] *= 2
        r.query_set(q_sum, q_count)
        got = r.score()
        want, _ = oracle_scores(hist, q_sum, q_count)
        assert np.array_equal(got, want)
        ids = r.select(mandatory=[5, 60])
        assert list(ids) == list(po.pick_topk(want, w.budget_blocks, 2, 0, [5, 60]))
        r.apply(ids)
        si, so, rm, c = store.set_selection(ids)
        assert np.array_equal(r.last_plan().remaps, rm)
    k, v = history_units(hist)
    lay_ids, bases = r.window_layout()
    for l in range(L):
        wk = r.window_read(l, False, 0, len(lay_ids)).view(np.uint16).reshape(
            len(lay_ids), t, hkv, d)
        for i, (b, base) in enumerate(zip(lay_ids, bases)):
            want = po.rope_block_f16(k[b, l].view(np.uint16).reshape(t, hkv, d), int(base),
                                     w.freq_base)
            assert f16_ulp_diff(wk[i], want).max() <= 2
    r.close()


@pytest.mark.parametrize("tie_higher", [1, 0])
def test_ties_follow_tie_rule(tie_higher):
    w = synth.Workload("ties", n_layer=2, n_head=8, n_head_kv=8, d_head=128, block_tokens=32,
                       n_blocks=40, budget_blocks=10, sink_blocks=1, reserve_blocks=0,
                       n_planted=0, seed=21)
    hist = synth.NumpyHistory(w)
    # blocks 10..29 are copies of block 9: twenty exactly tied scores
    T = w.block_tokens
    for b in range(10, 30):
        hist.k[:, b * T:(b + 1) * T] = hist.k[:, 9 * T:10 * T]
    # make block 9's content the best match so the tie straddles the cut
    hist.k[:, 9 * T:30 * T] += hist.q0.astype(np.float16).reshape(
        w.n_layer, 1, w.n_head_kv, w.d_head)
    r = kvmret.Retriever(config_for(w, tie_higher_id=tie_higher))
    append_history(r, hist, cuts=[])
    r.query_reset()
    r.query_add(torch.from_numpy(hist.q0.reshape(w.n_layer, 1, -1)).cuda())
    got = r.score()
    assert len(set(got[9:30].tolist())) == 1
    ids = r.select()
    want = po.pick_topk(got, w.budget_blocks, 1, 0, (), bool(tie_higher))
    assert list(ids) == list(want)
    tied = [i for i in ids if 9 <= i < 30]
    assert tied == (list(range(30 - len(tied), 30)) if tie_higher else list(range(9, 9 + len(tied))))
    r.close()


def test_stateless_rope_f16():
    rng = np.random.default_rng(3)
    n, hkv, d = 300, 8, 128
    x = rng.standard_normal((n, hkv, d)).astype(np.float16)
    k = torch.from_numpy(x).cuda()
    out = torch.empty_like(k)
    kvmret.rope_f16(k, out, 12345, hkv, d, 1e6)
    torch.cuda.synchronize()
    want = po.rope_block_f16(x.view(np.uint16), 12345, 1e6)
    assert f16_ulp_diff(out.cpu().numpy().view(np.uint16), want).max() <= 2


# ragged token counts (partial warp segments, a partial last 128-token chunk),
# every head size, FWHT on and off
@pytest.mark.parametrize("qt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("n,hkv,d,fwht", [(300, 8, 128, 128), (37, 2, 128, 0), (129, 4, 64, 64),
                                          (70, 2, 256, 256), (5, 6, 256, 0)])
def test_stateless_rope_quant(qt, n, hkv, d, fwht):
    rng = np.random.default_rng(n + d)
    x = (rng.standard_normal((n, hkv, d)) * 3).astype(np.float16)
    if qt == "q8_0":
        q = po.quant_q8_0(x.astype(np.float32)).reshape(n, -1)
        fn, want_fn, diff = kvmret.rope_q8_0, po.rope_block_q8_0, q8_blocks_diff
    else:
        q = po.quant_q4_0(x.astype(np.float32)).reshape(n, -1)
        fn, want_fn, diff = kvmret.rope_q4_0, po.rope_block_q4_0, q4_blocks_diff
    kq = torch.from_numpy(q).cuda()
    oq = torch.full_like(kq, 0xAB)
    fn(kq, oq, n, 777, hkv, d, 1e6, fwht_n=fwht)
    torch.cuda.synchronize()
    want = want_fn(q, n, hkv, d, 777, 1e6, fwht_n=fwht)
    dq, dd = diff(oq.cpu().numpy(), want)
    assert dq <= 1 and dd <= 1


def test_gpu_quantiser_matches_oracle_bit_exact():
    rng = np.random.default_rng(12)
    x = (rng.standard_normal(32 * 1000) * 3).astype(np.float16)
    x[:32] = 0  # an all-zero block (d = 0)
    xd = torch.from_numpy(x).cuda()
    q8 = kvmret.quantize_f16(xd, kvmret.TYPE_Q8_0).cpu().numpy()
    q4 = kvmret.quantize_f16(xd, kvmret.TYPE_Q4_0).cpu().numpy()
    assert np.array_equal(q8, po.quant_q8_0(x.astype(np.float32)))
    assert np.array_equal(q4, po.quant_q4_0(x.astype(np.float32)))


def test_d2d_batched():
    w = synth.CONFIGS[1]
    r = kvmret.Retriever(config_for(synth.scaled(w, n_blocks=8, budget_blocks=4)))
    src = torch.arange(4096, dtype=torch.uint8, device="cuda").repeat(8)
    dst = torch.zeros_like(src)
    sizes = [16, 4096, 333, 1000]
    offs = [0, 100, 5000, 20000]
    S = (ctypes.c_void_p * 4)(*[src.data_ptr() + o for o in offs])
    D = (ctypes.c_void_p * 4)(*[dst.data_ptr() + o + 7 for o in offs])
    N = (ctypes.c_uint64 * 4)(*sizes)
    torch.cuda.synchronize()
    assert kvmret.lib.kvmret_d2d_batched(r.h, S, D, N, 4) == 0
    r.sync()
    s, d_ = src.cpu().numpy(), dst.cpu().numpy()
    for o, z in zip(offs, sizes):
        assert np.array_equal(d_[o + 7:o + 7 + z], s[o:o + z])
    r.close()


def test_quant_k_partial_newest_block():
    """A q8_0 K history ending mid-block: the partial newest block, pinned by the
    mandatory list, is requantised row for row (the rows past its end stay
    untouched work items)."""
    w = synth.scaled(synth.CONFIGS[3], n_layer=2, n_blocks=24, budget_blocks=6,
                     reserve_blocks=2, n_planted=2, n_head=16)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w))
    T, L, E = w.block_tokens, w.n_layer, w.E
    n_app = 20 * T + 37
    kq, vq = _quant_rows(po.quant_q8_0, 1088), _quant_rows(po.quant_q4_0, 576)
    append_history(r, hist, cuts=[], k_rows_fn=kq, v_rows_fn=vq, stop=n_app)
    newest = n_app // T
    k_all = kq(hist.k.reshape(L, -1, E)[:, :n_app])
    for s in range(2):
        r.query_reset()
        r.query_add(torch.from_numpy(hist.queries(2)[s].reshape(L, 1, -1)).cuda())
        ids, _ = r.apply_retrieval(mandatory=[newest])
        assert newest in ids.tolist()
    lay, bases = r.window_layout()
    i = list(lay).index(newest)
    n_b = n_app - newest * T
    for l in range(L):
        wk = r.window_read(l, False, i, 1).reshape(T, -1)[:n_b]
        want = po.rope_block_q8_0(k_all[l, newest * T:n_app], n_b, w.n_head_kv, w.d_head,
                                  int(bases[i]), w.freq_base, fwht_n=128)
        dq, dd = q8_blocks_diff(wk, want)
        assert dq <= 1 and dd <= 1
    r.close()


def test_scores_bit_exact_with_wide_grid():
    """Enough (layer, 64-block) units for a full wave of scoring CTAs: the
    float2 two-blocks-per-lane form (the full-size form) against the oracle."""
    w = synth.Workload("wide", n_layer=16, n_head=4, n_head_kv=2, d_head=64, block_tokens=16,
                       n_blocks=3584, budget_blocks=40, sink_blocks=1, reserve_blocks=4,
                       n_planted=8, seed=91)
    hist = synth.NumpyHistory(w)
    r = kvmret.Retriever(config_for(w))
    append_history(r, hist, cuts=[w.n_tokens // 3])
    q = hist.queries(2)
    for s in range(2):
        q_sum = q[s].reshape(w.n_layer, -1).astype(np.float32)
        q_count = np.ones(w.n_layer, np.uint32)
        q_count[3] = 0  # a layer without a query
        r.query_set(q_sum, q_count)
        got = r.score()
        want, _ = oracle_scores(hist, q_sum, q_count)
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64))
        assert list(r.select()) == list(po.pick_topk(want, w.budget_blocks, w.sink_blocks))
    r.close()
