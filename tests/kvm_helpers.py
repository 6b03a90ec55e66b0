"""Shared helpers of the GPU parity tests."""
import numpy as np

import kvmret
import pyoracle as po


def config_for(w, **kw):
    c = dict(n_layer=w.n_layer, n_head=w.n_head, n_head_kv=w.n_head_kv, d_head=w.d_head,
             block_tokens=w.block_tokens, max_blocks=w.n_blocks, budget_blocks=w.budget_blocks,
             reserve_blocks=w.reserve_blocks, sink_blocks=w.sink_blocks, k_type=w.k_type,
             v_type=w.v_type, n_rot=w.d_head, freq_base=w.freq_base)
    c.update(kw)
    return kvmret.default_config(**c)


def f16_ulp_diff(a_bits, b_bits):
    """Distance in f16 ulps between two arrays of f16 bit patterns."""
    a = np.asarray(a_bits, np.uint16).astype(np.int32)
    b = np.asarray(b_bits, np.uint16).astype(np.int32)
    oa = np.where(a & 0x8000, 0x8000 - a, a)
    ob = np.where(b & 0x8000, 0x8000 - b, b)
    return np.abs(oa - ob)


def q8_blocks_diff(a, b):
    """(max |qs| LSB difference, max scale ulp difference) between q8_0 byte arrays."""
    a = np.asarray(a, np.uint8).reshape(-1, 34)
    b = np.asarray(b, np.uint8).reshape(-1, 34)
    da = a[:, :2].copy().view(np.uint16).reshape(-1)
    db = b[:, :2].copy().view(np.uint16).reshape(-1)
    qa = a[:, 2:].view(np.int8).astype(np.int32)
    qb = b[:, 2:].view(np.int8).astype(np.int32)
    return int(np.abs(qa - qb).max(initial=0)), int(f16_ulp_diff(da, db).max(initial=0))


def q4_blocks_diff(a, b):
    """(max nibble difference, max scale ulp difference) between q4_0 byte arrays."""
    a = np.asarray(a, np.uint8).reshape(-1, 18)
    b = np.asarray(b, np.uint8).reshape(-1, 18)
    da = a[:, :2].copy().view(np.uint16).reshape(-1)
    db = b[:, :2].copy().view(np.uint16).reshape(-1)
    qa = np.concatenate([a[:, 2:] & 15, a[:, 2:] >> 4], 1).astype(np.int32)
    qb = np.concatenate([b[:, 2:] & 15, b[:, 2:] >> 4], 1).astype(np.int32)
    return int(np.abs(qa - qb).max(initial=0)), int(f16_ulp_diff(da, db).max(initial=0))


def history_units(hist):
    """K/V of a NumpyHistory as [N][L][T][E] f16 (block, layer) units."""
    w = hist.w
    L, N, T, E = w.n_layer, w.n_blocks, w.block_tokens, w.E
    k = hist.k.reshape(L, N, T, E).transpose(1, 0, 2, 3)
    v = hist.v.reshape(L, N, T, E).transpose(1, 0, 2, 3)
    return k, v


def append_history(r, hist, cuts, k_rows_fn=None, v_rows_fn=None, start=0, stop=None):
    """Append tokens [start, stop) of the history (default: all) to a Retriever in
    chunks ending at token offsets `cuts`."""
    import torch
    w = hist.w
    L, n, E = w.n_layer, w.n_tokens, w.E
    k = hist.k.reshape(L, n, E)
    v = hist.v.reshape(L, n, E)
    t0 = start
    stop = n if stop is None else stop
    for t1 in [c for c in cuts if c < stop] + [stop]:
        if t1 <= t0:
            continue
        kc = torch.from_numpy(np.ascontiguousarray(k[:, t0:t1])).cuda()
        if v_rows_fn is None:
            vr = torch.from_numpy(np.ascontiguousarray(v[:, t0:t1])).cuda()
        else:
            vr = torch.from_numpy(np.ascontiguousarray(v_rows_fn(v[:, t0:t1]))).cuda()
        kr = None
        if k_rows_fn is not None:
            kr = torch.from_numpy(np.ascontiguousarray(k_rows_fn(k[:, t0:t1]))).cuda()
        r.append(kc, vr, k_rows=kr, pos0=t0)
        t0 = t1
    r.sync()


def oracle_scores(hist, q_sum, q_count, n_blocks=None):
    w = hist.w
    k, _ = history_units(hist)
    N = w.n_blocks if n_blocks is None else n_blocks
    mean = po.mean_k(k[:N].reshape(N * w.n_layer, w.block_tokens, w.E)).reshape(
        N, w.n_layer, w.E)
    has = np.ones(N, np.uint8)
    return po.score(mean, has, q_sum, q_count, w.n_head, w.n_head_kv, w.d_head), mean


def oracle_mean_tokens(hist, n_tok):
    """Summaries [N][L][E] of the first n_tok tokens (a partial last block)."""
    w = hist.w
    T, L, E = w.block_tokens, w.n_layer, w.E
    k = hist.k.reshape(L, w.n_tokens, E)[:, :n_tok]
    nb = (n_tok + T - 1) // T
    out = np.zeros((nb, L, E), np.float32)
    for b in range(nb):
        t1 = min(n_tok, (b + 1) * T)
        out[b] = po.mean_k(np.ascontiguousarray(k[:, b * T:t1]))
    return out


def oracle_ids_tokens(hist, n_tok, q, gen_first=None):
    """Top-k over the blocks before the decode blocks, plus the decode blocks."""
    w = hist.w
    mean = oracle_mean_tokens(hist, n_tok)
    nb = mean.shape[0]
    scores = po.score(mean, np.ones(nb, np.uint8), q.reshape(w.n_layer, -1).astype(np.float32),
                      np.ones(w.n_layer, np.uint32), w.n_head, w.n_head_kv, w.d_head)
    g0 = nb if gen_first is None else min(gen_first, nb)
    ids = po.pick_topk(scores[:g0], w.budget_blocks, w.sink_blocks)
    return sorted(set(ids.tolist()) | set(range(g0, nb)))


def check_window(r, hist, n_tok, want_ids, quant=False):
    """Layout chronological with running-sum bases; every slot's K and V
    against the oracle from the stored rows."""
    w = hist.w
    T, L = w.block_tokens, w.n_layer
    ids, bases = r.window_layout()
    assert list(ids) == list(want_ids)
    ntok = [min(T, n_tok - b * T) for b in want_ids]
    assert list(bases) == [int(x) for x in np.concatenate([[0], np.cumsum(ntok)[:-1]])]
    repo = r.repo_view()
    unit = int(kvmret.lib.kvmret_repo_unit_bytes(r.h))
    kb = int(kvmret.lib.kvmret_repo_k_bytes(r.h))
    for i, (b, base, n) in enumerate(zip(ids, bases, ntok)):
        for l in range(L):
            o = (int(b) * L + l) * unit
            src_k = np.array(repo[o:o + n * r.k_row])
            src_v = np.array(repo[o + kb:o + kb + n * r.v_row])
            wk = r.window_read(l, False, i, 1)[:n * r.k_row]
            wv = r.window_read(l, True, i, 1)[:n * r.v_row]
            assert np.array_equal(wv, src_v), (i, int(b), l)
            if quant:
                want = po.rope_block_q8_0(src_k, n, w.n_head_kv, w.d_head, int(base),
                                          w.freq_base, fwht_n=w.d_head)
                assert q8_blocks_diff(wk, want) <= (1, 1), (i, int(b), l)
            else:
                want = po.rope_block_f16(src_k.view(np.uint16).reshape(n, w.n_head_kv, w.d_head),
                                         int(base), w.freq_base)
                assert f16_ulp_diff(wk.view(np.uint16), want.reshape(-1)).max() <= 2, (i, int(b))
    return ids
