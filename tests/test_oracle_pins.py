"""Pin the CPU oracle before trusting it.

(1) Known answers of the reference's own unit tests for this path
    (kvmem/tests/kvmem_store_test.cpp, raw_kv_store_test.cpp), restated as
    vectors. (2) The oracle against the reference's libkvmem compiled from its
    sources into oracle/_ref (selection, plan, mean-K, RoPE), on seeded random
    cases including ties, mandatory lists and partial blocks.
"""
import numpy as np
import pytest

import pyoracle as po

needs_ref = pytest.mark.skipif(po.ref is None, reason="oracle/_ref not built (reference absent)")


# ---------------------------------------------------------------------------
# (1) reference unit-test known answers
def test_topk_budget_sink_recent_known_answer():
    # kvmem_store_test.cpp:284-314: budget 4, sink 1, recent 1; hottest 5, 6.
    s = np.zeros(10)
    s[5], s[6], s[3] = 100.0, 90.0, 10.0
    assert list(po.pick_topk(s, 4, sink=1, recent=1)) == [0, 5, 6, 9]


def test_topk_zero_recent_known_answer():
    # kvmem_store_test.cpp:316-339: recent 0 keeps no suffix.
    s = np.zeros(10)
    s[3], s[5], s[6], s[9] = 80.0, 100.0, 90.0, -100.0
    assert list(po.pick_topk(s, 4, sink=1, recent=0)) == [0, 3, 5, 6]


def test_topk_mandatory_inside_budget_known_answer():
    # kvmem_store_test.cpp:433-458.
    s = np.zeros(10)
    s[2], s[3], s[4], s[8], s[9] = 100.0, 90.0, 80.0, -10.0, -20.0
    assert list(po.pick_topk(s, 4, sink=1, recent=0, mandatory=[8, 9])) == [0, 2, 8, 9]


def test_mandatory_dedup_recent_best_effort_known_answer():
    # kvmem_store_test.cpp:460-477: sink 2, recent 3, mandatory {0, 0, 5}.
    assert list(po.pick_topk(np.zeros(10), 4, sink=2, recent=3, mandatory=[0, 0, 5])) == [
        0, 1, 5, 9]


def test_mandatory_overflow_trims_newest_known_answer():
    # kvmem_store_test.cpp:479-504: sink 1 + mandatory {1..4} over budget 4.
    assert list(po.pick_topk(np.zeros(10), 4, sink=1, recent=2, mandatory=[1, 2, 3, 4])) == [
        0, 2, 3, 4]


def test_topk_all_fit_and_empty_known_answer():
    # kvmem_store_test.cpp:763-781.
    assert list(po.pick_topk(np.zeros(3), 100)) == [0, 1, 2]
    assert list(po.pick_topk(np.zeros(0), 4)) == []


def test_selection_diff_and_remap_known_answer():
    # kvmem_store_test.cpp:53-110.
    s = po.Store(128)
    s.append(128 * 5)
    si, so, rm, c = s.set_selection([4, 0, 2])
    assert list(si) == [0, 2, 4] and list(so) == [1, 3]
    assert c[3] == 128 * 3
    assert [tuple(r[[0, 2, 3, 5]]) for r in rm] == [(0, 0, 0, 1), (2, 256, 128, 0),
                                                     (4, 512, 256, 0)]
    si, so, rm, c = s.set_selection([0, 2, 3])
    assert list(si) == [3] and list(so) == [4]
    assert [tuple(r[[0, 2, 3, 5]]) for r in rm] == [(0, 0, 0, 1), (2, 128, 128, 1),
                                                     (3, 384, 256, 0)]


def test_mean_k_ordered_f32_sum():
    # raw_kv_store_test.cpp:24-94: mean-K is the ordered F32 sum times 1/n.
    rng = np.random.default_rng(5)
    k = rng.standard_normal((3, 77, 64)).astype(np.float16)
    got = po.mean_k(k)
    for u in range(3):
        acc = np.zeros(64, np.float32)
        for t in range(77):
            acc = (acc + k[u, t].astype(np.float32)).astype(np.float32)
        want = acc * np.float32(np.float32(1.0) / np.float32(77))
        assert np.array_equal(got[u].view(np.uint32), want.astype(np.float32).view(np.uint32))


def test_rope_identity_at_pos0():
    # raw_kv_store_test.cpp:239-254: RoPE at position 0 is the identity.
    rng = np.random.default_rng(6)
    k = rng.standard_normal((1, 8, 128)).astype(np.float32)
    assert np.array_equal(po.rope_neox(k, 0, 1e6), k)


# ---------------------------------------------------------------------------
# (2) oracle == reference libkvmem
@needs_ref
@pytest.mark.parametrize("seed", range(40))
def test_pick_topk_matches_reference(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 600))
    budget = int(rng.integers(1, 80))
    sink = int(rng.integers(0, 4))
    recent = int(rng.integers(0, 4))
    scores = rng.standard_normal(n)
    if seed % 3 == 0:  # heavy ties
        scores = np.round(scores * 2) / 2
    if seed % 5 == 0:
        scores[:] = 0.0
    mand = rng.integers(0, n, size=int(rng.integers(0, 6)))
    got = po.pick_topk(scores, budget, sink, recent, mand, tie_higher_id=True)
    want = po.ref_pick_topk(scores, budget, sink, recent, mand)
    assert list(got) == list(want)


@needs_ref
@pytest.mark.parametrize("immutable", [False, True])
@pytest.mark.parametrize("seed", range(8))
def test_set_selection_matches_reference(seed, immutable):
    rng = np.random.default_rng(100 + seed)
    bt = 32
    o = po.Store(bt, immutable)
    r = po.RefRuntime(bt, 1 << 20, 1, immutable)
    n_tok = int(rng.integers(bt, bt * 60))
    o.append(n_tok)
    r.append(n_tok)
    nb = (n_tok + bt - 1) // bt
    for step in range(12):
        if rng.random() < 0.2:
            extra = int(rng.integers(1, 3 * bt))
            o.append(extra)
            r.append(extra)
            n_tok += extra
            nb = (n_tok + bt - 1) // bt
        k = int(rng.integers(0, nb + 1))
        ids = rng.choice(nb + 2, size=k, replace=True)  # stale / duplicate ids included
        force = bool(rng.random() < 0.1)
        a = o.set_selection(ids, force)
        b = r.set_selection(ids, force)
        for x, y in zip(a, b):
            assert np.array_equal(x, y), (step, x, y)


@needs_ref
def test_mean_k_matches_reference():
    rng = np.random.default_rng(7)
    for n in (1, 5, 128):
        k = rng.standard_normal((1, n, 1024)).astype(np.float16)
        got = po.mean_k(k)[0]
        want = np.zeros(1024, np.float32)
        kf = np.ascontiguousarray(k[0].astype(np.float32))
        po.ref.ref_mean_k_f32(kf.ctypes.data_as(po._PF), n, 1024, 128,
                              want.ctypes.data_as(po._PF))
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@needs_ref
@pytest.mark.parametrize("pos0", [0, 1, 127, 4096, 32768, 49151, 262143])
def test_rope_matches_reference(pos0):
    rng = np.random.default_rng(pos0)
    k = rng.standard_normal((16, 8, 128)).astype(np.float32)
    assert np.array_equal(po.rope_neox(k, pos0, 1e6), po.ref_rope_neox(k, pos0, 1e6))


# ---------------------------------------------------------------------------
# internal consistency of the restated kernels
def test_fwht_matches_hadamard_matrix():
    rng = np.random.default_rng(8)
    x = rng.standard_normal((32, 8 * 128)).astype(np.float32)
    a = po.fwht(x, 128)
    b = po.hadamard_rows(x, 8, 128, 128)
    np.testing.assert_allclose(a, b.reshape(-1), rtol=1e-5, atol=1e-5)
    # H is its own inverse
    np.testing.assert_allclose(po.fwht(a, 128), x.reshape(-1), rtol=1e-4, atol=1e-5)


def test_q8_q4_round_trip_error_bounds():
    rng = np.random.default_rng(9)
    x = rng.standard_normal(32 * 64).astype(np.float32)
    y8 = po.dequant_q8_0(po.quant_q8_0(x))
    # the scale is stored as f16: |err| <= d/2 + 127 * |d - f16(d)| <= 0.6 d
    d8 = np.abs(x.reshape(-1, 32)).max(1, keepdims=True) / 127
    assert np.all(np.abs(y8.reshape(-1, 32) - x.reshape(-1, 32)) <= d8 * 0.6)
    y4 = po.dequant_q4_0(po.quant_q4_0(x))
    d4 = np.abs(x.reshape(-1, 32)).max(1, keepdims=True) / 8
    assert np.all(np.abs(y4.reshape(-1, 32) - x.reshape(-1, 32)) <= d4 * 1.01)
