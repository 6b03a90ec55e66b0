"""The snapshot archive's layout, on the CPU, pinned to the reference's own
writer: RawKvStore::snapshot_write through SnapshotWriter
(kvmem/src/host/raw_kv_store.cpp:1225-1250, kvmem/include/kvmem/snapshot.hpp)
run by the reference library built from its sources. The archive of a store
filled the way this library stores a conversation (unrotated K rows with
their f32 sums, packed V rows) parses field by field as the C ABI documents
it, and its hash is the 64-bit FNV-1a of its bytes."""
import numpy as np
import pytest

import pyoracle as po

needs_ref = pytest.mark.skipif(po.ref is None, reason="oracle/_ref not built")


def fnv1a(b):
    h = 14695981039346656037
    for x in bytes(b):
        h = ((h ^ x) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


class Reader:
    def __init__(self, b):
        self.b, self.o = bytes(b), 0

    def take(self, n):
        v = self.b[self.o:self.o + n]
        assert len(v) == n
        self.o += n
        return v

    def u(self, n):
        return int.from_bytes(self.take(n), "little")

    def vec(self, itemsize):
        n = self.u(8)
        return n, self.take(n * itemsize)


@needs_ref
@pytest.mark.parametrize("n_tok", [8, 11, 3])
def test_reference_archive_layout(n_tok):
    L, E, T, vrow = 2, 8, 4, 16
    rng = np.random.default_rng(n_tok)
    k = rng.standard_normal((L, n_tok, E)).astype(np.float16)
    v = rng.integers(0, 255, size=(L, n_tok, vrow), dtype=np.uint8)
    arc, h = po.ref_snapshot_rows(L, E, T, 0, vrow, k.view(np.uint8).reshape(L, n_tok, 2 * E),
                                  k.astype(np.float32), v)
    assert h == fnv1a(arc)
    r = Reader(arc)
    assert r.u(4) == 0x31564B52
    assert [r.u(4) for _ in range(4)] == [L, E, E, T]
    assert [r.u(8) for _ in range(3)] == [0, 0, vrow]
    nb = r.u(8)
    assert nb == (n_tok + T - 1) // T
    for b in range(nb):
        size = r.u(8)
        start = r.o
        n = min(T, n_tok - b * T)
        for l in range(L):
            assert [r.u(4) for _ in range(4)] == [n, 0, n, n]
            assert (r.u(1), r.u(1)) == (0, 1)
            cnt, kb = r.vec(1)
            assert cnt == T * 2 * E
            assert kb[:n * 2 * E] == k[l, b * T:b * T + n].tobytes()
            assert kb[n * 2 * E:] == bytes(cnt - n * 2 * E)
            assert r.vec(2)[0] == 0 and r.vec(1)[0] == 0
            cnt, vb = r.vec(1)
            assert cnt == T * vrow and vb[:n * vrow] == v[l, b * T:b * T + n].tobytes()
            cnt, ks = r.vec(4)
            want = np.zeros(E, np.float32)
            for t in range(n):  # token-order f32 sum
                want = (want + k[l, b * T + t].astype(np.float32)).astype(np.float32)
            assert cnt == E and ks == want.tobytes()
        assert r.o - start == size
    assert r.o == len(arc)
