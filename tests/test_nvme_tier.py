"""The NVMe raw tier through the C ABI, on the CPU, with the known answers of
the reference's own tier test (kvmem/tests/nvme_kv_tier_test.cpp): slot
sizing and the disabled tier, lowest-slot placement, write / read / rewrite /
release, a backing file without a directory entry, slot ranges bounded by
their slot, least-recently-used eviction by touch order, coalesced span
batches (one system call for contiguous spans, page-cache drop accounting),
concurrent positional batches from two threads."""
import os
import threading

import numpy as np
import pytest

import kvmret


def test_disabled(tmp_path):
    t = kvmret.Nvme(str(tmp_path), total_bytes=0, slot_bytes=64)
    assert not t.enabled and t.slot_count == 0


def test_write_read_release(tmp_path):
    t = kvmret.Nvme(str(tmp_path), total_bytes=256, slot_bytes=64, drop_page_cache=True)
    assert t.enabled and t.slot_count == 4
    # the descriptor stays usable; the file has no directory entry
    assert not os.path.exists(t.path)
    a = np.arange(64, dtype=np.uint8)
    b = (255 - np.arange(64)).astype(np.uint8)
    t.write_block(10, a)
    assert t.block_slot(10) == 0
    assert np.array_equal(t.read_block(10, 64), a)
    t.write_block(10, b)
    assert np.array_equal(t.read_block(10, 64), b)
    t.release(10)
    assert t.block_slot(10) == -1 and t.free_slots == 4


def test_slot_ranges_and_file_names(tmp_path):
    t = kvmret.Nvme(str(tmp_path), total_bytes=256, slot_bytes=128,
                    file_name="kvmret_range_test.bin")
    assert "kvmret_range_test.bin" in t.path and not os.path.exists(t.path)
    slot, ev = t.place(7)
    assert slot == 0 and ev == -1
    main = np.full(80, 0x31, np.uint8)
    mtp = np.full(24, 0x92, np.uint8)
    t.write_range(slot, 0, main)
    t.write_range(slot, 96, mtp)
    assert np.array_equal(t.read_range(slot, 0, 80), main)
    assert np.array_equal(t.read_range(slot, 96, 24), mtp)
    with pytest.raises(kvmret.KvmretError, match="leaves its slot"):
        t.read_range(slot, 120, 24)


def test_evicting_place(tmp_path):
    t = kvmret.Nvme(str(tmp_path), total_bytes=128, slot_bytes=64)
    t.write_block(1, np.full(64, 1, np.uint8))
    t.write_block(2, np.full(64, 2, np.uint8))
    t.touch(1)  # block 2 becomes the least recently used
    assert t.lru_victim() == 2
    assert t.place(3) == (-1, -1)  # full, no eviction asked
    slot, ev = t.place(3, evict=True)
    assert (slot, ev) == (1, 2)
    assert t.block_slot(2) == -1 and t.block_slot(3) == 1
    c = np.full(64, 3, np.uint8)
    t.write_block(3, c)
    assert np.array_equal(t.read_block(3, 64), c)
    with pytest.raises(kvmret.KvmretError, match="not resident"):
        t.read_block(2, 64)


def test_coalesced_batch_io(tmp_path):
    t = kvmret.Nvme(str(tmp_path), total_bytes=64 * 8, slot_bytes=64, drop_page_cache=True)
    inp = ((np.arange(64 * 3) * 17) & 0xFF).astype(np.uint8)
    spans = []
    for block in range(3):
        slot, _ = t.place(100 + block)
        assert slot == block
        spans.append((slot, block * 64, 64))
    w = t.write_spans(spans, inp)
    assert w["bytes"] == inp.size and w["syscalls"] == 1
    assert w["cache_drop_bytes"] == inp.size and w["cache_drop_failures"] == 0
    out = np.zeros_like(inp)
    r = t.read_spans(spans, out)
    assert r["bytes"] == out.size and r["syscalls"] == 1
    assert r["cache_drop_bytes"] == out.size and r["cache_drop_failures"] == 0
    assert np.array_equal(out, inp)
    # spans that are not contiguous in the buffer do not merge
    r2 = t.read_spans([(0, 0, 64), (1, 128, 64)], np.zeros(192, np.uint8))
    assert r2["syscalls"] == 2


def test_concurrent_positional_batches(tmp_path):
    t = kvmret.Nvme(str(tmp_path), total_bytes=64 * 8, slot_bytes=64)
    a = np.full(64 * 3, 0x35, np.uint8)
    b = np.full(64 * 3, 0xCA, np.uint8)
    a_spans, b_spans = [], []
    for block in range(6):
        slot, _ = t.place(200 + block)
        assert slot == block
        (a_spans if block < 3 else b_spans).append((slot, (block % 3) * 64, 64))
    ths = [threading.Thread(target=t.write_spans, args=(a_spans, a)),
           threading.Thread(target=t.write_spans, args=(b_spans, b))]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    out = np.zeros(64 * 6, np.uint8)
    r = t.read_spans([(s, s * 64, 64) for s in range(6)], out)
    assert r["syscalls"] == 1
    assert np.array_equal(out[:192], a) and np.array_equal(out[192:], b)


def test_direct_reads_fall_back_or_align(tmp_path):
    """O_DIRECT reads need 4096-aligned buffers, offsets and sizes; any other
    read goes through the buffered descriptor with the same result."""
    t = kvmret.Nvme(str(tmp_path), total_bytes=4096 * 4, slot_bytes=4096, durable=True,
                    direct_read=True)
    data = (np.arange(4096 * 2) % 251).astype(np.uint8)
    t.write_spans([(0, 0, 4096), (1, 4096, 4096)], data)
    buf = np.zeros(4096 * 3, np.uint8)
    off = (-buf.ctypes.data) % 4096  # an aligned window of the buffer
    view = buf[off:off + 8192]
    r = t.read_spans([(0, 0, 4096), (1, 4096, 4096)], view)
    assert np.array_equal(view, data)
    if t.direct_reads:
        assert r["direct_bytes"] == 8192
    odd = np.zeros(100, np.uint8)
    t.read_spans([(0, 0, 100)], odd)
    assert np.array_equal(odd, data[:100])
    assert os.path.exists(t.path)  # durable: the file keeps its name
