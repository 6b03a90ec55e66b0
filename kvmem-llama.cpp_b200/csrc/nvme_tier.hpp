// NVMe raw tier: a file arena of fixed-size slots holding whole repository
// blocks, with positional I/O so several host threads may read and write at
// once. Semantics of the reference's NvmeKvTier
// (kvmem/include/kvmem/nvme_kv_tier.hpp:113-430): a slot count of
// total_bytes / slot_bytes (0 disables the tier), a block placed in the
// lowest free slot, least-recently-used eviction by touch order, slot-range
// I/O bounded by the slot, batches of spans whose file offsets and buffer
// ranges are both contiguous merged into one system call, an optional
// page-cache drop after each transfer, O_DIRECT reads when the buffer, the
// offset and the size are aligned (best effort: anything else reads through
// the buffered descriptor), and a backing file whose directory entry is
// removed right after it is opened unless the arena is durable.
#pragma once

#include <cstdint>
#include <list>
#include <mutex>
#include <set>
#include <string>
#include <unordered_map>
#include <vector>

namespace kvmret {

struct NvmeConfig {
    std::string dir;
    std::string file_name = "kvmret_nvme.bin";
    uint64_t total_bytes = 0;
    uint64_t slot_bytes = 0;
    bool durable = false;          // keep the directory entry, do not truncate
    bool direct_read = false;      // open a second O_DIRECT descriptor for reads
    bool drop_page_cache = false;  // POSIX_FADV_DONTNEED after each transfer
};

struct NvmeSpan {
    int32_t slot = -1;
    uint64_t buffer_offset = 0;
    uint64_t bytes = 0;
};

struct NvmeStats {
    uint64_t bytes = 0, syscalls = 0, direct_bytes = 0, cache_drop_bytes = 0,
             cache_drop_failures = 0;
};

class NvmeTier {
public:
    // Throws std::runtime_error when the file cannot be opened.
    explicit NvmeTier(NvmeConfig cfg);
    ~NvmeTier();
    NvmeTier(const NvmeTier &) = delete;
    NvmeTier &operator=(const NvmeTier &) = delete;

    bool enabled() const { return fd_ >= 0 && slot_count_ > 0; }
    uint32_t slot_count() const { return slot_count_; }
    uint64_t slot_bytes() const { return cfg_.slot_bytes; }
    const std::string &path() const { return path_; }
    bool direct_reads() const { return direct_fd_ >= 0; }
    uint32_t free_slots() const;
    int32_t block_slot(uint32_t block) const;

    // The block's slot, or the lowest free one (-1: none). With `evict`, a
    // full arena gives up its least recently used block (*evicted).
    int32_t place(uint32_t block, bool evict, int32_t *evicted);
    void release(uint32_t block);
    void touch(uint32_t block);
    int32_t lru_victim() const;

    // Whole-block transfers (place + write; read of a resident block). Throw
    // std::runtime_error on a bad size, a full arena or a short transfer.
    void write_block(uint32_t block, const void *data, uint64_t bytes, NvmeStats *st = nullptr);
    void read_block(uint32_t block, void *data, uint64_t bytes, NvmeStats *st = nullptr);
    // [offset, offset + bytes) of a slot; throws when it leaves the slot.
    void write_slot_range(int32_t slot, uint64_t offset, const void *data, uint64_t bytes,
                          NvmeStats *st = nullptr);
    void read_slot_range(int32_t slot, uint64_t offset, void *data, uint64_t bytes,
                         NvmeStats *st = nullptr);
    // Spans into one caller buffer of buffer_bytes; adjacent spans coalesce.
    void write_spans(const NvmeSpan *spans, uint32_t n, const void *buffer, uint64_t buffer_bytes,
                     NvmeStats *st = nullptr);
    void read_spans(const NvmeSpan *spans, uint32_t n, void *buffer, uint64_t buffer_bytes,
                    NvmeStats *st = nullptr);

private:
    void check_span(int32_t slot, uint64_t offset, uint64_t bytes) const;
    void io(bool write, uint64_t file_off, uint8_t *buf, uint64_t bytes, NvmeStats *st) const;
    void touch_locked(uint32_t block);

    NvmeConfig cfg_;
    std::string path_;
    int fd_ = -1, direct_fd_ = -1;
    uint32_t slot_count_ = 0;
    mutable std::mutex mu_;
    std::unordered_map<uint32_t, int32_t> slot_of_;
    std::vector<int64_t> block_of_;  // per slot, -1 when free
    std::set<int32_t> free_;
    std::list<uint32_t> lru_;        // front = least recently used
    std::unordered_map<uint32_t, std::list<uint32_t>::iterator> lru_pos_;
};

}  // namespace kvmret
