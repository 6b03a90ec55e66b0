#include "nvme_tier.hpp"

#include <fcntl.h>
#include <sys/stat.h>
#include <sys/types.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <stdexcept>

namespace kvmret {

namespace {

constexpr uint64_t kDirectAlign = 4096;

void make_dirs(const std::string &dir) {
    std::string cur;
    for (size_t i = 0; i <= dir.size(); ++i) {
        if (i == dir.size() || dir[i] == '/') {
            if (!cur.empty() && ::mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST)
                throw std::runtime_error("cannot create directory " + cur + ": " +
                                         std::strerror(errno));
        }
        if (i < dir.size()) cur.push_back(dir[i]);
    }
}

}  // namespace

NvmeTier::NvmeTier(NvmeConfig cfg) : cfg_(std::move(cfg)) {
    if (cfg_.slot_bytes > 0 && cfg_.total_bytes >= cfg_.slot_bytes)
        slot_count_ = static_cast<uint32_t>(cfg_.total_bytes / cfg_.slot_bytes);
    if (slot_count_ == 0 || cfg_.dir.empty()) {
        slot_count_ = 0;
        return;
    }
    if (cfg_.file_name.empty() || cfg_.file_name.find('/') != std::string::npos)
        throw std::runtime_error("NVMe tier file name must be a non-empty base name");
    make_dirs(cfg_.dir);
    path_ = cfg_.dir + "/" + cfg_.file_name;
    fd_ = ::open(path_.c_str(), O_CREAT | O_RDWR | O_CLOEXEC | (cfg_.durable ? 0 : O_TRUNC), 0644);
    if (fd_ < 0)
        throw std::runtime_error("cannot open NVMe tier file " + path_ + ": " +
                                 std::strerror(errno));
    if (cfg_.direct_read) {
#ifdef O_DIRECT
        direct_fd_ = ::open(path_.c_str(), O_RDONLY | O_CLOEXEC | O_DIRECT);
#endif
        // a file system without O_DIRECT keeps the buffered descriptor only
    }
    if (!cfg_.durable) ::unlink(path_.c_str());  // the arena dies with the process
    block_of_.assign(slot_count_, -1);
    for (uint32_t s = 0; s < slot_count_; ++s) free_.insert(static_cast<int32_t>(s));
}

NvmeTier::~NvmeTier() {
    if (direct_fd_ >= 0) ::close(direct_fd_);
    if (fd_ >= 0) ::close(fd_);
}

uint32_t NvmeTier::free_slots() const {
    std::lock_guard<std::mutex> lk(mu_);
    return static_cast<uint32_t>(free_.size());
}

int32_t NvmeTier::block_slot(uint32_t block) const {
    std::lock_guard<std::mutex> lk(mu_);
    const auto it = slot_of_.find(block);
    return it == slot_of_.end() ? -1 : it->second;
}

void NvmeTier::touch_locked(uint32_t block) {
    const auto it = lru_pos_.find(block);
    if (it != lru_pos_.end()) lru_.erase(it->second);
    lru_.push_back(block);
    lru_pos_[block] = std::prev(lru_.end());
}

void NvmeTier::touch(uint32_t block) {
    std::lock_guard<std::mutex> lk(mu_);
    if (slot_of_.count(block)) touch_locked(block);
}

int32_t NvmeTier::lru_victim() const {
    std::lock_guard<std::mutex> lk(mu_);
    return lru_.empty() ? -1 : static_cast<int32_t>(lru_.front());
}

int32_t NvmeTier::place(uint32_t block, bool evict, int32_t *evicted) {
    std::lock_guard<std::mutex> lk(mu_);
    if (evicted) *evicted = -1;
    if (!enabled()) return -1;
    const auto it = slot_of_.find(block);
    if (it != slot_of_.end()) return it->second;
    int32_t slot = -1;
    if (!free_.empty()) {
        slot = *free_.begin();
        free_.erase(free_.begin());
    } else if (evict && !lru_.empty()) {
        const uint32_t victim = lru_.front();
        lru_.pop_front();
        lru_pos_.erase(victim);
        slot = slot_of_[victim];
        slot_of_.erase(victim);
        if (evicted) *evicted = static_cast<int32_t>(victim);
    } else {
        return -1;
    }
    slot_of_[block] = slot;
    block_of_[slot] = block;
    touch_locked(block);
    return slot;
}

void NvmeTier::release(uint32_t block) {
    std::lock_guard<std::mutex> lk(mu_);
    const auto it = slot_of_.find(block);
    if (it == slot_of_.end()) return;
    free_.insert(it->second);
    block_of_[it->second] = -1;
    slot_of_.erase(it);
    const auto lp = lru_pos_.find(block);
    if (lp != lru_pos_.end()) {
        lru_.erase(lp->second);
        lru_pos_.erase(lp);
    }
}

void NvmeTier::check_span(int32_t slot, uint64_t offset, uint64_t bytes) const {
    if (!enabled()) throw std::runtime_error("NVMe tier is disabled");
    if (slot < 0 || static_cast<uint32_t>(slot) >= slot_count_)
        throw std::runtime_error("NVMe slot out of range");
    if (offset > cfg_.slot_bytes || bytes > cfg_.slot_bytes - offset)
        throw std::runtime_error("NVMe transfer leaves its slot");
}

void NvmeTier::io(bool write, uint64_t file_off, uint8_t *buf, uint64_t bytes,
                  NvmeStats *st) const {
    const bool direct = !write && direct_fd_ >= 0 && file_off % kDirectAlign == 0 &&
                        bytes % kDirectAlign == 0 &&
                        reinterpret_cast<uintptr_t>(buf) % kDirectAlign == 0;
    const int fd = direct ? direct_fd_ : fd_;
    uint64_t done = 0;
    while (done < bytes) {
        const ssize_t r = write ? ::pwrite(fd, buf + done, bytes - done,
                                           static_cast<off_t>(file_off + done))
                                : ::pread(fd, buf + done, bytes - done,
                                          static_cast<off_t>(file_off + done));
        if (st) ++st->syscalls;
        if (r < 0) {
            if (errno == EINTR) continue;
            throw std::runtime_error(std::string("NVMe ") + (write ? "write" : "read") +
                                     " failed: " + std::strerror(errno));
        }
        if (r == 0) throw std::runtime_error("NVMe read past the end of the arena");
        done += static_cast<uint64_t>(r);
    }
    if (st) {
        st->bytes += bytes;
        if (direct) st->direct_bytes += bytes;
    }
    if (cfg_.drop_page_cache && !direct) {
#ifdef POSIX_FADV_DONTNEED
        if (write) ::fdatasync(fd_);
        const int rc = ::posix_fadvise(fd_, static_cast<off_t>(file_off),
                                       static_cast<off_t>(bytes), POSIX_FADV_DONTNEED);
        if (st) {
            if (rc == 0) st->cache_drop_bytes += bytes;
            else ++st->cache_drop_failures;
        }
#endif
    }
}

void NvmeTier::write_slot_range(int32_t slot, uint64_t offset, const void *data, uint64_t bytes,
                                NvmeStats *st) {
    check_span(slot, offset, bytes);
    io(true, static_cast<uint64_t>(slot) * cfg_.slot_bytes + offset,
       const_cast<uint8_t *>(static_cast<const uint8_t *>(data)), bytes, st);
}

void NvmeTier::read_slot_range(int32_t slot, uint64_t offset, void *data, uint64_t bytes,
                               NvmeStats *st) {
    check_span(slot, offset, bytes);
    io(false, static_cast<uint64_t>(slot) * cfg_.slot_bytes + offset,
       static_cast<uint8_t *>(data), bytes, st);
}

void NvmeTier::write_block(uint32_t block, const void *data, uint64_t bytes, NvmeStats *st) {
    if (!data || bytes == 0 || bytes > cfg_.slot_bytes)
        throw std::runtime_error("NVMe block write of a bad size");
    const int32_t slot = place(block, false, nullptr);
    if (slot < 0) throw std::runtime_error("NVMe tier is full");
    write_slot_range(slot, 0, data, bytes, st);
    touch(block);
}

void NvmeTier::read_block(uint32_t block, void *data, uint64_t bytes, NvmeStats *st) {
    if (!data || bytes == 0 || bytes > cfg_.slot_bytes)
        throw std::runtime_error("NVMe block read of a bad size");
    const int32_t slot = block_slot(block);
    if (slot < 0) throw std::runtime_error("NVMe block is not resident");
    read_slot_range(slot, 0, data, bytes, st);
    touch(block);
}

namespace {
// Runs of spans that are contiguous both in the file and in the buffer.
template <typename Fn>
void coalesce(const NvmeSpan *spans, uint32_t n, uint64_t slot_bytes, Fn fn) {
    uint32_t i = 0;
    while (i < n) {
        uint64_t off = static_cast<uint64_t>(spans[i].slot) * slot_bytes;
        uint64_t buf = spans[i].buffer_offset, len = spans[i].bytes;
        uint32_t j = i + 1;
        while (j < n && static_cast<uint64_t>(spans[j].slot) * slot_bytes == off + len &&
               spans[j].buffer_offset == buf + len && spans[j - 1].bytes == slot_bytes) {
            len += spans[j].bytes;
            ++j;
        }
        fn(off, buf, len);
        i = j;
    }
}
}  // namespace

void NvmeTier::write_spans(const NvmeSpan *spans, uint32_t n, const void *buffer,
                           uint64_t buffer_bytes, NvmeStats *st) {
    for (uint32_t i = 0; i < n; ++i) {
        check_span(spans[i].slot, 0, spans[i].bytes);
        if (spans[i].buffer_offset > buffer_bytes ||
            spans[i].bytes > buffer_bytes - spans[i].buffer_offset)
            throw std::runtime_error("NVMe span leaves its buffer");
    }
    uint8_t *b = const_cast<uint8_t *>(static_cast<const uint8_t *>(buffer));
    coalesce(spans, n, cfg_.slot_bytes,
             [&](uint64_t off, uint64_t bo, uint64_t len) { io(true, off, b + bo, len, st); });
}

void NvmeTier::read_spans(const NvmeSpan *spans, uint32_t n, void *buffer, uint64_t buffer_bytes,
                          NvmeStats *st) {
    for (uint32_t i = 0; i < n; ++i) {
        check_span(spans[i].slot, 0, spans[i].bytes);
        if (spans[i].buffer_offset > buffer_bytes ||
            spans[i].bytes > buffer_bytes - spans[i].buffer_offset)
            throw std::runtime_error("NVMe span leaves its buffer");
    }
    uint8_t *b = static_cast<uint8_t *>(buffer);
    coalesce(spans, n, cfg_.slot_bytes,
             [&](uint64_t off, uint64_t bo, uint64_t len) { io(false, off, b + bo, len, st); });
}

}  // namespace kvmret

// ---------------------------------------------------------------------------
// C ABI (include/kvmret.h): the tier on its own. No exception crosses it.
#include "kvmret.h"

namespace kvmret {
int set_error(int code, const char *msg);  // context.cpp: feeds kvmret_last_error()
}

struct kvmret_nvme {
    kvmret::NvmeTier tier;
    explicit kvmret_nvme(kvmret::NvmeConfig c) : tier(std::move(c)) {}
};

namespace {
int nvme_fail(const std::exception &e) { return kvmret::set_error(KVMRET_ERR_STATE, e.what()); }
void to_stats(const kvmret::NvmeStats &s, kvmret_nvme_stats *out) {
    if (!out) return;
    out->bytes = s.bytes;
    out->syscalls = s.syscalls;
    out->direct_bytes = s.direct_bytes;
    out->cache_drop_bytes = s.cache_drop_bytes;
    out->cache_drop_failures = s.cache_drop_failures;
}
}  // namespace

extern "C" {

int kvmret_nvme_create(const kvmret_nvme_config *cfg, kvmret_nvme **out) {
    if (!cfg || !out || !cfg->dir) return kvmret::set_error(KVMRET_ERR_ARG, "null argument");
    *out = nullptr;
    kvmret::NvmeConfig c;
    c.dir = cfg->dir;
    if (cfg->file_name) c.file_name = cfg->file_name;
    c.total_bytes = cfg->total_bytes;
    c.slot_bytes = cfg->slot_bytes;
    c.durable = cfg->durable != 0;
    c.direct_read = cfg->direct_read != 0;
    c.drop_page_cache = cfg->drop_page_cache != 0;
    try {
        *out = new kvmret_nvme(std::move(c));
    } catch (const std::exception &e) {
        return nvme_fail(e);
    }
    return KVMRET_OK;
}

void kvmret_nvme_destroy(kvmret_nvme *t) { delete t; }
uint32_t kvmret_nvme_slot_count(kvmret_nvme *t) { return t ? t->tier.slot_count() : 0; }
uint32_t kvmret_nvme_free_slots(kvmret_nvme *t) { return t ? t->tier.free_slots() : 0; }
int kvmret_nvme_direct_reads(kvmret_nvme *t) { return t && t->tier.direct_reads() ? 1 : 0; }
int32_t kvmret_nvme_block_slot(kvmret_nvme *t, uint32_t block) {
    return t ? t->tier.block_slot(block) : -1;
}
int32_t kvmret_nvme_lru_victim(kvmret_nvme *t) { return t ? t->tier.lru_victim() : -1; }

int kvmret_nvme_path(kvmret_nvme *t, char *out, uint32_t cap) {
    if (!t || !out || cap == 0) return kvmret::set_error(KVMRET_ERR_ARG, "null argument");
    const std::string &p = t->tier.path();
    const size_t n = std::min<size_t>(p.size(), cap - 1);
    std::memcpy(out, p.data(), n);
    out[n] = 0;
    return KVMRET_OK;
}

int32_t kvmret_nvme_place(kvmret_nvme *t, uint32_t block, int evict, int32_t *evicted) {
    if (!t) return -1;
    return t->tier.place(block, evict != 0, evicted);
}

int kvmret_nvme_release(kvmret_nvme *t, uint32_t block) {
    if (!t) return kvmret::set_error(KVMRET_ERR_ARG, "null tier");
    t->tier.release(block);
    return KVMRET_OK;
}

int kvmret_nvme_touch(kvmret_nvme *t, uint32_t block) {
    if (!t) return kvmret::set_error(KVMRET_ERR_ARG, "null tier");
    t->tier.touch(block);
    return KVMRET_OK;
}

int kvmret_nvme_write_block(kvmret_nvme *t, uint32_t block, const void *data, uint64_t bytes) {
    if (!t) return kvmret::set_error(KVMRET_ERR_ARG, "null tier");
    try {
        t->tier.write_block(block, data, bytes);
    } catch (const std::exception &e) {
        return nvme_fail(e);
    }
    return KVMRET_OK;
}

int kvmret_nvme_read_block(kvmret_nvme *t, uint32_t block, void *data, uint64_t bytes) {
    if (!t) return kvmret::set_error(KVMRET_ERR_ARG, "null tier");
    try {
        t->tier.read_block(block, data, bytes);
    } catch (const std::exception &e) {
        return nvme_fail(e);
    }
    return KVMRET_OK;
}

int kvmret_nvme_write_range(kvmret_nvme *t, int32_t slot, uint64_t offset, const void *data,
                            uint64_t bytes) {
    if (!t || !data) return kvmret::set_error(KVMRET_ERR_ARG, "null argument");
    try {
        t->tier.write_slot_range(slot, offset, data, bytes);
    } catch (const std::exception &e) {
        return nvme_fail(e);
    }
    return KVMRET_OK;
}

int kvmret_nvme_read_range(kvmret_nvme *t, int32_t slot, uint64_t offset, void *data,
                           uint64_t bytes) {
    if (!t || !data) return kvmret::set_error(KVMRET_ERR_ARG, "null argument");
    try {
        t->tier.read_slot_range(slot, offset, data, bytes);
    } catch (const std::exception &e) {
        return nvme_fail(e);
    }
    return KVMRET_OK;
}

int kvmret_nvme_write_spans(kvmret_nvme *t, const kvmret_nvme_span *spans, uint32_t n,
                            const void *buffer, uint64_t buffer_bytes, kvmret_nvme_stats *stats) {
    if (!t || (n && (!spans || !buffer))) return kvmret::set_error(KVMRET_ERR_ARG, "null argument");
    static_assert(sizeof(kvmret_nvme_span) == sizeof(kvmret::NvmeSpan), "span layout");
    kvmret::NvmeStats st;
    try {
        t->tier.write_spans(reinterpret_cast<const kvmret::NvmeSpan *>(spans), n, buffer,
                            buffer_bytes, &st);
    } catch (const std::exception &e) {
        return nvme_fail(e);
    }
    to_stats(st, stats);
    return KVMRET_OK;
}

int kvmret_nvme_read_spans(kvmret_nvme *t, const kvmret_nvme_span *spans, uint32_t n,
                           void *buffer, uint64_t buffer_bytes, kvmret_nvme_stats *stats) {
    if (!t || (n && (!spans || !buffer))) return kvmret::set_error(KVMRET_ERR_ARG, "null argument");
    kvmret::NvmeStats st;
    try {
        t->tier.read_spans(reinterpret_cast<const kvmret::NvmeSpan *>(spans), n, buffer,
                           buffer_bytes, &st);
    } catch (const std::exception &e) {
        return nvme_fail(e);
    }
    to_stats(st, stats);
    return KVMRET_OK;
}

}  // extern "C"
