// Page-slot metadata manager. Behaviour follows the reference's v0 manager
// (src/block_manager.cpp:45-134 for allocate/retain/release/publish/lookup,
// :214-226 for the prefix hash); see the header for what differs internally.
#include "kvflux/block_manager.h"

#include <algorithm>
#include <utility>

namespace kvflux {

BlockManager::BlockManager(std::size_t capacity, std::size_t block_size, Hasher hasher)
    : slots_(capacity), meta_(capacity), block_size_(block_size), hasher_(std::move(hasher)),
      zero_log_(kZeroLog) {
    if (capacity == 0 || block_size == 0 || !hasher_) {
        throw std::invalid_argument("block manager needs a positive capacity, block size and a hasher");
    }
    // Stack with id 0 on top: the first allocations hand out 0, 1, 2, ...
    free_stack_.resize(capacity);
    for (std::size_t i = 0; i < capacity; ++i) free_stack_[i] = capacity - 1 - i;
}

void BlockManager::idle_push(std::size_t id) noexcept {
    SlotMeta& s = meta_[id];
    s.idle_prev = idle_newest_;
    s.idle_next = kNone;
    if (idle_newest_ == kNone) idle_oldest_ = id;
    else meta_[idle_newest_].idle_next = id;
    idle_newest_ = id;
    ++idle_count_;
}

void BlockManager::idle_remove(std::size_t id) noexcept {
    SlotMeta& s = meta_[id];
    if (s.idle_prev == kNone) idle_oldest_ = s.idle_next;
    else meta_[s.idle_prev].idle_next = s.idle_next;
    if (s.idle_next == kNone) idle_newest_ = s.idle_prev;
    else meta_[s.idle_next].idle_prev = s.idle_prev;
    s.idle_prev = s.idle_next = kNone;
    --idle_count_;
}

void BlockManager::drop_index(std::size_t id) {
    SlotMeta& m = meta_[id];
    auto bucket = index_.find(m.hash);
    if (bucket != index_.end()) {
        auto& ids = bucket->second;
        ids.erase(std::remove(ids.begin(), ids.end(), id), ids.end());
        if (ids.empty()) index_.erase(bucket);
    }
    slots_[id].published = false;
    m.prefix.clear();
    m.prefix.shrink_to_fit();
}

BlockHandle BlockManager::allocate() {
    std::size_t id;
    const bool from_free = !free_stack_.empty();
    if (from_free) id = free_stack_.back();
    else if (idle_oldest_ != kNone) id = idle_oldest_;
    else throw CapacityError();

    Slot& s = slots_[id];
    if (s.generation == std::numeric_limits<std::uint64_t>::max()) {
        throw std::overflow_error("block generation counter exhausted");
    }
    if (from_free) {
        free_stack_.pop_back();
    } else {
        // Evict the least recently idled cached page; it had no references.
        idle_remove(id);
        drop_index(id);
    }
    s.state = State::Active;
    s.refs = 1;
    ++s.generation;
    ++active_count_;
    return {id, s.generation};
}

void BlockManager::retain(BlockHandle h) {
    Slot& s = live(h);
    if (s.refs == std::numeric_limits<std::uint32_t>::max()) {
        throw std::overflow_error("block reference count exhausted");
    }
    if (s.state == State::Idle) {
        idle_remove(h.id);
        s.state = State::Active;
        ++active_count_;
    }
    ++s.refs;
}

void BlockManager::release(BlockHandle h) {
    Slot& s = live(h);
    if (s.refs == 0) throw std::invalid_argument("block has no reference to release");
    if (--s.refs != 0) return;
    zero_log_[zero_events_ % kZeroLog] = h.id;
    ++zero_events_;
    --active_count_;
    if (s.published) {
        s.state = State::Idle;
        idle_push(h.id);
    } else {
        s.state = State::Free;
        free_stack_.push_back(h.id);
    }
}

bool BlockManager::is_published(BlockHandle h) const { return live(h).published; }

void BlockManager::publish(BlockHandle h, const Tokens& prefix) {
    Slot& s = live(h);
    if (s.refs != 1 || s.published || prefix.empty() || prefix.size() % block_size_ != 0) {
        throw std::invalid_argument("publish needs a privately held block and a whole-block prefix");
    }
    const std::uint64_t hash = hasher_(prefix);
    auto bucket = index_.find(hash);
    if (bucket != index_.end()) {
        for (std::size_t other : bucket->second) {
            if (meta_[other].prefix == prefix) {
                throw std::invalid_argument("prefix is already published");
            }
        }
    }
    // Everything that can throw happens before the slot is marked published.
    Tokens stored(prefix);
    auto [it, inserted] = index_.try_emplace(hash);
    try {
        it->second.push_back(h.id);
    } catch (...) {
        if (inserted) index_.erase(it);
        throw;
    }
    meta_[h.id].prefix = std::move(stored);
    meta_[h.id].hash = hash;
    s.published = true;
}

bool BlockManager::lookup(const Tokens& prefix, BlockHandle& out) {
    if (prefix.empty() || prefix.size() % block_size_ != 0) return false;
    auto bucket = index_.find(hasher_(prefix));
    if (bucket == index_.end()) return false;
    for (std::size_t id : bucket->second) {
        if (meta_[id].prefix != prefix) continue;  // same hash, different tokens
        const BlockHandle hit{id, slots_[id].generation};
        retain(hit);
        out = hit;
        return true;
    }
    return false;
}

BlockTable BlockManager::acquire(const Tokens& tokens) {
    BlockTable table;
    table.token_count = tokens.size();
    const std::size_t blocks = tokens.size() / block_size_ + (tokens.size() % block_size_ != 0);
    table.blocks.reserve(blocks);
    Tokens prefix;
    prefix.reserve(tokens.size());
    try {
        std::size_t start = 0;
        while (start < tokens.size()) {
            const std::size_t count = std::min(block_size_, tokens.size() - start);
            prefix.insert(prefix.end(), tokens.begin() + static_cast<std::ptrdiff_t>(start),
                          tokens.begin() + static_cast<std::ptrdiff_t>(start + count));
            const bool whole = count == block_size_;
            BlockHandle h{};
            if (whole && lookup(prefix, h)) {
                table.blocks.push_back(h);
            } else {
                h = allocate();
                table.blocks.push_back(h);  // capacity reserved: cannot throw
                if (whole) publish(h, prefix);
            }
            start += count;
        }
    } catch (...) {
        for (const BlockHandle& h : table.blocks) release(h);
        throw;
    }
    return table;
}

void BlockManager::check_table(const BlockTable& table) const {
    const std::size_t expected =
        table.token_count / block_size_ + (table.token_count % block_size_ != 0);
    if (expected != table.blocks.size()) throw std::invalid_argument("block table size mismatch");
    for (std::size_t i = 0; i < table.blocks.size(); ++i) {
        if (live(table.blocks[i]).refs == 0) throw std::invalid_argument("block table entry not held");
        for (std::size_t j = 0; j < i; ++j) {
            if (table.blocks[i] == table.blocks[j]) throw std::invalid_argument("duplicate block in table");
        }
    }
}

BlockTable BlockManager::share(const BlockTable& table) {
    check_table(table);
    BlockTable copy = table;
    std::size_t done = 0;
    try {
        for (const BlockHandle& h : copy.blocks) {
            retain(h);
            ++done;
        }
    } catch (...) {
        for (std::size_t i = 0; i < done; ++i) release(copy.blocks[i]);
        throw;
    }
    return copy;
}

void BlockManager::release(BlockTable& table) {
    check_table(table);
    for (const BlockHandle& h : table.blocks) release(h);
    table.blocks.clear();
    table.token_count = 0;
}

BlockHandle BlockManager::block_at(const BlockTable& table, std::size_t token_index) const {
    if (token_index >= table.token_count) throw std::out_of_range("token index beyond table");
    const BlockHandle h = table.blocks.at(token_index / block_size_);
    if (live(h).refs == 0) throw std::invalid_argument("block table entry not held");
    return h;
}

bool BlockManager::zero_ref_ids_since(std::uint64_t since, std::vector<std::size_t>& out) const {
    if (since > zero_events_) return false;
    if (zero_events_ - since > kZeroLog) return false;
    for (std::uint64_t e = since; e < zero_events_; ++e) out.push_back(zero_log_[e % kZeroLog]);
    return true;
}

BlockManager::Stats BlockManager::stats() const noexcept {
    return {slots_.size(), free_stack_.size(), active_count_, idle_count_};
}

std::uint64_t BlockManager::prefix_hash(const Tokens& prefix) noexcept {
    // FNV-1a 64: offset basis 0xcbf29ce484222325, prime 0x100000001b3.
    std::uint64_t h = 0xcbf29ce484222325ULL;
    for (const Token t : prefix) {
        std::uint32_t bits = static_cast<std::uint32_t>(t);
        for (int b = 0; b < 4; ++b, bits >>= 8) {
            h ^= bits & 0xffu;
            h *= 0x100000001b3ULL;
        }
    }
    return h;
}

} // namespace kvflux
