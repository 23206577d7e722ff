#pragma once
// Page-slot metadata manager: the dependency under kvflux::PhysicalBlockPool.
//
// Same public interface and observable behaviour as the reference's v0
// manager (include/kvflux/block_manager.h:18-104, src/block_manager.cpp):
//   * allocation order is LIFO over a free list that starts as 0,1,2,...
//     (every fragmented-pool fixture of the reference depends on this);
//   * handles carry a generation that is bumped on every allocation, so a
//     handle from an earlier lifetime of the same slot is rejected;
//   * a published (full-prefix) block whose reference count drops to zero is
//     kept as an evictable idle entry, reclaimed oldest-first only when the
//     free list is empty;
//   * lookup compares the full token prefix, so hash collisions never alias.
// Differences that are not observable through the API: the free list is a
// vector stack, the idle entries sit in an index-linked list, and stats() is
// O(1) from counters kept up to date instead of a scan over all slots.
#include <cstddef>
#include <cstdint>
#include <functional>
#include <limits>
#include <stdexcept>
#include <unordered_map>
#include <vector>

namespace kvflux {

using Token = std::int32_t;
using Tokens = std::vector<Token>;

struct BlockHandle {
    std::size_t id;
    std::uint64_t generation;
    bool operator==(const BlockHandle& other) const noexcept {
        return id == other.id && generation == other.generation;
    }
};

// Teaching-level (v0) sequence table: copying it does not add references.
struct BlockTable {
    std::vector<BlockHandle> blocks;
    std::size_t token_count = 0;
};

class CapacityError : public std::runtime_error {
public:
    CapacityError() : std::runtime_error("no reclaimable KV block") {}
};

// Single-threaded; handles are only meaningful for the instance that made them.
class BlockManager {
public:
    using Hasher = std::function<std::uint64_t(const Tokens&)>;
    struct Stats {
        std::size_t capacity, free, active, cached_idle;
    };

    explicit BlockManager(std::size_t capacity, std::size_t block_size,
                          Hasher hasher = prefix_hash);
    BlockManager(const BlockManager&) = delete;
    BlockManager& operator=(const BlockManager&) = delete;
    BlockManager(BlockManager&&) = delete;
    BlockManager& operator=(BlockManager&&) = delete;

    BlockHandle allocate();
    void retain(BlockHandle handle);
    void release(BlockHandle handle);
    std::size_t ref_count(BlockHandle handle) const;
    bool is_published(BlockHandle handle) const;

    // prefix: every token from the start of the sequence to the end of this block.
    void publish(BlockHandle handle, const Tokens& prefix);
    // On a hit adds one reference and writes `out`; on a miss leaves `out` alone.
    bool lookup(const Tokens& prefix, BlockHandle& out);

    BlockTable acquire(const Tokens& tokens);
    BlockTable share(const BlockTable& table);
    void release(BlockTable& table);
    BlockHandle block_at(const BlockTable& table, std::size_t token_index) const;

    Stats stats() const noexcept;
    std::size_t capacity() const noexcept { return slots_.size(); }
    // Log of pages whose reference count fell to zero (the only way a handle
    // that was live can go stale: its page must first lose every reference).
    // zero_ref_events() counts such events since construction;
    // zero_ref_ids_since(e, out) appends the ids of the events after the
    // count was e, oldest first, and returns false (appending nothing) when
    // more than kZeroLog of them happened since, i.e. the log cannot tell.
    // A holder of handles checked when the count read e knows they are all
    // still live if none of its ids is among them.
    static constexpr std::size_t kZeroLog = 8192;
    std::uint64_t zero_ref_events() const noexcept { return zero_events_; }
    bool zero_ref_ids_since(std::uint64_t since, std::vector<std::size_t>& out) const;
    // Hint: bring the bookkeeping of `h` into cache ahead of a lookup. No
    // check, no effect on state.
    void prefetch(BlockHandle h) const noexcept {
        if (h.id < slots_.size()) __builtin_prefetch(slots_.data() + h.id);
    }
    std::size_t block_size() const noexcept { return block_size_; }
    // FNV-1a (64-bit) over each token's four bytes, least significant first.
    static std::uint64_t prefix_hash(const Tokens& prefix) noexcept;

private:
    static constexpr std::size_t kNone = std::numeric_limits<std::size_t>::max();
    enum class State : std::uint8_t { Free, Active, Idle };
    // What every handle check reads, packed densely: validating a large page
    // table touches only this array. 16 bytes, so that no slot straddles two
    // cache lines (one miss per checked entry).
    struct Slot {
        std::uint64_t generation = 0;
        std::uint32_t refs = 0;
        State state = State::Free;
        bool published = false;
    };
    static_assert(sizeof(Slot) == 16, "Slot must pack into 16 bytes");
    // What only publish/lookup/eviction read.
    struct SlotMeta {
        std::uint64_t hash = 0;
        Tokens prefix;
        std::size_t idle_prev = kNone, idle_next = kNone;
    };

    const Slot& live(BlockHandle handle) const;
    Slot& live(BlockHandle handle);
    void check_table(const BlockTable& table) const;
    void idle_push(std::size_t id) noexcept;
    void idle_remove(std::size_t id) noexcept;
    void drop_index(std::size_t id);

    std::vector<Slot> slots_;
    std::vector<SlotMeta> meta_;
    std::size_t block_size_;
    Hasher hasher_;
    std::vector<std::size_t> free_stack_;  // top of stack = back()
    std::size_t idle_oldest_ = kNone, idle_newest_ = kNone;
    std::size_t active_count_ = 0, idle_count_ = 0;
    std::unordered_map<std::uint64_t, std::vector<std::size_t>> index_;
    std::vector<std::size_t> zero_log_;  // ring of kZeroLog ids
    std::uint64_t zero_events_ = 0;
};

// Hot-path accessors, inline so page-table builds validate each entry cheaply.
inline const BlockManager::Slot& BlockManager::live(BlockHandle h) const {
    if (h.id >= slots_.size()) throw std::invalid_argument("block handle id out of range");
    const Slot& s = slots_[h.id];
    if (s.state == State::Free || s.generation != h.generation) {
        throw std::invalid_argument("stale or released block handle");
    }
    return s;
}

inline BlockManager::Slot& BlockManager::live(BlockHandle h) {
    return const_cast<Slot&>(static_cast<const BlockManager*>(this)->live(h));
}

inline std::size_t BlockManager::ref_count(BlockHandle h) const { return live(h).refs; }

} // namespace kvflux
