#pragma once
// Owner of physical KV page ids and their reference counts (reference:
// include/kvflux/physical_block_pool.h:11-58). Pure metadata: it allocates no
// device memory. PagedKVStorage turns an id into a device address.
#include "kvflux/block_manager.h"

#include <cstddef>
#include <cstdint>
#include <vector>

namespace kvflux {

// Index of a physical page in the KV cache; not a pointer, not ownership.
using PhysicalBlockID = std::size_t;
using PhysicalBlockHandle = BlockHandle;

// Single-threaded, like BlockManager; callers lock across threads.
class PhysicalBlockPool {
public:
    PhysicalBlockPool(std::size_t capacity, std::size_t block_size,
                      BlockManager::Hasher hasher = BlockManager::prefix_hash);

    PhysicalBlockPool(const PhysicalBlockPool&) = delete;
    PhysicalBlockPool& operator=(const PhysicalBlockPool&) = delete;
    PhysicalBlockPool(PhysicalBlockPool&&) = delete;
    PhysicalBlockPool& operator=(PhysicalBlockPool&&) = delete;

    PhysicalBlockHandle allocate();
    void retain(PhysicalBlockHandle handle);
    void free(PhysicalBlockHandle handle);

    void publish(PhysicalBlockHandle handle, const Tokens& prefix);
    bool lookup(const Tokens& prefix, PhysicalBlockHandle& out);
    bool is_published(PhysicalBlockHandle handle) const;

    // Only a live handle yields an id; a stale generation throws invalid_argument.
    PhysicalBlockID id(PhysicalBlockHandle handle) const;
    void prefetch(PhysicalBlockHandle handle) const noexcept { manager_.prefetch(handle); }
    std::size_t ref_count(PhysicalBlockHandle handle) const;
    std::size_t capacity() const noexcept;
    std::size_t block_size() const noexcept;
    // Pages that can be handed out now: free plus evictable idle cached pages.
    std::size_t available() const noexcept;
    // The manager's log of pages whose references fell to zero
    // (BlockManager::zero_ref_events / zero_ref_ids_since).
    std::uint64_t zero_ref_events() const noexcept { return manager_.zero_ref_events(); }
    bool zero_ref_ids_since(std::uint64_t since, std::vector<std::size_t>& out) const {
        return manager_.zero_ref_ids_since(since, out);
    }

private:
    BlockManager manager_;
};

inline PhysicalBlockID PhysicalBlockPool::id(PhysicalBlockHandle handle) const {
    // ref_count validates range, liveness and generation; an idle cached page
    // (zero references) must not be addressed through a stale holder either.
    if (manager_.ref_count(handle) == 0) {
        throw std::invalid_argument("physical page has no live reference");
    }
    return handle.id;
}

inline std::size_t PhysicalBlockPool::ref_count(PhysicalBlockHandle handle) const {
    return manager_.ref_count(handle);
}

} // namespace kvflux
