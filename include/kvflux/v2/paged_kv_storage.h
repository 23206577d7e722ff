#pragma once
// Device memory of one layer's paged K/V on one GPU (reference:
// include/kvflux/v2/paged_kv_storage.h:14-45). One cudaMalloc holds the K
// region followed by the V region; PhysicalBlockPool stays the only owner of
// page ids and references.
//
// Besides the cache itself a storage keeps a small per-device runtime that the
// data-plane calls reuse (device copies of slot/page tables, pinned staging,
// decode workspace), so no call allocates device memory once it has run once
// with a given size.
#include "kvflux/physical_block_pool.h"
#include "kvflux/v2/paged_kv_layout.h"
#include "kvflux/v2/slot_mapping.h"

#include <cstddef>
#include <memory>

namespace kvflux::v2 {

namespace detail { struct StorageRuntime; }

class PagedKVStorage {
public:
    PagedKVStorage(PhysicalBlockPool& pool, std::size_t num_kv_heads,
                   std::size_t head_size, DType dtype, int device = 0);
    ~PagedKVStorage() noexcept;

    PagedKVStorage(const PagedKVStorage&) = delete;
    PagedKVStorage& operator=(const PagedKVStorage&) = delete;

    const PagedKVLayout& layout() const noexcept { return layout_; }
    int device() const noexcept { return device_; }
    bool uses_pool(const BlockTable& table) const noexcept { return table.uses_pool(pool_); }
    void* key_base() const;
    void* value_base() const;

    // Device addresses (the host must not dereference them).
    void* page_address(KVKind kind, PhysicalBlockHandle handle) const;
    void* element_address(KVKind kind, PhysicalBlockHandle handle,
                          std::size_t head, std::size_t token, std::size_t dimension) const;
    void* slot_address(KVKind kind, PhysicalSlot slot,
                       std::size_t head, std::size_t dimension) const;

    // Byte-exact copy of the whole K page and V page of `source` into the
    // private, unpublished page `destination`; returns after the device is done.
    void copy_block(PhysicalBlockHandle source, PhysicalBlockHandle destination) const;

    // Runtime used by the data-plane entry points; not part of the reference API.
    detail::StorageRuntime& runtime() const { return *runtime_; }

private:
    PhysicalBlockPool& pool_;
    PagedKVLayout layout_;
    int device_;
    void* base_ = nullptr;
    std::unique_ptr<detail::StorageRuntime> runtime_;
};

} // namespace kvflux::v2
