// write_paged_kv and read_paged_kv: the reference's host-side contract
// (src/v2/paged_kv_write.cu:101-139, src/v2/paged_kv_read.cu:106-155) in the
// same check order, with the per-call cudaMalloc replaced by reused scratch
// and the kernels reached through the C ABI.
#include "kvflux/v2/paged_kv_read.h"
#include "kvflux/v2/paged_kv_write.h"
#include "runtime.h"

namespace kvflux::v2 {

void write_paged_kv(PagedKVStorage& storage, const void* key_new_device, const void* value_new_device,
                    const SlotMapping& slot_mapping) {
    if (slot_mapping.empty()) return;
    if (key_new_device == nullptr || value_new_device == nullptr) {
        throw std::invalid_argument("K_new and V_new device pointers are required");
    }
    const PagedKVLayout& layout = storage.layout();
    detail::StorageRuntime& rt = storage.runtime();

    // Range and duplicate checks in input order (the first offence decides the
    // exception type, as in the reference). One bit per slot, cleared after.
    const std::size_t words = (layout.slot_count() + 63) / 64;
    if (rt.seen.size() < words) rt.seen.assign(words, 0);
    std::size_t checked = 0;
    auto clear_seen = [&] {
        for (std::size_t i = 0; i < checked; ++i) {
            const PhysicalSlot s = slot_mapping[i];
            rt.seen[s >> 6] &= ~(std::uint64_t{1} << (s & 63));
        }
    };
    for (const PhysicalSlot s : slot_mapping) {
        if (s >= layout.slot_count()) {
            clear_seen();
            throw std::out_of_range("KV write slot out of range");
        }
        std::uint64_t& w = rt.seen[s >> 6];
        const std::uint64_t bit = std::uint64_t{1} << (s & 63);
        if (w & bit) {
            clear_seen();
            throw std::invalid_argument("duplicate KV write slot");
        }
        w |= bit;
        ++checked;
    }
    clear_seen();

    const std::size_t elements = detail::mul_checked(
        detail::mul_checked(slot_mapping.size(), layout.num_kv_heads(), "paged KV write"),
        layout.head_size(), "paged KV write");
    (void)detail::mul_checked(elements, layout.element_bytes(), "paged KV write");
    const std::size_t slot_bytes = detail::mul_checked(slot_mapping.size(), sizeof(PhysicalSlot), "paged KV write");

    detail::DeviceGuard guard(storage.device());
    detail::require_device_pointer(key_new_device, storage.device(), "K_new");
    detail::require_device_pointer(value_new_device, storage.device(), "V_new");
    const void* host[1] = {slot_mapping.data()};
    void* dev[1] = {nullptr};
    rt.upload(host, &slot_bytes, 1, dev);
    detail::check_kvfx(kvfx_write(&rt.cache, key_new_device, value_new_device,
                                  static_cast<const uint64_t*>(dev[0]), slot_mapping.size(), nullptr),
                       "paged KV write");
    rt.finish("paged KV write synchronize");
}

void read_paged_kv(const PagedKVStorage& storage, const SequenceState& sequence, void* key_out_device,
                   void* value_out_device) {
    if (!storage.uses_pool(sequence.block_table())) {
        throw std::invalid_argument("sequence and KV storage must use one physical pool");
    }
    const PagedKVLayout& layout = storage.layout();
    if (sequence.block_size() != layout.block_size()) {
        throw std::invalid_argument("sequence and KV storage block sizes differ");
    }
    if (sequence.num_tokens() == 0) return;
    if (key_out_device == nullptr || value_out_device == nullptr) {
        throw std::invalid_argument("K and V output device pointers are required");
    }
    const ReadBlockTable blocks = build_read_block_table(sequence);
    for (const PhysicalBlockID b : blocks) {
        if (b >= layout.num_blocks()) throw std::out_of_range("KV read block out of range");
    }
    const std::size_t elements = detail::mul_checked(
        detail::mul_checked(sequence.num_tokens(), layout.num_kv_heads(), "paged KV read"),
        layout.head_size(), "paged KV read");
    const std::size_t out_bytes = detail::mul_checked(elements, layout.element_bytes(), "paged KV read");
    const std::size_t table_bytes = detail::mul_checked(blocks.size(), sizeof(PhysicalBlockID), "paged KV read");

    detail::DeviceGuard guard(storage.device());
    detail::require_device_pointer(key_out_device, storage.device(), "K_out");
    detail::require_device_pointer(value_out_device, storage.device(), "V_out");
    if (detail::overlaps(key_out_device, out_bytes, value_out_device, out_bytes) ||
        detail::overlaps(key_out_device, out_bytes, storage.key_base(), layout.total_bytes()) ||
        detail::overlaps(value_out_device, out_bytes, storage.key_base(), layout.total_bytes())) {
        throw std::invalid_argument("KV read outputs must not overlap each other or the cache");
    }
    detail::StorageRuntime& rt = storage.runtime();
    const void* host[1] = {blocks.data()};
    void* dev[1] = {nullptr};
    rt.upload(host, &table_bytes, 1, dev);
    detail::check_kvfx(kvfx_gather(&rt.cache, static_cast<const uint64_t*>(dev[0]), sequence.num_tokens(),
                                   key_out_device, value_out_device, nullptr),
                       "paged KV read");
    rt.finish("paged KV read synchronize");
}

} // namespace kvflux::v2
