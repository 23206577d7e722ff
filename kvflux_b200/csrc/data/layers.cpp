// write_paged_kv_layers and read_paged_kv_layers
// (include/kvflux/v2/paged_kv_layers.h): the single-layer checks of
// write_read.cpp, then one kvfx_write_layers / kvfx_gather_layers launch.
#include "kvflux/v2/paged_kv_layers.h"

#include "runtime.h"

namespace kvflux::v2 {

namespace {

// Every layer non-null and of the first layer's layout and device.
const PagedKVStorage& check_layers(const PagedKVStorage* const* layers, std::size_t n, const char* op) {
    if (n == 0) throw std::invalid_argument(std::string(op) + " needs at least one layer");
    if (n > KVFX_MAX_LAYERS) throw std::invalid_argument(std::string(op) + ": more than 128 layers");
    for (std::size_t l = 0; l < n; ++l) {
        if (layers[l] == nullptr) throw std::invalid_argument(std::string(op) + ": null layer storage");
    }
    const PagedKVStorage& first = *layers[0];
    const PagedKVLayout& a = first.layout();
    for (std::size_t l = 1; l < n; ++l) {
        const PagedKVLayout& b = layers[l]->layout();
        if (b.num_blocks() != a.num_blocks() || b.num_kv_heads() != a.num_kv_heads() ||
            b.block_size() != a.block_size() || b.head_size() != a.head_size() || b.dtype() != a.dtype() ||
            layers[l]->device() != first.device()) {
            throw std::invalid_argument(std::string(op) + ": layer storages differ in layout or device");
        }
    }
    return first;
}

std::vector<kvfx_cache> descriptors(const PagedKVStorage* const* layers, std::size_t n) {
    std::vector<kvfx_cache> out(n);
    for (std::size_t l = 0; l < n; ++l) out[l] = layers[l]->runtime().cache;
    return out;
}

} // namespace

void write_paged_kv_layers(const std::vector<PagedKVStorage*>& layers, const void* key_new_device,
                           const void* value_new_device, const SlotMapping& slot_mapping) {
    std::vector<const PagedKVStorage*> view(layers.begin(), layers.end());
    const PagedKVStorage& first = check_layers(view.data(), view.size(), "layered KV write");
    if (slot_mapping.empty()) return;
    if (key_new_device == nullptr || value_new_device == nullptr) {
        throw std::invalid_argument("K_new and V_new device pointers are required");
    }
    const PagedKVLayout& layout = first.layout();
    detail::StorageRuntime& rt = first.runtime();

    // Range and duplicate checks in input order, as write_paged_kv.
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
        detail::mul_checked(slot_mapping.size(), layout.num_kv_heads(), "layered KV write"), layout.head_size(),
        "layered KV write");
    const std::size_t layer_bytes = detail::mul_checked(elements, layout.element_bytes(), "layered KV write");
    (void)detail::mul_checked(layer_bytes, layers.size(), "layered KV write");
    const std::size_t slot_bytes = detail::mul_checked(slot_mapping.size(), sizeof(PhysicalSlot), "layered KV write");

    detail::DeviceGuard guard(first.device());
    detail::require_device_pointer(key_new_device, first.device(), "K_new");
    detail::require_device_pointer(value_new_device, first.device(), "V_new");
    const void* host[1] = {slot_mapping.data()};
    void* dev[1] = {nullptr};
    rt.upload(host, &slot_bytes, 1, dev);
    const std::vector<kvfx_cache> caches = descriptors(view.data(), view.size());
    detail::check_kvfx(kvfx_write_layers(caches.data(), static_cast<uint32_t>(caches.size()), key_new_device,
                                         value_new_device, layer_bytes, static_cast<const uint64_t*>(dev[0]),
                                         slot_mapping.size(), nullptr),
                       "layered KV write");
    rt.finish("layered KV write synchronize");
}

void read_paged_kv_layers(const std::vector<const PagedKVStorage*>& layers, const SequenceState& sequence,
                          void* key_out_device, void* value_out_device) {
    const PagedKVStorage& first = check_layers(layers.data(), layers.size(), "layered KV read");
    for (const PagedKVStorage* l : layers) {
        if (!l->uses_pool(sequence.block_table())) {
            throw std::invalid_argument("sequence and KV storage must use one physical pool");
        }
    }
    const PagedKVLayout& layout = first.layout();
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
        detail::mul_checked(sequence.num_tokens(), layout.num_kv_heads(), "layered KV read"), layout.head_size(),
        "layered KV read");
    const std::size_t layer_bytes = detail::mul_checked(elements, layout.element_bytes(), "layered KV read");
    const std::size_t out_bytes = detail::mul_checked(layer_bytes, layers.size(), "layered KV read");

    detail::DeviceGuard guard(first.device());
    detail::require_device_pointer(key_out_device, first.device(), "K_out");
    detail::require_device_pointer(value_out_device, first.device(), "V_out");
    if (detail::overlaps(key_out_device, out_bytes, value_out_device, out_bytes)) {
        throw std::invalid_argument("KV read outputs must not overlap each other or the cache");
    }
    for (const PagedKVStorage* l : layers) {
        if (detail::overlaps(key_out_device, out_bytes, l->key_base(), layout.total_bytes()) ||
            detail::overlaps(value_out_device, out_bytes, l->key_base(), layout.total_bytes())) {
            throw std::invalid_argument("KV read outputs must not overlap each other or the cache");
        }
    }
    // Device staging: the page ids, the length, and the two one-entry output lists.
    const std::uint64_t len = sequence.num_tokens();
    const std::uint64_t kp = reinterpret_cast<std::uintptr_t>(key_out_device);
    const std::uint64_t vp = reinterpret_cast<std::uintptr_t>(value_out_device);
    const std::size_t bytes[4] = {blocks.size() * sizeof(PhysicalBlockID), sizeof(len), sizeof(kp), sizeof(vp)};
    const void* host[4] = {blocks.data(), &len, &kp, &vp};
    void* dev[4] = {nullptr, nullptr, nullptr, nullptr};
    detail::StorageRuntime& rt = first.runtime();
    rt.upload(host, bytes, 4, dev);
    const std::vector<kvfx_cache> caches = descriptors(layers.data(), layers.size());
    detail::check_kvfx(kvfx_gather_layers(caches.data(), static_cast<uint32_t>(caches.size()),
                                          static_cast<const uint64_t*>(dev[0]), static_cast<const uint64_t*>(dev[1]),
                                          1, blocks.size(), static_cast<void* const*>(dev[2]),
                                          static_cast<void* const*>(dev[3]), layer_bytes, nullptr),
                       "layered KV read");
    rt.finish("layered KV read synchronize");
}

} // namespace kvflux::v2
