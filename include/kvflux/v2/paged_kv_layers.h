#pragma once
// Layer-batched paged KV write and read for a model that keeps one
// PagedKVStorage per layer over one shared PhysicalBlockPool, the reference's
// multi-layer plan (docs/v2_paged_kv_storage.md:19): a slot or page id then
// names the same place in every layer. No counterpart functions in the
// reference; each is its single-layer call (write_paged_kv,
// include/kvflux/v2/paged_kv_write.h:14-15; read_paged_kv,
// include/kvflux/v2/paged_kv_read.h:18-19) over every layer in one launch,
// with the same checks, check order, exception types and synchronous
// legacy-default-stream contract. All layers must have one layout (blocks,
// KV heads, block size, head size, dtype) and one device; at most 128 layers.
#include "kvflux/v2/paged_kv_read.h"
#include "kvflux/v2/paged_kv_storage.h"

#include <vector>

namespace kvflux::v2 {

// key_new_device / value_new_device: [layers][slot_mapping.size()][num_kv_heads][head_size].
void write_paged_kv_layers(const std::vector<PagedKVStorage*>& layers, const void* key_new_device,
                           const void* value_new_device, const SlotMapping& slot_mapping);

// key_out_device / value_out_device: [layers][num_tokens][num_kv_heads][head_size].
void read_paged_kv_layers(const std::vector<const PagedKVStorage*>& layers, const SequenceState& sequence,
                          void* key_out_device, void* value_out_device);

} // namespace kvflux::v2
