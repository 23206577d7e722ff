#pragma once
// Scatter of new K/V rows into their cache slots (reference:
// include/kvflux/v2/paged_kv_write.h:14-15). K_new/V_new are device arrays
// [batch][num_kv_heads][head_size] in the storage dtype; slot_mapping has one
// slot per batch row. Synchronous on the legacy default stream. An empty
// mapping returns before touching any pointer. Rejects null pointers,
// out-of-range slots (out_of_range), duplicate slots and pointers that are not
// device memory of the storage's GPU (invalid_argument).
#include "kvflux/v2/paged_kv_storage.h"

namespace kvflux::v2 {

void write_paged_kv(PagedKVStorage& storage, const void* key_new_device,
                    const void* value_new_device, const SlotMapping& slot_mapping);

} // namespace kvflux::v2
