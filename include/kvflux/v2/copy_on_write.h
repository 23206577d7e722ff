#pragma once
// Decode append with a device-side copy-on-write of a shared partial last
// page (reference: include/kvflux/v2/copy_on_write.h:10). The returned slot
// still has to be written with the new token's K/V.
#include "kvflux/v2/paged_kv_storage.h"

namespace kvflux::v2 {

TokenLocation append_token_cow(const PagedKVStorage& storage, SequenceState& sequence);

} // namespace kvflux::v2
