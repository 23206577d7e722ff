#pragma once
// Element types and K/V selector shared by the v2 paged layout
// (reference: include/kvflux/kv_layout.h:7-8). The enumerator order is the
// numeric dtype code used by the C-ABI in kvfx.h (0 f16, 1 bf16, 2 f32).
#include <cstddef>

namespace kvflux {

enum class DType { Float16, BFloat16, Float32 };
enum class KVKind { Key, Value };

} // namespace kvflux
