// Thin page-id owner over BlockManager (reference: src/physical_block_pool.cpp:12-50).
#include "kvflux/physical_block_pool.h"

#include <stdexcept>
#include <utility>

namespace kvflux {

PhysicalBlockPool::PhysicalBlockPool(std::size_t capacity, std::size_t block_size,
                                     BlockManager::Hasher hasher)
    : manager_(capacity, block_size, std::move(hasher)) {}

PhysicalBlockHandle PhysicalBlockPool::allocate() { return manager_.allocate(); }
void PhysicalBlockPool::retain(PhysicalBlockHandle h) { manager_.retain(h); }
void PhysicalBlockPool::free(PhysicalBlockHandle h) { manager_.release(h); }
void PhysicalBlockPool::publish(PhysicalBlockHandle h, const Tokens& prefix) {
    manager_.publish(h, prefix);
}
bool PhysicalBlockPool::lookup(const Tokens& prefix, PhysicalBlockHandle& out) {
    return manager_.lookup(prefix, out);
}
bool PhysicalBlockPool::is_published(PhysicalBlockHandle h) const { return manager_.is_published(h); }

std::size_t PhysicalBlockPool::capacity() const noexcept { return manager_.capacity(); }
std::size_t PhysicalBlockPool::block_size() const noexcept { return manager_.block_size(); }
std::size_t PhysicalBlockPool::available() const noexcept {
    const auto s = manager_.stats();
    return s.free + s.cached_idle;
}

} // namespace kvflux
