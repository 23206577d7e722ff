// PagedKVStorage and the shared data-plane runtime (reference:
// src/v2/paged_kv_storage.cpp:38-93 for the storage semantics).
#include <cstring>
#include <limits>

#include "kvflux/v2/paged_kv_storage.h"
#include "runtime.h"

namespace kvflux::v2 {
namespace detail {

void throw_cuda(const char* op, cudaError_t e) {
    throw std::runtime_error(std::string(op) + ": " + cudaGetErrorString(e));
}

void check_kvfx(int code, const char* op) {
    if (code == KVFX_OK) return;
    const std::string msg = std::string(op) + ": " + kvfx_last_error();
    switch (code) {
    case KVFX_EINVAL: throw std::invalid_argument(msg);
    case KVFX_ERANGE: throw std::out_of_range(msg);
    case KVFX_EOVERFLOW: throw std::overflow_error(msg);
    default: throw std::runtime_error(msg);
    }
}

std::size_t mul_checked(std::size_t a, std::size_t b, const char* what) {
    if (b != 0 && a > std::numeric_limits<std::size_t>::max() / b) {
        throw std::overflow_error(std::string(what) + " size overflow");
    }
    return a * b;
}

DeviceGuard::DeviceGuard(int device) {
    cuda_check(cudaGetDevice(&previous_), "cudaGetDevice");
    if (previous_ != device) cuda_check(cudaSetDevice(device), "cudaSetDevice");
}

DeviceGuard::~DeviceGuard() noexcept { (void)cudaSetDevice(previous_); }

void require_device_pointer(const void* p, int device, const char* name) {
    cudaPointerAttributes a{};
    const cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess || a.type != cudaMemoryTypeDevice || a.device != device) {
        if (e != cudaSuccess) (void)cudaGetLastError();
        throw std::invalid_argument(std::string(name) + " must be device memory of the storage's GPU");
    }
}

bool overlaps(const void* a, std::size_t a_bytes, const void* b, std::size_t b_bytes) {
    const auto x = reinterpret_cast<std::uintptr_t>(a);
    const auto y = reinterpret_cast<std::uintptr_t>(b);
    return x <= y ? y - x < a_bytes : x - y < b_bytes;
}

StorageRuntime::~StorageRuntime() {
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return;
    if (cudaSetDevice(device) != cudaSuccess) return;
    if (dev_scratch) (void)cudaFree(dev_scratch);
    if (workspace) (void)cudaFree(workspace);
    if (workspace2) (void)cudaFree(workspace2);
    if (io) (void)cudaFree(io);
    if (pinned) (void)cudaFreeHost(pinned);
    if (side_ready) (void)cudaEventDestroy(side_ready);
    if (side_done) (void)cudaEventDestroy(side_done);
    if (side) (void)cudaStreamDestroy(side);
    (void)cudaSetDevice(prev);
}

void StorageRuntime::stage(const std::size_t* bytes, int n, void** host_out, void** device_out) {
    std::size_t total = 0;
    std::size_t offsets[8];
    for (int i = 0; i < n; ++i) {
        offsets[i] = total;
        total += (bytes[i] + 255) & ~std::size_t(255);
    }
    if (total > pinned_bytes) {
        if (pinned) cuda_check(cudaFreeHost(pinned), "free pinned staging");
        pinned = nullptr;
        pinned_bytes = 0;
        const std::size_t cap = std::max<std::size_t>(total, 4096);
        cuda_check(cudaHostAlloc(&pinned, cap, cudaHostAllocPortable), "allocate pinned staging");
        pinned_bytes = cap;
    }
    if (total > dev_bytes) {
        if (dev_scratch) cuda_check(cudaFree(dev_scratch), "free device scratch");
        dev_scratch = nullptr;
        dev_bytes = 0;
        const std::size_t cap = std::max<std::size_t>(total, 4096);
        cuda_check(cudaMalloc(&dev_scratch, cap), "allocate device scratch");
        dev_bytes = cap;
    }
    for (int i = 0; i < n; ++i) {
        host_out[i] = static_cast<unsigned char*>(pinned) + offsets[i];
        device_out[i] = static_cast<unsigned char*>(dev_scratch) + offsets[i];
    }
    staged_bytes = total;
}

void StorageRuntime::push() {
    // The staging buffer is reused by the next call only after this call has
    // synchronised the stream, so one buffer suffices.
    cuda_check(cudaMemcpyAsync(dev_scratch, pinned, staged_bytes, cudaMemcpyHostToDevice, nullptr),
               "upload tables");
}

void StorageRuntime::push_range(std::size_t offset, std::size_t bytes, cudaStream_t stream) {
    if (bytes == 0) return;
    cuda_check(cudaMemcpyAsync(static_cast<unsigned char*>(dev_scratch) + offset,
                               static_cast<const unsigned char*>(pinned) + offset, bytes, cudaMemcpyHostToDevice,
                               stream),
               "upload tables");
}

void StorageRuntime::ensure_side() {
    if (side == nullptr) cuda_check(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking), "create side stream");
    if (side_ready == nullptr) {
        cuda_check(cudaEventCreateWithFlags(&side_ready, cudaEventDisableTiming), "create side event");
    }
    if (side_done == nullptr) {
        cuda_check(cudaEventCreateWithFlags(&side_done, cudaEventDisableTiming), "create side event");
    }
}

void StorageRuntime::upload(const void* const* host, const std::size_t* bytes, int n, void** device_out) {
    void* staging[8];
    stage(bytes, n, staging, device_out);
    for (int i = 0; i < n; ++i) {
        if (bytes[i] != 0) std::memcpy(staging[i], host[i], bytes[i]);
    }
    push();
}

void* StorageRuntime::ensure_workspace(std::size_t bytes, int slot) {
    if (bytes == 0) return nullptr;
    void*& ptr = slot == 0 ? workspace : workspace2;
    std::size_t& size = slot == 0 ? workspace_bytes : workspace2_bytes;
    if (bytes > size) {
        if (ptr) cuda_check(cudaFree(ptr), "free workspace");
        ptr = nullptr;
        size = 0;
        cuda_check(cudaMalloc(&ptr, bytes), "allocate workspace");
        cuda_check(cudaMemsetAsync(ptr, 0, bytes, nullptr), "clear workspace");
        size = bytes;
    }
    return ptr;
}

void* StorageRuntime::ensure_io(std::size_t bytes) {
    if (bytes > io_bytes) {
        if (io) cuda_check(cudaFree(io), "free input staging");
        io = nullptr;
        io_bytes = 0;
        cuda_check(cudaMalloc(&io, bytes), "allocate input staging");
        io_bytes = bytes;
    }
    return io;
}

void StorageRuntime::finish(const char* op) const {
    const cudaError_t e = cudaStreamSynchronize(nullptr);
    if (e != cudaSuccess) throw_cuda(op, e);
    uint32_t flags = 0;
    if (kvfx_device_status(device, &flags, 1) == KVFX_OK && flags != 0) {
        if (flags & KVFX_FLAG_TIMEOUT) {
            throw std::runtime_error(std::string(op) + ": a bounded device wait timed out");
        }
        throw std::runtime_error(std::string(op) + ": a kernel saw an out-of-range page or slot id");
    }
}

} // namespace detail

namespace {

std::size_t backing_bytes(const PagedKVLayout& layout) { return layout.total_bytes(); }

} // namespace

PagedKVStorage::PagedKVStorage(PhysicalBlockPool& pool, std::size_t num_kv_heads, std::size_t head_size,
                               DType dtype, int device)
    : pool_(pool), layout_(pool.capacity(), num_kv_heads, pool.block_size(), head_size, dtype),
      device_(device), runtime_(std::make_unique<detail::StorageRuntime>()) {
    if (device < 0) throw std::invalid_argument("device ordinal must be non-negative");
    int count = 0;
    detail::cuda_check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (device >= count) throw std::invalid_argument("GPU device index out of range");
    detail::DeviceGuard guard(device_);
    detail::cuda_check(cudaMalloc(&base_, backing_bytes(layout_)), "cudaMalloc KV cache");
    auto& rt = *runtime_;
    rt.device = device_;
    rt.cache.k_base = base_;
    rt.cache.v_base = static_cast<unsigned char*>(base_) + layout_.cache_bytes();
    rt.cache.num_blocks = layout_.num_blocks();
    rt.cache.num_kv_heads = static_cast<uint32_t>(layout_.num_kv_heads());
    rt.cache.block_size = static_cast<uint32_t>(layout_.block_size());
    rt.cache.head_size = static_cast<uint32_t>(layout_.head_size());
    rt.cache.dtype = static_cast<uint32_t>(layout_.dtype());
    rt.cache.device = device_;
    rt.cache.reserved = 0;
    if (layout_.num_kv_heads() > UINT32_MAX || layout_.block_size() > UINT32_MAX ||
        layout_.head_size() > UINT32_MAX) {
        (void)cudaFree(base_);
        throw std::invalid_argument("KV layout dimensions above 2^32 are not supported");
    }
}

PagedKVStorage::~PagedKVStorage() noexcept {
    runtime_.reset();
    int prev = 0;
    if (base_ && cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(device_) == cudaSuccess) {
        (void)cudaFree(base_);
        (void)cudaSetDevice(prev);
    }
}

void* PagedKVStorage::key_base() const { return base_; }

void* PagedKVStorage::value_base() const {
    return static_cast<unsigned char*>(base_) + layout_.cache_bytes();
}

void* PagedKVStorage::page_address(KVKind kind, PhysicalBlockHandle handle) const {
    const PhysicalBlockID id = pool_.id(handle);
    return static_cast<unsigned char*>(base_) + layout_.page_byte_offset(kind, id);
}

void* PagedKVStorage::element_address(KVKind kind, PhysicalBlockHandle handle, std::size_t head,
                                      std::size_t token, std::size_t dimension) const {
    const PhysicalBlockID id = pool_.id(handle);
    return static_cast<unsigned char*>(base_) + layout_.byte_offset(kind, id, head, token, dimension);
}

void* PagedKVStorage::slot_address(KVKind kind, PhysicalSlot slot, std::size_t head,
                                   std::size_t dimension) const {
    return static_cast<unsigned char*>(base_) + layout_.slot_byte_offset(kind, slot, head, dimension);
}

void PagedKVStorage::copy_block(PhysicalBlockHandle source, PhysicalBlockHandle destination) const {
    const PhysicalBlockID src = pool_.id(source);
    const PhysicalBlockID dst = pool_.id(destination);
    if (src == dst || pool_.ref_count(destination) != 1 || pool_.is_published(destination)) {
        throw std::invalid_argument("copy destination must be a private, unpublished page");
    }
    detail::DeviceGuard guard(device_);
    try {
        detail::check_kvfx(kvfx_copy_page(&runtime_->cache, src, dst, nullptr), "copy KV page");
        runtime_->finish("synchronize KV page copy");
    } catch (...) {
        // Work already queued must finish before the caller reuses the page.
        (void)cudaStreamSynchronize(nullptr);
        throw;
    }
}

} // namespace kvflux::v2
