// Internal helpers of the C++ data plane: the per-storage runtime (reusable
// device/pinned scratch, decode workspace, duplicate-slot bitmap), the device
// guard, pointer validation, and the mapping of C-ABI codes to the
// reference's exception types.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

#include "kvflux/v2/paged_kv_storage.h"
#include "kvflux/v2/sequence_state.h"
#include "kvfx.h"

namespace kvflux::v2::detail {

[[noreturn]] void throw_cuda(const char* op, cudaError_t e);
inline void cuda_check(cudaError_t e, const char* op) {
    if (e != cudaSuccess) throw_cuda(op, e);
}

// Throws the exception type the reference raises for this C-ABI code.
void check_kvfx(int code, const char* op);

std::size_t mul_checked(std::size_t a, std::size_t b, const char* what);

// Switches to `device` for a scope and restores the previous device.
class DeviceGuard {
public:
    explicit DeviceGuard(int device);
    ~DeviceGuard() noexcept;
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;

private:
    int previous_ = 0;
};

// invalid_argument unless `p` is device memory (cudaMemoryTypeDevice) of `device`.
void require_device_pointer(const void* p, int device, const char* name);
bool overlaps(const void* a, std::size_t a_bytes, const void* b, std::size_t b_bytes);

// One run of a table patch: ids[src, src + count) go to table[dst, dst + count).
struct TablePatchRun {
    uint64_t dst;
    uint64_t src;
    uint64_t count;
};
// Enqueues the copy of every run (table, runs and ids are device memory).
cudaError_t launch_table_patch(uint64_t* table, const TablePatchRun* runs, const uint64_t* ids, uint32_t num_runs,
                               cudaStream_t stream);

struct StorageRuntime;

// The device-resident copy of the padded [rows][width] page table of the last
// batch decode on a storage (reference: build_batch_block_table,
// src/v2/batch_block_table.cpp:18-48, whose table paged_attention_batch
// uploads whole on every call, src/v2/paged_attention.cu:287-292). Each call
// re-reads, checks and uploads only the entries that changed since the last
// call: a row is keyed by its BlockTable's lineage and revision, so a row that
// only grew re-reads its new entries and an unchanged row re-reads nothing.
// Unchanged entries need no generation re-check unless one of their pages
// lost its last reference since (the pool's zero-reference log): that is the
// only way a handle checked earlier can go stale, so only then is every row
// re-checked, in row order, raising what build_batch_block_table would.
class ResidentTable {
public:
    ResidentTable() = default;
    ~ResidentTable();
    ResidentTable(const ResidentTable&) = delete;
    ResidentTable& operator=(const ResidentTable&) = delete;

    struct View {
        const uint64_t* table;  // device [rows][width]
        std::size_t width;      // row stride in entries (>= every row's pages)
        const uint64_t* lens;   // device [rows]: num_tokens of each row
        std::size_t h2d_bytes;  // bytes uploaded by this refresh
    };
    // Brings the device table up to date with `sequences` (already checked to
    // share one pool and to have `lens[r]` tokens and at most `widest` pages)
    // and uploads the lengths, all through rt's staging with one copy and at
    // most one patch launch on the legacy default stream. Throws what
    // build_batch_block_table throws for a stale handle and out_of_range for
    // an id outside the storage; after any exception the copy is forgotten.
    View refresh(StorageRuntime& rt, const std::vector<const SequenceState*>& sequences,
                 const std::vector<std::size_t>& lens, std::size_t widest, std::size_t num_blocks);
    // Forgets the copy: the next refresh re-reads every row.
    void invalidate() noexcept;

private:
    struct RowKey {
        std::uint64_t lineage = 0;
        std::uint64_t revision = 0;
        std::size_t count = 0;
    };
    void unhold(std::size_t row, std::size_t from) noexcept;

    uint64_t* dev_ = nullptr;
    int device_ = -1;
    std::size_t rows_cap_ = 0, width_ = 0;
    std::vector<RowKey> rows_;                 // rows currently held
    std::vector<PhysicalBlockID> mirror_;      // host copy [rows_cap_][width_]
    std::vector<std::uint32_t> holders_;       // per page id: held entries naming it
    const PhysicalBlockPool* pool_ = nullptr;
    std::uint64_t zero_events_ = 0;            // pool's zero-reference count when last checked
    std::vector<std::size_t> released_;        // scratch: ids from the zero-reference log
    std::vector<std::size_t> dirty_from_;      // scratch: per row, first entry to re-read
};

struct StorageRuntime {
    kvfx_cache cache{};
    int device = 0;

    // Device scratch for per-call tables and the pinned host staging that
    // feeds it; both grow and are reused, never shrink.
    void* dev_scratch = nullptr;
    std::size_t dev_bytes = 0;
    void* pinned = nullptr;
    std::size_t pinned_bytes = 0;

    // Decode/attention workspaces, zero-filled when (re)allocated; the
    // kernels leave them reusable (the decode's split counters sit at the
    // start of each and return to zero at the end of every launch). Slot 0
    // serves single launches and the first of two concurrent chunks, slot 1
    // the second chunk, so each counter region stays where it was.
    void* workspace = nullptr;
    std::size_t workspace_bytes = 0;
    void* workspace2 = nullptr;
    std::size_t workspace2_bytes = 0;

    // One bit per slot for the duplicate check of write_paged_kv.
    std::vector<std::uint64_t> seen;

    ~StorageRuntime();
    // Copies `n` arrays (host pointers and byte counts) into device scratch
    // with one H2D copy on the legacy default stream; returns device pointers.
    void upload(const void* const* host, const std::size_t* bytes, int n, void** device_out);
    // The two halves of upload for callers that write straight into the
    // staging: stage() sizes pinned staging and device scratch for `n`
    // arrays (each at a 256-byte aligned offset) and returns the host and
    // device addresses of each; push() issues the one H2D copy.
    void stage(const std::size_t* bytes, int n, void** host_out, void** device_out);
    void push();
    // Copies bytes [offset, offset + bytes) of the staging to the same range
    // of the device scratch on `stream`.
    void push_range(std::size_t offset, std::size_t bytes, cudaStream_t stream);
    std::size_t staged_bytes = 0;
    // A non-blocking stream for uploads and kernels that overlap the kernels
    // of the default stream, with two events: `side_ready` (recorded on the
    // default stream) orders the side stream after the caller's earlier work,
    // `side_done` (recorded on the side stream) orders the default stream
    // after the side stream's work. Created on first use.
    void ensure_side();
    cudaStream_t side = nullptr;
    cudaEvent_t side_ready = nullptr;
    cudaEvent_t side_done = nullptr;
    // Workspace of `slot` (0 or 1) with at least `bytes`, or nullptr for 0 bytes.
    void* ensure_workspace(std::size_t bytes, int slot = 0);
    std::size_t workspace_size(int slot = 0) const { return slot == 0 ? workspace_bytes : workspace2_bytes; }
    // Device buffer for inputs staged from the caller's host memory (Q of
    // paged_attention_batch_host); grows, never shrinks.
    void* io = nullptr;
    std::size_t io_bytes = 0;
    void* ensure_io(std::size_t bytes);
    // Synchronises the legacy default stream and raises on device-side flags.
    void finish(const char* op) const;
    // Device-resident page table of paged_attention_batch(_host), and the
    // bytes its last refresh uploaded (tables and lengths).
    ResidentTable batch_table;
    std::size_t last_table_upload = 0;
};

// Runs fn(begin, end) over [0, n) in chunks of `grain` on a small pool of
// persistent host threads plus the caller (inline when n <= grain). fn must
// be safe to run concurrently on disjoint ranges; the call returns when all
// chunks are done.
void parallel_for(std::size_t n, std::size_t grain, const std::function<void(std::size_t, std::size_t)>& fn);

} // namespace kvflux::v2::detail
