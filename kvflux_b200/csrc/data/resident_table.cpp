// ResidentTable: the device-resident batch page table (see runtime.h).
#include <algorithm>
#include <cstring>

#include "kvflux/v2/batch_block_table.h"
#include "runtime.h"

namespace kvflux::v2::detail {

ResidentTable::~ResidentTable() {
    if (dev_ == nullptr) return;
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return;
    if (cudaSetDevice(device_) == cudaSuccess) (void)cudaFree(dev_);
    (void)cudaSetDevice(prev);
}

void ResidentTable::invalidate() noexcept {
    rows_.clear();
    std::fill(holders_.begin(), holders_.end(), 0u);
    pool_ = nullptr;
}

void ResidentTable::unhold(std::size_t row, std::size_t from) noexcept {
    const PhysicalBlockID* ids = mirror_.data() + row * width_;
    for (std::size_t j = from; j < rows_[row].count; ++j) --holders_[ids[j]];
}

ResidentTable::View ResidentTable::refresh(StorageRuntime& rt, const std::vector<const SequenceState*>& sequences,
                                           const std::vector<std::size_t>& lens, std::size_t widest,
                                           std::size_t num_blocks) {
    const std::size_t batch = sequences.size();
    const PhysicalBlockPool& pool = sequences.front()->block_table().pool();
    if (pool_ != &pool || holders_.size() != num_blocks) {
        invalidate();
        holders_.assign(num_blocks, 0u);
        pool_ = &pool;
        zero_events_ = pool.zero_ref_events();
    }
    // Room for the batch: grow the row stride with headroom, so that rows
    // growing a page per 16 decode steps rarely force a re-layout.
    if (widest > width_ || batch > rows_cap_ || dev_ == nullptr) {
        const std::size_t width = std::max(widest + widest / 4 + 16, width_);
        const std::size_t rows = std::max(batch, rows_cap_);
        const std::size_t bytes = mul_checked(mul_checked(rows, width, "batch table"), sizeof(uint64_t),
                                              "batch table");
        invalidate();
        holders_.assign(num_blocks, 0u);
        pool_ = &pool;
        zero_events_ = pool.zero_ref_events();
        if (dev_ != nullptr) {
            cuda_check(cudaFree(dev_), "free batch table");
            dev_ = nullptr;
        }
        cuda_check(cudaMalloc(reinterpret_cast<void**>(&dev_), bytes), "allocate batch table");
        cuda_check(cudaGetDevice(&device_), "cudaGetDevice");
        mirror_.assign(rows * width, BatchBlockTable::invalid_block());
        rows_cap_ = rows;
        width_ = width;
    }

    try {
        // 1. Which entries of each row must be re-read; stop holding the old
        //    ones there, and every entry of rows past the batch.
        for (std::size_t r = batch; r < rows_.size(); ++r) unhold(r, 0);
        if (rows_.size() > batch) rows_.resize(batch);
        dirty_from_.assign(batch, 0);
        std::size_t runs = 0, fresh = 0;
        for (std::size_t r = 0; r < batch; ++r) {
            const BlockTable& t = sequences[r]->block_table();
            const std::size_t n = t.size();
            std::size_t from = 0;
            if (r < rows_.size() && rows_[r].lineage == t.lineage()) {
                from = std::min(t.first_changed_since(rows_[r].revision), rows_[r].count);
            }
            if (r < rows_.size()) unhold(r, from);
            dirty_from_[r] = from;
            if (from < n) {
                ++runs;
                fresh += n - from;
            }
        }
        // 2. Entries kept from earlier calls were checked then; one of them
        //    can be stale only if its page has lost every reference since.
        released_.clear();
        bool suspect = !pool.zero_ref_ids_since(zero_events_, released_);
        for (std::size_t i = 0; !suspect && i < released_.size(); ++i) {
            suspect = released_[i] < holders_.size() && holders_[released_[i]] != 0;
        }
        if (suspect) (void)build_batch_block_table(sequences);  // raises what the reference raises

        // 3. Stage the lengths, the runs and their ids; check the new ids.
        void* host[3] = {nullptr, nullptr, nullptr};
        void* dev[3] = {nullptr, nullptr, nullptr};
        const std::size_t bytes[3] = {batch * sizeof(uint64_t), runs * sizeof(TablePatchRun),
                                      fresh * sizeof(uint64_t)};
        rt.stage(bytes, 3, host, dev);
        std::memcpy(host[0], lens.data(), bytes[0]);
        auto* run = static_cast<TablePatchRun*>(host[1]);
        auto* ids = static_cast<PhysicalBlockID*>(host[2]);
        std::size_t at = 0;
        for (std::size_t r = 0; r < batch; ++r) {
            const BlockTable& t = sequences[r]->block_table();
            const std::size_t n = t.size();
            const std::size_t from = dirty_from_[r];
            if (r >= rows_.size()) rows_.push_back(RowKey{});
            rows_[r].count = from;  // entries held so far (a throw below leaves this row consistent)
            if (from < n) {
                t.copy_ids(ids + at, from);
                bool bad = false;
                for (std::size_t j = 0; j < n - from; ++j) bad |= ids[at + j] >= num_blocks;
                if (bad) throw std::out_of_range("batch attention block out of range");
                PhysicalBlockID* m = mirror_.data() + r * width_;
                for (std::size_t j = from; j < n; ++j) {
                    m[j] = ids[at + j - from];
                    ++holders_[m[j]];
                }
                *run++ = TablePatchRun{r * width_ + from, at, n - from};
                at += n - from;
            }
            rows_[r] = RowKey{t.lineage(), t.revision(), n};
        }
        zero_events_ = pool.zero_ref_events();
        rt.push();
        cuda_check(launch_table_patch(dev_, static_cast<const TablePatchRun*>(dev[1]),
                                      static_cast<const uint64_t*>(dev[2]), static_cast<uint32_t>(runs), nullptr),
                   "patch batch table");
        return View{dev_, width_, static_cast<const uint64_t*>(dev[0]), rt.staged_bytes};
    } catch (...) {
        invalidate();
        throw;
    }
}

}  // namespace kvflux::v2::detail
