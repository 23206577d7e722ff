// Incremental update of a device-resident page table: the host stages the
// changed entries (runs of consecutive ids) and one launch writes them into
// place, so a batch table whose rows only grew by a page or two costs a few
// hundred bytes of upload instead of the whole [rows][width] table.
#include <cuda_runtime.h>
#include <stdint.h>

#include "data/runtime.h"

namespace kvflux::v2::detail {
namespace {

// One CTA per run: run r copies runs[r].count ids from ids[runs[r].src] to
// table[runs[r].dst]. Runs are whole rows (up to a few thousand entries) or
// single appended entries; both are short, so one CTA each is enough.
__global__ void __launch_bounds__(128) table_patch_kernel(uint64_t* __restrict__ table,
                                                          const TablePatchRun* __restrict__ runs,
                                                          const uint64_t* __restrict__ ids) {
    const TablePatchRun r = runs[blockIdx.x];
    for (uint64_t i = threadIdx.x; i < r.count; i += blockDim.x) table[r.dst + i] = ids[r.src + i];
}

}  // namespace

cudaError_t launch_table_patch(uint64_t* table, const TablePatchRun* runs, const uint64_t* ids, uint32_t num_runs,
                               cudaStream_t stream) {
    if (num_runs == 0) return cudaSuccess;
    table_patch_kernel<<<num_runs, 128, 0, stream>>>(table, runs, ids);
    return cudaGetLastError();
}

}  // namespace kvflux::v2::detail
