// kvfx_decode_noalloc: batch decode for callers that cannot allocate device
// memory.
//
// Who needs it: engines that reserve (nearly) all device memory for the KV
// pool at start-up and hand out nothing afterwards, so a cudaMalloc for a
// split-K workspace would fail or fragment that reservation; latency-critical
// serving loops that cannot take the implicit synchronisation of cudaMalloc /
// cudaFree; and embedders whose allocator policy forbids device allocations
// outside their own allocator. They still pass Q, O and the tables; the only
// scratch this path needs (split-K partials and per-(request, head) counters)
// lives in the file-scope array below.
//
// The array is kNoAllocScratchBytes (16 MiB) of device memory on every GPU
// where this module is loaded (with CUDA's lazy module loading, the GPUs on
// which this entry point has run), held until the process exits. Its device
// address, and that of a status word beside it, are looked up once per device
// (cudaGetSymbolAddress, with that device current) on the first call made on
// that device; make that first call before any stream capture. The addresses
// are kept for the life of the process: a device reset (cudaDeviceReset) or
// a torn-down context invalidates them, so an embedder that resets a device
// must not call this entry point on it afterwards. Every call
// shares the one array and it keeps the previous call's contents: the split
// counters at its start return to zero at the end of every launch, and are
// cleared on the call's stream by the first call on a device and by a call
// whose cache has a different number of KV heads than the previous call's
// (the counters' region depends on it); calls that overlap on the GPU (on
// different streams, or from different threads without ordering) race on the
// array. Device-side flags (an out-of-range page id, a bounded wait that gave
// up) go to the status word, which kvfx_device_status reads with the others.
#include <algorithm>
#include <mutex>
#include <string>

#include "common.cuh"
#include "launch.h"

namespace kvfx {
namespace {

constexpr uint64_t kNoAllocScratchBytes = 16ull << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ unsigned g_noalloc_status;  // KVFX_FLAG_* bits of this entry point's launches

struct DeviceState {
    void* scratch = nullptr;    // device address of g_noalloc_scratch
    unsigned* status = nullptr; // device address of g_noalloc_status
    uint32_t counter_heads = 0; // KV heads the counter region was last laid out for (0: never)
};
std::mutex g_scratch_mu;
DeviceState g_state[64];

// Set-up of `device` (which must be current), once: the symbols' addresses.
cudaError_t device_state(int device, DeviceState** out) {
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    DeviceState& st = g_state[device];
    if (st.scratch == nullptr) {
        void* scratch = nullptr;
        void* status = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        e = cudaGetSymbolAddress(&status, g_noalloc_status);
        if (e != cudaSuccess) return e;
        st.scratch = scratch;
        st.status = static_cast<unsigned*>(status);
    }
    *out = &st;
    return cudaSuccess;
}

int fail(int code, const std::string& msg) {
    set_last_error(msg.c_str());
    return code;
}

class DeviceScope {
public:
    explicit DeviceScope(int device) {
        err_ = cudaGetDevice(&prev_);
        if (err_ == cudaSuccess && prev_ != device) {
            err_ = cudaSetDevice(device);
            switched_ = err_ == cudaSuccess;
        }
    }
    ~DeviceScope() {
        if (switched_) (void)cudaSetDevice(prev_);
    }
    cudaError_t error() const { return err_; }

private:
    int prev_ = 0;
    bool switched_ = false;
    cudaError_t err_ = cudaSuccess;
};

}  // namespace
}  // namespace kvfx

extern "C" int kvfx_decode_noalloc(const kvfx_cache* cache, const float* q, float* o, const uint64_t* block_table,
                                   const uint64_t* seq_lens, uint64_t batch, uint64_t max_blocks_per_seq,
                                   uint32_t q_heads, uint64_t max_seq_len, void* stream) {
    using namespace kvfx;
    if (cache == nullptr || cache->k_base == nullptr || cache->v_base == nullptr || cache->num_blocks == 0 ||
        cache->num_kv_heads == 0 || cache->block_size == 0 || cache->head_size == 0 || cache->dtype > KVFX_F32 ||
        cache->reserved != 0 || cache->device < 0) {
        return fail(KVFX_EINVAL, "kvfx_decode_noalloc: invalid cache descriptor");
    }
    CacheView c;
    c.k = static_cast<char*>(cache->k_base);
    c.v = static_cast<char*>(cache->v_base);
    c.num_blocks = cache->num_blocks;
    c.heads = cache->num_kv_heads;
    c.bs = cache->block_size;
    c.hd = cache->head_size;
    c.dtype = cache->dtype;
    c.elem = cache->dtype == KVFX_F32 ? 4u : 2u;
    c.device = cache->device;
    c.row_bytes = static_cast<uint64_t>(c.hd) * c.elem;
    c.chunk_bytes = c.row_bytes * c.bs;
    c.page_bytes = c.chunk_bytes * c.heads;
    c.slot_count = c.num_blocks * c.bs;
    if (c.page_bytes / c.heads != c.chunk_bytes || c.num_blocks > UINT64_MAX / c.page_bytes) {
        return fail(KVFX_EOVERFLOW, "kvfx_decode_noalloc: cache size overflows");
    }
    if (q_heads == 0 || q_heads % c.heads != 0) {
        return fail(KVFX_EINVAL, "kvfx_decode_noalloc: q_heads must be a positive multiple of num_kv_heads");
    }
    if (batch == 0) return KVFX_OK;
    if (q == nullptr || o == nullptr || block_table == nullptr || seq_lens == nullptr) {
        return fail(KVFX_EINVAL, "kvfx_decode_noalloc: q, o, block_table and seq_lens must be non-null");
    }
    if (batch > 65535) return fail(KVFX_EINVAL, "kvfx_decode_noalloc: batch above 65535 sequences per launch");
    if (max_seq_len == 0) return fail(KVFX_EINVAL, "kvfx_decode_noalloc: max_seq_len must be positive");
    if (max_blocks_per_seq < ceil_div(max_seq_len, c.bs)) {
        return fail(KVFX_EINVAL, "kvfx_decode_noalloc: max_blocks_per_seq is smaller than max_seq_len needs");
    }

    DeviceScope scope(c.device);
    if (scope.error() != cudaSuccess) {
        return fail(KVFX_ECUDA, std::string("kvfx_decode_noalloc: select device: ") + cudaGetErrorString(scope.error()));
    }
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    DecodeArgs a{q, o, block_table, seq_lens, batch, max_blocks_per_seq, max_seq_len, q_heads, 0, nullptr, 0};

    std::lock_guard<std::mutex> lock(g_scratch_mu);
    DeviceState* st = nullptr;
    cudaError_t e = device_state(c.device, &st);
    if (e != cudaSuccess) {
        return fail(KVFX_ECUDA, std::string("kvfx_decode_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    }

    // Shapes of the generic kernel need no scratch at all.
    if (decode_workspace_bytes(c, batch, q_heads, max_seq_len, 0) == 0) {
        e = launch_decode(c, a, st->status, s);
        return e == cudaSuccess ? KVFX_OK
                                : fail(KVFX_ECUDA, std::string("kvfx_decode_noalloc: launch: ") + cudaGetErrorString(e));
    }

    // Fewest pages per split (most parallelism) whose workspace fits the
    // array: the counter region (fixed by the KV heads), then the partials.
    const uint64_t pairs = batch * c.heads;
    const uint64_t per_split = 8ull * (c.hd + 2) * 4;
    const uint64_t counters = decode_counter_bytes(c.heads);
    if (counters + 256 + pairs * per_split > kNoAllocScratchBytes) {
        return fail(KVFX_ENOSPACE,
                    "kvfx_decode_noalloc: batch x num_kv_heads = " + std::to_string(pairs) +
                        " needs more than the 16 MiB static scratch even with one split per sequence");
    }
    const uint64_t max_pages = ceil_div(max_seq_len, c.bs);
    const uint64_t splits_fit = (kNoAllocScratchBytes - counters - 256) / (pairs * per_split);
    uint64_t pps = decode_pages_per_split(c, batch, q_heads, max_seq_len, 0);
    pps = std::max<uint64_t>(pps, ceil_div(max_pages, std::max<uint64_t>(splits_fit, 1)));
    a.pages_per_split = static_cast<uint32_t>(std::min<uint64_t>(pps, 1u << 30));
    const uint64_t need = decode_workspace_bytes(c, batch, q_heads, max_seq_len, a.pages_per_split);
    if (need > kNoAllocScratchBytes) {
        return fail(KVFX_ENOSPACE, "kvfx_decode_noalloc: workspace of " + std::to_string(need) +
                                       " bytes exceeds the 16 MiB static scratch");
    }
    a.workspace = st->scratch;
    a.workspace_bytes = kNoAllocScratchBytes;
    // The counters must start at zero: they do after any launch laid out for
    // the same number of KV heads; otherwise (first use, or the last call
    // used another head count, whose partials may lie in this region) clear
    // them on the stream.
    if (st->counter_heads != c.heads) {
        e = cudaMemsetAsync(st->scratch, 0, counters, s);
        if (e != cudaSuccess) {
            return fail(KVFX_ECUDA, std::string("kvfx_decode_noalloc: clear counters: ") + cudaGetErrorString(e));
        }
        st->counter_heads = c.heads;
    }
    const CacheMaps* maps = cache_maps(c, &e);
    if (maps == nullptr) {
        return fail(KVFX_ECUDA, std::string("kvfx_decode_noalloc: tensor maps: ") +
                                    cudaGetErrorString(e != cudaSuccess ? e : cudaErrorInvalidValue));
    }
    e = launch_decode_with_maps(c, a, *maps, st->status, s);
    return e == cudaSuccess ? KVFX_OK
                            : fail(KVFX_ECUDA, std::string("kvfx_decode_noalloc: launch: ") + cudaGetErrorString(e));
}

namespace kvfx {

bool noalloc_status(int device, unsigned* flags, bool clear) {
    *flags = 0;
    if (device < 0 || device >= 64) return true;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_state[device].status == nullptr) return true;  // never set up: nothing raised
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return false;
    if (prev != device && cudaSetDevice(device) != cudaSuccess) return false;
    bool ok = cudaMemcpyFromSymbol(flags, g_noalloc_status, sizeof(unsigned)) == cudaSuccess;
    if (ok && clear && *flags != 0) {
        const unsigned zero = 0;
        ok = cudaMemcpyToSymbol(g_noalloc_status, &zero, sizeof(unsigned)) == cudaSuccess;
    }
    if (prev != device) (void)cudaSetDevice(prev);
    return ok;
}

}  // namespace kvfx
