// C ABI entry points (include/kvfx.h): argument validation, device selection,
// and dispatch to the kernel launchers. No entry point allocates device
// memory per call; the only allocation is the per-device status word (one
// mapped host word, made on a device's first call).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <mutex>
#include <string>

#include "kernels/launch.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(const char* op, cudaError_t e) {
    return fail(KVFX_ECUDA, std::string(op) + ": " + cudaGetErrorString(e));
}

bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) {
    if (b != 0 && a > std::numeric_limits<uint64_t>::max() / b) return false;
    *out = a * b;
    return true;
}

// Makes the cache's device current for the duration of a call.
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

int make_view(const kvfx_cache* c, kvfx::CacheView* v) {
    if (c == nullptr) return fail(KVFX_EINVAL, "cache descriptor is null");
    if (c->k_base == nullptr || c->v_base == nullptr) return fail(KVFX_EINVAL, "cache base pointer is null");
    if (c->num_blocks == 0 || c->num_kv_heads == 0 || c->block_size == 0 || c->head_size == 0) {
        return fail(KVFX_EINVAL, "cache dimensions must be positive");
    }
    if (c->dtype > KVFX_F32) return fail(KVFX_EINVAL, "unsupported cache dtype");
    if (c->reserved != 0) return fail(KVFX_EINVAL, "kvfx_cache.reserved must be 0");
    if (c->device < 0) return fail(KVFX_EINVAL, "device ordinal must be non-negative");
    v->k = static_cast<char*>(c->k_base);
    v->v = static_cast<char*>(c->v_base);
    v->num_blocks = c->num_blocks;
    v->heads = c->num_kv_heads;
    v->bs = c->block_size;
    v->hd = c->head_size;
    v->dtype = c->dtype;
    v->elem = c->dtype == KVFX_F32 ? 4u : 2u;
    v->device = c->device;
    if (!mul_ok(v->hd, v->elem, &v->row_bytes) || !mul_ok(v->row_bytes, v->bs, &v->chunk_bytes) ||
        !mul_ok(v->chunk_bytes, v->heads, &v->page_bytes) || !mul_ok(v->num_blocks, v->bs, &v->slot_count)) {
        return fail(KVFX_EOVERFLOW, "cache size arithmetic overflows");
    }
    uint64_t total = 0;
    if (!mul_ok(v->page_bytes, v->num_blocks, &total)) return fail(KVFX_EOVERFLOW, "cache size overflows");
    return KVFX_OK;
}

std::mutex g_status_mu;
unsigned* g_status[64] = {nullptr};

// Mapped host word the kernels atomically OR flags into. nullptr if the
// device has no mapping support (kernels then skip flagging).
unsigned* status_word(int device) {
    if (device < 0 || device >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_status_mu);
    if (g_status[device] == nullptr) {
        void* h = nullptr;
        if (cudaHostAlloc(&h, 64, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
            (void)cudaGetLastError();
            return nullptr;
        }
        std::memset(h, 0, 64);
        void* d = nullptr;
        if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
            (void)cudaGetLastError();
            return nullptr;
        }
        g_status[device] = static_cast<unsigned*>(d);
    }
    return g_status[device];
}

}  // namespace

namespace kvfx {
void set_last_error(const char* msg) { g_last_error = msg; }
}  // namespace kvfx

extern "C" {

const char* kvfx_last_error(void) { return g_last_error.c_str(); }

const char* kvfx_version(void) { return "kvflux-b200 0.1.0 sm_100a"; }

int kvfx_device_status(int device, uint32_t* flags, int clear) {
    if (flags == nullptr) return fail(KVFX_EINVAL, "flags pointer is null");
    unsigned* w = status_word(device);
    if (w == nullptr) {
        *flags = 0;
        return fail(KVFX_ECUDA, "status word unavailable on this device");
    }
    volatile unsigned* vw = w;  // mapped host memory: host and device views coincide (UVA)
    *flags = *vw;
    if (clear) *vw = 0;
    // kvfx_decode_noalloc's launches keep their flags in a device variable
    // (that entry point allocates nothing, not even this mapped word).
    unsigned extra = 0;
    if (!kvfx::noalloc_status(device, &extra, clear != 0)) {
        return fail(KVFX_ECUDA, "reading the no-allocation decode's status word failed");
    }
    *flags |= extra;
    return KVFX_OK;
}

int kvfx_selftest_wait_timeout(int device) {
    if (device < 0) return fail(KVFX_EINVAL, "device ordinal must be non-negative");
    DeviceScope scope(device);
    if (scope.error() != cudaSuccess) return cuda_fail("select device", scope.error());
    unsigned* st = status_word(device);
    if (st == nullptr) return fail(KVFX_ECUDA, "status word unavailable on this device");
    volatile unsigned* flags = st;
    const unsigned before = *flags;
    *flags = 0;
    int completed[2] = {-1, -1};
    const cudaError_t e = kvfx::launch_wait_selftest(st, nullptr, completed);
    const unsigned seen = *flags;
    *flags = before | (seen & ~KVFX_FLAG_TIMEOUT);  // the self-test's own flag is not left behind
    if (e != cudaSuccess) return cuda_fail("wait self-test", e);
    if (completed[0] != 0 || completed[1] != 0 || (seen & KVFX_FLAG_TIMEOUT) == 0) {
        return fail(KVFX_EINVAL, "a bounded wait on an unsignalled barrier did not report a timeout");
    }
    return fail(KVFX_ETIMEOUT, "bounded device waits gave up on an unsignalled barrier and reported it");
}

int kvfx_write(const kvfx_cache* cache, const void* k_new, const void* v_new, const uint64_t* slots,
               uint64_t num_tokens, void* stream) {
    kvfx::CacheView c;
    if (int rc = make_view(cache, &c); rc != KVFX_OK) return rc;
    if (num_tokens == 0) return KVFX_OK;
    if (k_new == nullptr || v_new == nullptr || slots == nullptr) {
        return fail(KVFX_EINVAL, "k_new, v_new and slots must be non-null");
    }
    uint64_t rows = 0, bytes = 0;
    if (!mul_ok(num_tokens, c.heads, &rows) || !mul_ok(rows, c.row_bytes, &bytes)) {
        return fail(KVFX_EOVERFLOW, "write size overflows");
    }
    DeviceScope scope(c.device);
    if (scope.error() != cudaSuccess) return cuda_fail("select device", scope.error());
    const cudaError_t e = kvfx::launch_write(c, k_new, v_new, slots, num_tokens, status_word(c.device),
                                             static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? KVFX_OK : cuda_fail("paged KV write launch", e);
}

int kvfx_gather(const kvfx_cache* cache, const uint64_t* blocks, uint64_t num_tokens, void* k_out,
                void* v_out, void* stream) {
    kvfx::CacheView c;
    if (int rc = make_view(cache, &c); rc != KVFX_OK) return rc;
    if (num_tokens == 0) return KVFX_OK;
    if (blocks == nullptr || k_out == nullptr || v_out == nullptr) {
        return fail(KVFX_EINVAL, "blocks, k_out and v_out must be non-null");
    }
    uint64_t rows = 0, bytes = 0;
    if (!mul_ok(num_tokens, c.heads, &rows) || !mul_ok(rows, c.row_bytes, &bytes)) {
        return fail(KVFX_EOVERFLOW, "gather size overflows");
    }
    DeviceScope scope(c.device);
    if (scope.error() != cudaSuccess) return cuda_fail("select device", scope.error());
    kvfx::GatherArgs a{};
    a.blocks = blocks;
    a.lens = nullptr;
    a.single_len = num_tokens;
    a.batch = 1;
    a.max_blocks = kvfx::ceil_div(num_tokens, c.bs);
    a.k_out = k_out;
    a.v_out = v_out;
    a.max_len = num_tokens;
    const cudaError_t e = kvfx::launch_gather(c, a, status_word(c.device), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? KVFX_OK : cuda_fail("paged KV gather launch", e);
}

int kvfx_gather_batch(const kvfx_cache* cache, const uint64_t* blocks, const uint64_t* seq_lens,
                      uint64_t batch, uint64_t max_blocks_per_seq, void* const* k_out,
                      void* const* v_out, void* stream) {
    kvfx::CacheView c;
    if (int rc = make_view(cache, &c); rc != KVFX_OK) return rc;
    if (batch == 0 || max_blocks_per_seq == 0) return KVFX_OK;
    if (blocks == nullptr || seq_lens == nullptr || k_out == nullptr || v_out == nullptr) {
        return fail(KVFX_EINVAL, "blocks, seq_lens, k_out and v_out must be non-null");
    }
    if (batch > 65535) return fail(KVFX_EINVAL, "batch above 65535 sequences per launch");
    uint64_t max_len = 0;
    if (!mul_ok(max_blocks_per_seq, c.bs, &max_len)) return fail(KVFX_EOVERFLOW, "table size overflows");
    DeviceScope scope(c.device);
    if (scope.error() != cudaSuccess) return cuda_fail("select device", scope.error());
    kvfx::GatherArgs a{};
    a.blocks = blocks;
    a.lens = seq_lens;
    a.batch = batch;
    a.max_blocks = max_blocks_per_seq;
    a.k_out_list = k_out;
    a.v_out_list = v_out;
    a.max_len = max_len;
    const cudaError_t e = kvfx::launch_gather(c, a, status_word(c.device), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? KVFX_OK : cuda_fail("paged KV batched gather launch", e);
}

// Views of num_layers caches that must agree in everything but their bases.
int make_layer_views(const kvfx_cache* caches, uint32_t num_layers, kvfx::CacheView* views) {
    if (caches == nullptr) return fail(KVFX_EINVAL, "caches array is null");
    if (num_layers > KVFX_MAX_LAYERS) return fail(KVFX_EINVAL, "more than KVFX_MAX_LAYERS layers");
    for (uint32_t l = 0; l < num_layers; ++l) {
        if (int rc = make_view(caches + l, views + l); rc != KVFX_OK) return rc;
        const kvfx::CacheView& a = views[0];
        const kvfx::CacheView& b = views[l];
        if (b.num_blocks != a.num_blocks || b.heads != a.heads || b.bs != a.bs || b.hd != a.hd ||
            b.dtype != a.dtype || b.device != a.device) {
            return fail(KVFX_EINVAL, "layer caches differ in shape, dtype or device");
        }
    }
    return KVFX_OK;
}

int kvfx_write_layers(const kvfx_cache* caches, uint32_t num_layers, const void* k_new, const void* v_new,
                      uint64_t layer_stride_bytes, const uint64_t* slots, uint64_t num_tokens, void* stream) {
    kvfx::CacheView views[KVFX_MAX_LAYERS];
    if (int rc = make_layer_views(caches, num_layers, views); rc != KVFX_OK) return rc;
    if (num_layers == 0 || num_tokens == 0) return KVFX_OK;
    if (k_new == nullptr || v_new == nullptr || slots == nullptr) {
        return fail(KVFX_EINVAL, "k_new, v_new and slots must be non-null");
    }
    const kvfx::CacheView& c = views[0];
    uint64_t rows = 0, bytes = 0, span = 0;
    if (!mul_ok(num_tokens, c.heads, &rows) || !mul_ok(rows, c.row_bytes, &bytes) ||
        !mul_ok(layer_stride_bytes, num_layers - 1, &span) || span + bytes < span) {
        return fail(KVFX_EOVERFLOW, "layered write size overflows");
    }
    if (num_layers > 1 && layer_stride_bytes < bytes) {
        return fail(KVFX_EINVAL, "layer_stride_bytes is smaller than one layer's rows");
    }
    DeviceScope scope(c.device);
    if (scope.error() != cudaSuccess) return cuda_fail("select device", scope.error());
    const cudaError_t e = kvfx::launch_write_layers(views, num_layers, k_new, v_new, layer_stride_bytes, slots,
                                                    num_tokens, status_word(c.device),
                                                    static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? KVFX_OK : cuda_fail("layered paged KV write launch", e);
}

int kvfx_gather_layers(const kvfx_cache* caches, uint32_t num_layers, const uint64_t* blocks,
                       const uint64_t* seq_lens, uint64_t batch, uint64_t max_blocks_per_seq,
                       void* const* k_out, void* const* v_out, uint64_t out_layer_stride_bytes, void* stream) {
    kvfx::CacheView views[KVFX_MAX_LAYERS];
    if (int rc = make_layer_views(caches, num_layers, views); rc != KVFX_OK) return rc;
    if (num_layers == 0 || batch == 0 || max_blocks_per_seq == 0) return KVFX_OK;
    if (blocks == nullptr || seq_lens == nullptr || k_out == nullptr || v_out == nullptr) {
        return fail(KVFX_EINVAL, "blocks, seq_lens, k_out and v_out must be non-null");
    }
    if (batch > 65535) return fail(KVFX_EINVAL, "batch above 65535 sequences per launch");
    const kvfx::CacheView& c = views[0];
    uint64_t max_len = 0, per_seq = 0, tmp = 0, span = 0;
    if (!mul_ok(max_blocks_per_seq, c.bs, &max_len) || !mul_ok(max_len, c.heads, &tmp) ||
        !mul_ok(tmp, c.row_bytes, &per_seq) || !mul_ok(out_layer_stride_bytes, num_layers - 1, &span)) {
        return fail(KVFX_EOVERFLOW, "layered gather size overflows");
    }
    DeviceScope scope(c.device);
    if (scope.error() != cudaSuccess) return cuda_fail("select device", scope.error());
    kvfx::GatherArgs a{};
    a.blocks = blocks;
    a.lens = seq_lens;
    a.batch = batch;
    a.max_blocks = max_blocks_per_seq;
    a.k_out_list = k_out;
    a.v_out_list = v_out;
    a.max_len = max_len;
    unsigned* st = status_word(c.device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = kvfx::launch_gather_layers(views, num_layers, a, out_layer_stride_bytes, st, s);
    if (e == cudaErrorNotSupported) {  // rows or alignments the 16-byte kernel cannot take: per layer
        e = cudaSuccess;
        a.force_simt = true;
        for (uint32_t l = 0; l < num_layers && e == cudaSuccess; ++l) {
            a.out_offset = l * out_layer_stride_bytes;
            e = kvfx::launch_gather(views[l], a, st, s);
        }
    }
    return e == cudaSuccess ? KVFX_OK : cuda_fail("layered paged KV gather launch", e);
}

int kvfx_copy_page(const kvfx_cache* cache, uint64_t src_block, uint64_t dst_block, void* stream) {
    kvfx::CacheView c;
    if (int rc = make_view(cache, &c); rc != KVFX_OK) return rc;
    if (src_block >= c.num_blocks || dst_block >= c.num_blocks) return fail(KVFX_ERANGE, "page id out of range");
    if (src_block == dst_block) return fail(KVFX_EINVAL, "source and destination page are the same");
    DeviceScope scope(c.device);
    if (scope.error() != cudaSuccess) return cuda_fail("select device", scope.error());
    const cudaError_t e = kvfx::launch_copy_page(c, src_block, dst_block, status_word(c.device),
                                                 static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? KVFX_OK : cuda_fail("page copy launch", e);
}

uint32_t kvfx_decode_pages_per_split(const kvfx_cache* cache, uint64_t batch, uint32_t q_heads,
                                     uint64_t max_seq_len, uint64_t total_tokens) {
    kvfx::CacheView c;
    if (make_view(cache, &c) != KVFX_OK) return 0;
    return kvfx::decode_pages_per_split(c, batch, q_heads, max_seq_len, total_tokens);
}

uint64_t kvfx_decode_workspace_bytes(const kvfx_cache* cache, uint64_t batch, uint32_t q_heads,
                                     uint64_t max_seq_len, uint32_t pages_per_split) {
    kvfx::CacheView c;
    if (make_view(cache, &c) != KVFX_OK || q_heads == 0 || q_heads % c.heads != 0) return 0;
    return kvfx::decode_workspace_bytes(c, batch, q_heads, max_seq_len, pages_per_split);
}

int kvfx_decode(const kvfx_cache* cache, const float* q, float* o, const uint64_t* block_table,
                const uint64_t* seq_lens, uint64_t batch, uint64_t max_blocks_per_seq, uint32_t q_heads,
                uint64_t max_seq_len, uint32_t pages_per_split, void* workspace,
                uint64_t workspace_bytes, void* stream) {
    kvfx::CacheView c;
    if (int rc = make_view(cache, &c); rc != KVFX_OK) return rc;
    if (q_heads == 0 || q_heads % c.heads != 0) {
        return fail(KVFX_EINVAL, "q_heads must be a positive multiple of num_kv_heads");
    }
    if (batch == 0) return KVFX_OK;
    if (q == nullptr || o == nullptr || block_table == nullptr || seq_lens == nullptr) {
        return fail(KVFX_EINVAL, "q, o, block_table and seq_lens must be non-null");
    }
    if (batch > 65535) return fail(KVFX_EINVAL, "batch above 65535 sequences per launch");
    if (max_seq_len == 0) return fail(KVFX_EINVAL, "max_seq_len must be positive");
    if (max_blocks_per_seq < kvfx::ceil_div(max_seq_len, c.bs)) {
        return fail(KVFX_EINVAL, "max_blocks_per_seq is smaller than max_seq_len needs");
    }
    uint64_t elems = 0, tmp = 0;
    if (!mul_ok(batch, q_heads, &tmp) || !mul_ok(tmp, c.hd, &elems)) {
        return fail(KVFX_EOVERFLOW, "query size overflows");
    }
    const uint64_t need = kvfx::decode_workspace_bytes(c, batch, q_heads, max_seq_len, pages_per_split);
    if (need != 0 && (workspace == nullptr || workspace_bytes < need)) {
        return fail(KVFX_ENOSPACE, "decode workspace is smaller than kvfx_decode_workspace_bytes()");
    }
    DeviceScope scope(c.device);
    if (scope.error() != cudaSuccess) return cuda_fail("select device", scope.error());
    kvfx::DecodeArgs a{q, o, block_table, seq_lens, batch, max_blocks_per_seq, max_seq_len,
                       q_heads, pages_per_split, workspace, workspace_bytes};
    const cudaError_t e = kvfx::launch_decode(c, a, status_word(c.device), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? KVFX_OK : cuda_fail("batch decode launch", e);
}

int kvfx_decode_append(const kvfx_cache* cache, const void* k_new, const void* v_new,
                       const uint64_t* new_slots, const float* q, float* o, uint64_t* block_table,
                       const uint64_t* seq_lens, uint64_t batch, uint64_t max_blocks_per_seq,
                       uint32_t q_heads, uint64_t max_seq_len, uint32_t pages_per_split, void* workspace,
                       uint64_t workspace_bytes, void* stream) {
    kvfx::CacheView c;
    if (int rc = make_view(cache, &c); rc != KVFX_OK) return rc;
    if (q_heads == 0 || q_heads % c.heads != 0) {
        return fail(KVFX_EINVAL, "q_heads must be a positive multiple of num_kv_heads");
    }
    if (batch == 0) return KVFX_OK;
    if (k_new == nullptr || v_new == nullptr || new_slots == nullptr || q == nullptr || o == nullptr ||
        block_table == nullptr || seq_lens == nullptr) {
        return fail(KVFX_EINVAL, "k_new, v_new, new_slots, q, o, block_table and seq_lens must be non-null");
    }
    if (batch > 65535) return fail(KVFX_EINVAL, "batch above 65535 sequences per launch");
    if (max_seq_len == 0) return fail(KVFX_EINVAL, "max_seq_len must be positive");
    if (max_blocks_per_seq < kvfx::ceil_div(max_seq_len, c.bs)) {
        return fail(KVFX_EINVAL, "max_blocks_per_seq is smaller than max_seq_len needs");
    }
    uint64_t elems = 0, tmp = 0;
    if (!mul_ok(batch, q_heads, &tmp) || !mul_ok(tmp, c.hd, &elems) || !mul_ok(batch, c.heads, &tmp) ||
        !mul_ok(tmp, c.row_bytes, &elems)) {
        return fail(KVFX_EOVERFLOW, "query or new-token size overflows");
    }
    const uint64_t need = kvfx::decode_workspace_bytes(c, batch, q_heads, max_seq_len, pages_per_split);
    if (need != 0 && (workspace == nullptr || workspace_bytes < need)) {
        return fail(KVFX_ENOSPACE, "decode workspace is smaller than kvfx_decode_workspace_bytes()");
    }
    DeviceScope scope(c.device);
    if (scope.error() != cudaSuccess) return cuda_fail("select device", scope.error());
    kvfx::DecodeArgs a{q, o, block_table, seq_lens, batch, max_blocks_per_seq, max_seq_len,
                       q_heads, pages_per_split, workspace, workspace_bytes};
    a.k_new = k_new;
    a.v_new = v_new;
    a.new_slots = new_slots;
    a.table_out = block_table;
    const cudaError_t e = kvfx::launch_decode(c, a, status_word(c.device), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? KVFX_OK : cuda_fail("batch decode append launch", e);
}

uint64_t kvfx_attention_workspace_bytes(const kvfx_cache* cache, uint64_t query_tokens, uint64_t kv_tokens,
                                        uint32_t q_heads) {
    kvfx::CacheView c;
    if (make_view(cache, &c) != KVFX_OK || q_heads == 0 || q_heads % c.heads != 0) return 0;
    return kvfx::attention_workspace_bytes(c, query_tokens, kv_tokens, q_heads);
}

int kvfx_attention(const kvfx_cache* cache, const float* q, float* o, const uint64_t* blocks,
                   uint64_t query_tokens, uint64_t kv_tokens, uint32_t q_heads, void* workspace,
                   uint64_t workspace_bytes, void* stream) {
    kvfx::CacheView c;
    if (int rc = make_view(cache, &c); rc != KVFX_OK) return rc;
    if (q_heads == 0 || q_heads % c.heads != 0 || query_tokens > kv_tokens) {
        return fail(KVFX_EINVAL, "invalid attention shape");
    }
    if (query_tokens == 0) return KVFX_OK;
    if (q == nullptr || o == nullptr || blocks == nullptr) {
        return fail(KVFX_EINVAL, "q, o and blocks must be non-null");
    }
    uint64_t elems = 0, tmp = 0;
    if (!mul_ok(query_tokens, q_heads, &tmp) || !mul_ok(tmp, c.hd, &elems)) {
        return fail(KVFX_EOVERFLOW, "query size overflows");
    }
    const uint64_t need = kvfx::attention_workspace_bytes(c, query_tokens, kv_tokens, q_heads);
    if (need != 0 && (workspace == nullptr || workspace_bytes < need)) {
        return fail(KVFX_ENOSPACE, "attention workspace is smaller than kvfx_attention_workspace_bytes()");
    }
    DeviceScope scope(c.device);
    if (scope.error() != cudaSuccess) return cuda_fail("select device", scope.error());
    kvfx::AttentionArgs a{q, o, blocks, query_tokens, kv_tokens, q_heads, workspace, workspace_bytes};
    const cudaError_t e = kvfx::launch_attention(c, a, status_word(c.device), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? KVFX_OK : cuda_fail("paged attention launch", e);
}

int kvfx_attention_batch(const kvfx_cache* cache, uint32_t num_seqs, const float* const* q, float* const* o,
                         const uint64_t* block_table, uint64_t max_blocks_per_seq,
                         const uint64_t* query_tokens, const uint64_t* kv_tokens, uint32_t q_heads,
                         void* workspace, uint64_t workspace_bytes, void* stream) {
    kvfx::CacheView c;
    if (int rc = make_view(cache, &c); rc != KVFX_OK) return rc;
    if (num_seqs > KVFX_MAX_PREFILL_SEQS) return fail(KVFX_EINVAL, "more sequences than KVFX_MAX_PREFILL_SEQS");
    if (num_seqs == 0) return KVFX_OK;
    if (q == nullptr || o == nullptr || query_tokens == nullptr || kv_tokens == nullptr) {
        return fail(KVFX_EINVAL, "q, o, query_tokens and kv_tokens must be non-null");
    }
    if (q_heads == 0 || q_heads % c.heads != 0) return fail(KVFX_EINVAL, "invalid attention shape");
    kvfx::AttentionArgs seqs[KVFX_MAX_PREFILL_SEQS];
    uint32_t n = 0;
    uint64_t need = 0;
    for (uint32_t i = 0; i < num_seqs; ++i) {
        const uint64_t qt = query_tokens[i], kt = kv_tokens[i];
        if (qt > kt) return fail(KVFX_EINVAL, "invalid attention shape");
        if (qt == 0) continue;
        if (block_table == nullptr || q[i] == nullptr || o[i] == nullptr) {
            return fail(KVFX_EINVAL, "q, o and block_table must be non-null");
        }
        if (kvfx::ceil_div(kt, c.bs) > max_blocks_per_seq) {
            return fail(KVFX_EINVAL, "a sequence needs more pages than max_blocks_per_seq");
        }
        uint64_t elems = 0, tmp = 0;
        if (!mul_ok(qt, q_heads, &tmp) || !mul_ok(tmp, c.hd, &elems)) {
            return fail(KVFX_EOVERFLOW, "query size overflows");
        }
        if (!mul_ok(i, max_blocks_per_seq, &tmp)) return fail(KVFX_EOVERFLOW, "block table size overflows");
        seqs[n] = kvfx::AttentionArgs{q[i], o[i], block_table + tmp, qt, kt, q_heads, workspace, workspace_bytes};
        need = std::max(need, kvfx::attention_workspace_bytes(c, qt, kt, q_heads));
        ++n;
    }
    // Tensor-core shapes first (stable order), the rest after them.
    const auto tc_end = std::stable_partition(seqs, seqs + n, [&](const kvfx::AttentionArgs& a) {
        return kvfx::prefill_tc_supported(c, a);
    });
    const uint32_t n_tc = static_cast<uint32_t>(tc_end - seqs);
    if (n == 0) return KVFX_OK;
    if (need != 0 && (workspace == nullptr || workspace_bytes < need)) {
        return fail(KVFX_ENOSPACE, "attention workspace is smaller than the largest kvfx_attention_workspace_bytes()");
    }
    DeviceScope scope(c.device);
    if (scope.error() != cudaSuccess) return cuda_fail("select device", scope.error());
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (n_tc != 0) {
        const cudaError_t e = kvfx::launch_prefill_tc_batch(c, seqs, n_tc, status_word(c.device), s);
        if (e != cudaSuccess) return cuda_fail("batched prefill launch", e);
    }
    for (uint32_t i = n_tc; i < n; ++i) {
        const cudaError_t e = kvfx::launch_attention(c, seqs[i], status_word(c.device), s);
        if (e != cudaSuccess) return cuda_fail("paged attention launch", e);
    }
    return KVFX_OK;
}

}  // extern "C"
