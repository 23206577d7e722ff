// Python binding of the C++ v2 API (the drop-in surface), used by the tests,
// the smoke check and the benchmark. Names and argument order follow
// include/kvflux/v2; device buffers are passed as torch tensors, integers
// (raw addresses) or None (a null pointer).
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>

#include "kvflux/v2/batch_block_table.h"
#include "kvflux/v2/batch_decode_session.h"
#include "kvflux/v2/copy_on_write.h"
#include "kvflux/v2/paged_attention.h"
#include "kvflux/v2/paged_kv_layers.h"
#include "kvflux/v2/paged_kv_read.h"
#include "kvflux/v2/paged_kv_storage.h"
#include "kvflux/v2/paged_kv_write.h"
#include "kvflux/v2/prefix_cache.h"
#include "kvflux/v2/reference_attention.h"
#include "kvflux/v2/sequence_lifecycle.h"
#include "kvflux/v2/slot_mapping.h"

namespace py = pybind11;
using namespace kvflux::v2;  // BlockTable below is the v2 class, not the v0 struct
using kvflux::BlockHandle;
using kvflux::BlockManager;
using kvflux::CapacityError;
using kvflux::DType;
using kvflux::KVKind;
using kvflux::PhysicalBlockHandle;
using kvflux::PhysicalBlockPool;
using kvflux::Tokens;

namespace {

// Address of a buffer argument: tensor.data_ptr(), numpy .ctypes.data, an int, or None.
std::uintptr_t address_of(const py::object& o) {
    if (o.is_none()) return 0;
    if (py::hasattr(o, "data_ptr")) return o.attr("data_ptr")().cast<std::uintptr_t>();
    if (py::hasattr(o, "ctypes")) return o.attr("ctypes").attr("data").cast<std::uintptr_t>();
    return o.cast<std::uintptr_t>();
}

template <typename T>
T* ptr(const py::object& o) {
    return reinterpret_cast<T*>(address_of(o));
}

std::vector<TokenWrite> to_writes(const std::vector<std::pair<const SequenceState*, std::size_t>>& batch) {
    std::vector<TokenWrite> out;
    out.reserve(batch.size());
    for (const auto& [s, pos] : batch) out.push_back({s, pos});
    return out;
}

} // namespace

PYBIND11_MODULE(_C, m) {
    m.doc() = "KVFlux v2 paged-KV API on B200 (sm_100a) kernels";

    static py::exception<CapacityError> capacity_error(m, "CapacityError", PyExc_RuntimeError);
    static py::exception<std::logic_error> logic_error(m, "LogicError", PyExc_RuntimeError);
    py::register_exception_translator([](std::exception_ptr p) {
        try {
            if (p) std::rethrow_exception(p);
        } catch (const CapacityError& e) {
            py::set_error(capacity_error, e.what());
        } catch (const std::invalid_argument& e) {
            PyErr_SetString(PyExc_ValueError, e.what());
        } catch (const std::out_of_range& e) {
            PyErr_SetString(PyExc_IndexError, e.what());
        } catch (const std::overflow_error& e) {
            PyErr_SetString(PyExc_OverflowError, e.what());
        } catch (const std::logic_error& e) {
            py::set_error(logic_error, e.what());
        }
    });

    py::enum_<DType>(m, "DType")
        .value("Float16", DType::Float16)
        .value("BFloat16", DType::BFloat16)
        .value("Float32", DType::Float32);
    py::enum_<KVKind>(m, "KVKind").value("Key", KVKind::Key).value("Value", KVKind::Value);

    py::class_<BlockHandle>(m, "BlockHandle")
        .def(py::init([](std::size_t id, std::uint64_t gen) { return BlockHandle{id, gen}; }),
             py::arg("id"), py::arg("generation"))
        .def_readonly("id", &BlockHandle::id)
        .def_readonly("generation", &BlockHandle::generation)
        .def("__eq__", [](const BlockHandle& a, const BlockHandle& b) { return a == b; })
        .def("__repr__", [](const BlockHandle& h) {
            return "BlockHandle(id=" + std::to_string(h.id) + ", generation=" + std::to_string(h.generation) + ")";
        });

    py::class_<PhysicalBlockPool>(m, "PhysicalBlockPool")
        .def(py::init<std::size_t, std::size_t>(), py::arg("capacity"), py::arg("block_size"))
        .def(py::init([](std::size_t capacity, std::size_t block_size, py::function hasher) {
                 BlockManager::Hasher h = [hasher](const Tokens& t) { return hasher(t).cast<std::uint64_t>(); };
                 return new PhysicalBlockPool(capacity, block_size, std::move(h));
             }),
             py::arg("capacity"), py::arg("block_size"), py::arg("hasher"))
        .def("allocate", &PhysicalBlockPool::allocate)
        .def("retain", &PhysicalBlockPool::retain)
        .def("free", &PhysicalBlockPool::free)
        .def("publish", &PhysicalBlockPool::publish)
        .def("lookup", [](PhysicalBlockPool& p, const Tokens& prefix) -> py::object {
            BlockHandle h{};
            if (p.lookup(prefix, h)) return py::cast(h);
            return py::none();
        })
        .def("is_published", &PhysicalBlockPool::is_published)
        .def("id", &PhysicalBlockPool::id)
        .def("ref_count", &PhysicalBlockPool::ref_count)
        .def("capacity", &PhysicalBlockPool::capacity)
        .def("block_size", &PhysicalBlockPool::block_size)
        .def("available", &PhysicalBlockPool::available)
        .def("zero_ref_events", &PhysicalBlockPool::zero_ref_events)
        .def("zero_ref_ids_since", [](const PhysicalBlockPool& p, std::uint64_t since) -> py::object {
            std::vector<std::size_t> ids;
            if (!p.zero_ref_ids_since(since, ids)) return py::none();
            return py::cast(ids);
        });
    m.def("prefix_hash", &BlockManager::prefix_hash);

    py::class_<BlockTable>(m, "BlockTable")
        .def(py::init<PhysicalBlockPool&>(), py::keep_alive<1, 2>())
        .def("append_new", &BlockTable::append_new)
        .def("append_existing", &BlockTable::append_existing)
        .def("append_shared", &BlockTable::append_shared)
        .def("physical_id", &BlockTable::physical_id)
        .def("__getitem__", &BlockTable::physical_id)
        .def("handle", &BlockTable::handle)
        .def("ref_count", &BlockTable::ref_count)
        .def("size", &BlockTable::size)
        .def("__len__", &BlockTable::size)
        .def("empty", &BlockTable::empty)
        .def("shares_pool_with", &BlockTable::shares_pool_with)
        .def("uses_pool", &BlockTable::uses_pool)
        .def("pop_back", &BlockTable::pop_back)
        .def("replace_last_owned", &BlockTable::replace_last_owned)
        .def("clear", &BlockTable::clear)
        .def("lineage", &BlockTable::lineage)
        .def("revision", &BlockTable::revision)
        .def("first_changed_since", &BlockTable::first_changed_since)
        .def("move_from", [](BlockTable& self, BlockTable& other) { self = std::move(other); });

    py::class_<TokenLocation>(m, "TokenLocation")
        .def_readonly("physical_block", &TokenLocation::physical_block)
        .def_readonly("offset_in_block", &TokenLocation::offset_in_block);

    py::class_<SequenceState>(m, "SequenceState")
        .def(py::init<RequestID, PhysicalBlockPool&>(), py::arg("request_id"), py::arg("pool"),
             py::keep_alive<1, 3>())
        .def("request_id", &SequenceState::request_id)
        .def("num_tokens", &SequenceState::num_tokens)
        .def("block_size", &SequenceState::block_size)
        .def("block_table", &SequenceState::block_table, py::return_value_policy::reference_internal)
        .def("num_allocated_blocks", &SequenceState::num_allocated_blocks)
        .def("last_block_num_tokens", &SequenceState::last_block_num_tokens)
        .def("append_tokens", &SequenceState::append_tokens)
        .def("append_token", &SequenceState::append_token)
        .def("fork_shared", &SequenceState::fork_shared, py::keep_alive<0, 1>())
        .def("append_token_with_copy",
             [](SequenceState& s, py::object copier) {
                 if (copier.is_none()) return s.append_token_with_copy({});
                 return s.append_token_with_copy(
                     [copier](PhysicalBlockHandle a, PhysicalBlockHandle b) { copier(a, b); });
             })
        .def("physical_block_id", &SequenceState::physical_block_id)
        .def("token_location", &SequenceState::token_location)
        .def("move_from", [](SequenceState& self, SequenceState& other) { self = std::move(other); });

    py::class_<BatchBlockTable>(m, "BatchBlockTable")
        .def("num_sequences", &BatchBlockTable::num_sequences)
        .def("max_blocks_per_sequence", &BatchBlockTable::max_blocks_per_sequence)
        .def("block_table", &BatchBlockTable::block_table)
        .def("sequence_lengths", &BatchBlockTable::sequence_lengths)
        .def("physical_id", &BatchBlockTable::physical_id)
        .def_static("invalid_block", &BatchBlockTable::invalid_block);
    m.def("build_batch_block_table", &build_batch_block_table);

    m.def("build_slot_mapping", [](const std::vector<std::pair<const SequenceState*, std::size_t>>& batch) {
        return build_slot_mapping(to_writes(batch));
    });
    m.def("build_read_block_table", &build_read_block_table);
    m.def(
        "reference_attention",
        [](const std::vector<float>& q, const std::vector<float>& k, const std::vector<float>& v,
           std::size_t query_tokens, std::size_t kv_tokens, std::size_t query_heads, std::size_t kv_heads,
           std::size_t head_size) {
            return reference_attention(q, k, v, AttentionShape{query_tokens, kv_tokens, query_heads, kv_heads,
                                                               head_size});
        },
        py::arg("query"), py::arg("key"), py::arg("value"), py::arg("query_tokens"), py::arg("kv_tokens"),
        py::arg("query_heads"), py::arg("kv_heads"), py::arg("head_size"));

    py::class_<PagedKVLayout>(m, "PagedKVLayout")
        .def(py::init<std::size_t, std::size_t, std::size_t, std::size_t, DType>())
        .def("num_blocks", &PagedKVLayout::num_blocks)
        .def("num_kv_heads", &PagedKVLayout::num_kv_heads)
        .def("block_size", &PagedKVLayout::block_size)
        .def("head_size", &PagedKVLayout::head_size)
        .def("dtype", &PagedKVLayout::dtype)
        .def("element_bytes", &PagedKVLayout::element_bytes)
        .def("page_bytes", &PagedKVLayout::page_bytes)
        .def("cache_bytes", &PagedKVLayout::cache_bytes)
        .def("total_bytes", &PagedKVLayout::total_bytes)
        .def("slot_count", &PagedKVLayout::slot_count)
        .def("page_byte_offset", &PagedKVLayout::page_byte_offset)
        .def("byte_offset", &PagedKVLayout::byte_offset)
        .def("slot_byte_offset", &PagedKVLayout::slot_byte_offset);

    py::class_<PagedKVStorage>(m, "PagedKVStorage")
        .def(py::init<PhysicalBlockPool&, std::size_t, std::size_t, DType, int>(), py::arg("pool"),
             py::arg("num_kv_heads"), py::arg("head_size"), py::arg("dtype"), py::arg("device") = 0,
             py::keep_alive<1, 2>())
        .def("layout", &PagedKVStorage::layout, py::return_value_policy::reference_internal)
        .def("device", &PagedKVStorage::device)
        .def("uses_pool", &PagedKVStorage::uses_pool)
        .def("key_base", [](const PagedKVStorage& s) { return reinterpret_cast<std::uintptr_t>(s.key_base()); })
        .def("value_base", [](const PagedKVStorage& s) { return reinterpret_cast<std::uintptr_t>(s.value_base()); })
        .def("page_address", [](const PagedKVStorage& s, KVKind k, BlockHandle h) {
            return reinterpret_cast<std::uintptr_t>(s.page_address(k, h));
        })
        .def("element_address", [](const PagedKVStorage& s, KVKind k, BlockHandle h, std::size_t head,
                                   std::size_t token, std::size_t dim) {
            return reinterpret_cast<std::uintptr_t>(s.element_address(k, h, head, token, dim));
        })
        .def("slot_address", [](const PagedKVStorage& s, KVKind k, PhysicalSlot slot, std::size_t head,
                                std::size_t dim) {
            return reinterpret_cast<std::uintptr_t>(s.slot_address(k, slot, head, dim));
        })
        .def("copy_block", &PagedKVStorage::copy_block);

    m.def("write_paged_kv", [](PagedKVStorage& s, py::object k, py::object v, const SlotMapping& slots) {
        write_paged_kv(s, ptr<const void>(k), ptr<const void>(v), slots);
    });
    m.def("read_paged_kv", [](const PagedKVStorage& s, const SequenceState& seq, py::object k, py::object v) {
        read_paged_kv(s, seq, ptr<void>(k), ptr<void>(v));
    });
    m.def("paged_attention", [](const PagedKVStorage& s, const SequenceState& seq, py::object q, py::object o,
                                std::size_t query_tokens, std::size_t query_heads) {
        paged_attention(s, seq, ptr<const float>(q), ptr<float>(o), query_tokens, query_heads);
    });
    m.def("paged_attention_batch", [](const PagedKVStorage& s, const std::vector<const SequenceState*>& seqs,
                                      py::object q, py::object o, std::size_t query_heads) {
        paged_attention_batch(s, seqs, ptr<const float>(q), ptr<float>(o), query_heads);
    });
    m.def("paged_attention_batch_host", [](const PagedKVStorage& s, const std::vector<const SequenceState*>& seqs,
                                           py::object q, py::object o, std::size_t query_heads) {
        paged_attention_batch_host(s, seqs, ptr<const float>(q), ptr<float>(o), query_heads);
    });
    m.def("paged_attention_batch_table_upload_bytes", &paged_attention_batch_table_upload_bytes);
    m.def("paged_attention_prefill_batch",
          [](const PagedKVStorage& s, const std::vector<const SequenceState*>& seqs, const py::list& qs,
             const py::list& os, const std::vector<std::size_t>& query_tokens, std::size_t query_heads) {
              std::vector<const float*> q;
              std::vector<float*> o;
              for (const auto& x : qs) q.push_back(ptr<const float>(py::reinterpret_borrow<py::object>(x)));
              for (const auto& x : os) o.push_back(ptr<float>(py::reinterpret_borrow<py::object>(x)));
              paged_attention_prefill_batch(s, seqs, q, o, query_tokens, query_heads);
          });
    m.def("append_token_cow", &append_token_cow);
    m.def("write_paged_kv_layers", [](const std::vector<PagedKVStorage*>& layers, py::object k, py::object v,
                                      const SlotMapping& slots) {
        write_paged_kv_layers(layers, ptr<const void>(k), ptr<const void>(v), slots);
    });
    m.def("read_paged_kv_layers", [](const std::vector<const PagedKVStorage*>& layers, const SequenceState& seq,
                                     py::object k, py::object v) {
        read_paged_kv_layers(layers, seq, ptr<void>(k), ptr<void>(v));
    });

    py::class_<PrefixCache>(m, "PrefixCache")
        .def(py::init<PhysicalBlockPool&>(), py::keep_alive<1, 2>())
        .def("attach_cached_prefix", &PrefixCache::attach_cached_prefix)
        .def("publish_computed_block", &PrefixCache::publish_computed_block);

    py::class_<BatchDecodeSession>(m, "BatchDecodeSession")
        .def(py::init<const PagedKVStorage&, std::vector<SequenceState*>, std::size_t>(), py::keep_alive<1, 2>(),
             py::keep_alive<1, 3>())
        .def("step", [](BatchDecodeSession& b, py::object k, py::object v, py::object q, py::object o) {
            return b.step(ptr<const void>(k), ptr<const void>(v), ptr<const float>(q), ptr<float>(o));
        })
        .def("step_host", [](BatchDecodeSession& b, py::object k, py::object v, py::object q, py::object o) {
            return b.step_host(ptr<const void>(k), ptr<const void>(v), ptr<const float>(q), ptr<float>(o));
        })
        .def("refresh", &BatchDecodeSession::refresh)
        .def("refresh_all", &BatchDecodeSession::refresh_all)
        .def("batch_size", &BatchDecodeSession::batch_size)
        .def("table_width", &BatchDecodeSession::table_width)
        .def("device_table", [](const BatchDecodeSession& b) {
            return reinterpret_cast<std::uintptr_t>(b.device_table());
        });

    py::class_<SequenceLifecycle>(m, "SequenceLifecycle")
        .def(py::init<RequestID, PhysicalBlockPool&, PagedKVStorage&, std::size_t>(), py::keep_alive<1, 3>(),
             py::keep_alive<1, 4>())
        .def("prefill", [](SequenceLifecycle& l, std::size_t n, py::object k, py::object v, py::object q,
                           py::object o) {
            l.prefill(n, ptr<const void>(k), ptr<const void>(v), ptr<const float>(q), ptr<float>(o));
        })
        .def("decode", [](SequenceLifecycle& l, py::object k, py::object v, py::object q, py::object o) {
            return l.decode(ptr<const void>(k), ptr<const void>(v), ptr<const float>(q), ptr<float>(o));
        })
        .def("finish", &SequenceLifecycle::finish)
        .def("finished", &SequenceLifecycle::finished)
        .def("sequence", &SequenceLifecycle::sequence, py::return_value_policy::reference_internal);
}
