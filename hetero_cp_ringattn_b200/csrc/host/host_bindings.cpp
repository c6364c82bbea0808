// Python module `hetero_cp_ringattn_b200._host`: bindings of the host runtime library.
// C++ RingError / CapacityError surface as the package's own exception classes.
#include <algorithm>
#include <cstring>

#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "hcp_host.h"

namespace py = pybind11;
using namespace hcp::host;

namespace {

py::array_t<int64_t> ToArray(const std::vector<int64_t>& v) {
  py::array_t<int64_t> a(py::ssize_t(v.size()));
  if (!v.empty()) std::memcpy(a.mutable_data(), v.data(), v.size() * sizeof(int64_t));
  return a;
}

std::vector<int64_t> FromArray(const py::array_t<int64_t, py::array::c_style | py::array::forcecast>& a) {
  return std::vector<int64_t>(a.data(), a.data() + a.size());
}

using I64Arr = py::array_t<int64_t, py::array::c_style | py::array::forcecast>;
using F32Arr = py::array_t<float, py::array::c_style | py::array::forcecast>;

std::vector<int64_t> ToVec(const py::handle& obj) {
  I64Arr a = I64Arr::ensure(obj);
  if (!a) throw ProtocolError("expected an integer array");
  return std::vector<int64_t>(a.data(), a.data() + a.size());
}

Field ToField(FieldKind k, const py::handle& v) {
  Field f;
  f.kind = k;
  const bool none = v.is_none();
  switch (k) {
    case FieldKind::kI64: f.i = py::cast<int64_t>(v); break;
    case FieldKind::kF64: f.f = py::cast<double>(v); break;
    case FieldKind::kBool: f.i = py::cast<bool>(v) ? 1 : 0; break;
    case FieldKind::kStr: f.s = py::cast<std::string>(v); break;
    case FieldKind::kI64Array: f.a = ToVec(v); break;
    case FieldKind::kPairs:
      f.a = ToVec(v);
      if (f.a.size() % 2) throw ProtocolError("pairs field needs rows of two integers");
      break;
    case FieldKind::kOptI64:
      f.present = !none;
      if (!none) f.i = py::cast<int64_t>(v);
      break;
    case FieldKind::kOptI64Array:
      f.present = !none;
      if (!none) f.a = ToVec(v);
      break;
    case FieldKind::kOptF32Array:
      f.present = !none;
      if (!none) {
        F32Arr a = F32Arr::ensure(v);
        if (!a) throw ProtocolError("expected a float array");
        f.fa.assign(a.data(), a.data() + a.size());
      }
      break;
  }
  return f;
}

py::object FromField(const Field& f) {
  auto arr = [](const std::vector<int64_t>& v) { return py::object(ToArray(v)); };
  switch (f.kind) {
    case FieldKind::kI64: return py::int_(f.i);
    case FieldKind::kF64: return py::float_(f.f);
    case FieldKind::kBool: return py::bool_(f.i != 0);
    case FieldKind::kStr: return py::str(f.s);
    case FieldKind::kI64Array: return arr(f.a);
    case FieldKind::kPairs: {
      py::array_t<int64_t> a({py::ssize_t(f.a.size() / 2), py::ssize_t(2)});
      if (!f.a.empty()) std::memcpy(a.mutable_data(), f.a.data(), f.a.size() * sizeof(int64_t));
      return a;
    }
    case FieldKind::kOptI64: return f.present ? py::object(py::int_(f.i)) : py::none();
    case FieldKind::kOptI64Array: return f.present ? arr(f.a) : py::none();
    case FieldKind::kOptF32Array: {
      if (!f.present) return py::none();
      py::array_t<float> a(py::ssize_t(f.fa.size()));
      if (!f.fa.empty()) std::memcpy(a.mutable_data(), f.fa.data(), f.fa.size() * sizeof(float));
      return a;
    }
  }
  return py::none();
}

void RaiseAs(const char* cls_name, const char* what) {
  py::object cls = py::module_::import("hetero_cp_ringattn_b200.errors").attr(cls_name);
  PyErr_SetString(cls.ptr(), what);
}

}  // namespace

PYBIND11_MODULE(_host, m) {
  m.doc() = "host runtime: ring layouts, capacity chunking and admission, KV growth schedule, "
            "page allocator, batch scheduler core";
  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const ProtocolError& e) {
      RaiseAs("ProtocolError", e.what());
    } catch (const CapacityError& e) {
      RaiseAs("CapacityError", e.what());
    } catch (const RingError& e) {
      RaiseAs("RingError", e.what());
    }
  });
  m.attr("UNKNOWN_CAPACITY") = py::int_(kUnknownCapacity);

  // layouts
  m.def("build_assignment", [](const std::vector<int64_t>& chunks, const std::string& strategy) {
    return ToArray(BuildAssignment(chunks, ParseStrategy(strategy)));
  }, py::arg("chunks"), py::arg("strategy"));
  m.def("build_domain_positions",
        [](const py::array_t<int64_t, py::array::c_style | py::array::forcecast>& a, int64_t n) {
          py::list out;
          for (const auto& v : BuildDomainPositions(FromArray(a), n)) out.append(ToArray(v));
          return out;
        }, py::arg("assignment"), py::arg("num_domains") = -1);
  m.def("build_inverse_perm",
        [](const py::array_t<int64_t, py::array::c_style | py::array::forcecast>& a) {
          return ToArray(BuildInversePerm(FromArray(a)));
        }, py::arg("assignment"));

  // capacity
  m.def("allocate_by_capacity", &AllocateByCapacity, py::arg("prompt_len"), py::arg("capacities"));
  m.def("equal_chunks", &EqualChunks, py::arg("prompt_len"), py::arg("n"));
  m.def("chunk_sizes", &ChunkSizes, py::arg("prompt_len"), py::arg("num_domains"),
        py::arg("explicit_sizes"), py::arg("capacities_mb"), py::arg("capacity_aware"),
        py::arg("ratio"), py::arg("activation_reserve_mb"));
  m.def("continuation_split", &ContinuationSplit, py::arg("segment_len"), py::arg("tickets"));
  m.def("capacity_mb_to_bytes", &CapacityMbToBytes, py::arg("capacity_mb"));
  m.def("admit_reserved_kv_bytes",
        [](const std::vector<std::vector<uint64_t>>& caps, const std::vector<uint64_t>& budgets,
           uint64_t hkv, uint64_t d, uint64_t elem) {
          auto a = AdmitReservedKvBytes(caps, budgets, hkv, d, elem);
          return py::make_tuple(a.bytes_per_token_per_layer, a.required_bytes_per_domain);
        });
  py::class_<KvLedger>(m, "KvLedger")
      .def(py::init<std::vector<uint64_t>>(), py::arg("budgets"))
      .def("try_reserve", &KvLedger::TryReserve, py::arg("request_id"), py::arg("bytes_per_domain"))
      .def("release", &KvLedger::Release, py::arg("request_id"))
      .def("free_bytes", &KvLedger::FreeBytes)
      .def("holds", &KvLedger::Holds)
      .def_property_readonly("used", &KvLedger::Used)
      .def_property_readonly("budgets", &KvLedger::Budgets);

  // schedule
  py::class_<FrozenKvAssigneeSchedule>(m, "FrozenKvAssigneeSchedule")
      .def(py::init<const std::vector<uint64_t>&, uint64_t, uint64_t>(), py::arg("tickets"),
           py::arg("request_id"), py::arg("total_units"))
      .def("assignee_for",
           [](const FrozenKvAssigneeSchedule& s, int64_t t, int64_t l, int64_t n) -> py::object {
             const int64_t a = s.AssigneeFor(t, l, n);
             return a < 0 ? py::none() : py::object(py::int_(a));
           })
      .def("per_rank_units", &FrozenKvAssigneeSchedule::PerRankUnits)
      .def_property_readonly("sequence", &FrozenKvAssigneeSchedule::Sequence)
      .def_property_readonly("counts", &FrozenKvAssigneeSchedule::Counts)
      .def_property_readonly("phase", &FrozenKvAssigneeSchedule::Phase)
      .def("total_units", [](const FrozenKvAssigneeSchedule& s) { return s.Sequence().size(); });
  m.def("assignee_table",
        [](const std::vector<uint64_t>& tickets, uint64_t rid, int64_t horizon, int64_t layers) {
          auto v = AssigneeTable(tickets, rid, horizon, layers);
          py::array_t<int64_t> a({py::ssize_t(std::max<int64_t>(horizon, 0)),
                                  py::ssize_t(std::max<int64_t>(layers, 0))});
          if (!v.empty()) std::memcpy(a.mutable_data(), v.data(), v.size() * sizeof(int64_t));
          return a;
        }, py::arg("tickets"), py::arg("request_id"), py::arg("horizon"), py::arg("layers"));
  m.def("stationary_layer_starters", &StationaryLayerStarters, py::arg("initial_starter"),
        py::arg("layers"), py::arg("domains"));

  // pages
  py::class_<PageAllocator>(m, "PageAllocator")
      .def(py::init<int64_t, int64_t>(), py::arg("num_pages"), py::arg("page_size"))
      .def("alloc", &PageAllocator::Alloc, py::arg("n"), py::arg("request_id"))
      .def("free", &PageAllocator::Free, py::arg("pages"))
      .def("owner_of", &PageAllocator::OwnerOf)
      .def_property_readonly("free_pages", &PageAllocator::FreePages)
      .def_property_readonly("num_pages", &PageAllocator::NumPages)
      .def_property_readonly("page_size", &PageAllocator::PageSize);

  // control protocol frames
  m.attr("PROTOCOL_VERSION") = py::int_(kProtocolVersion);
  m.def("message_schema", [](int type) { return std::string(MessageSchema(type)); });
  m.def("encode_frame", [](int type, const py::sequence& values) {
    const std::string kinds = MessageSchema(type);
    if (kinds.empty() && type != 8) throw ProtocolError("not a protocol message type");
    if (size_t(py::len(values)) != kinds.size())
      throw ProtocolError("message type " + std::to_string(type) + " takes " +
                          std::to_string(kinds.size()) + " fields");
    std::vector<Field> fields;
    for (size_t k = 0; k < kinds.size(); ++k) fields.push_back(ToField(FieldKind(kinds[k]), values[k]));
    return py::bytes(EncodeFrame(type, fields));
  }, py::arg("type"), py::arg("values"));
  m.def("decode_frame", [](const py::bytes& frame) {
    int type = 0;
    const auto fields = DecodeFrame(std::string(frame), &type);
    py::list out;
    for (const auto& f : fields) out.append(FromField(f));
    return py::make_tuple(type, out);
  }, py::arg("frame"));

  // f64 attention oracle: q [L, H, D], k / v [L, Hkv, D] float64 arrays
  using F64Arr = py::array_t<double, py::array::c_style | py::array::forcecast>;
  auto vec3 = [](const F64Arr& a, int64_t* L, int64_t* H, int64_t* D) {
    if (a.ndim() != 3) throw RingError("attention oracle: expected a [L, heads, D] array");
    *L = a.shape(0);
    *H = a.shape(1);
    *D = a.shape(2);
    return std::vector<double>(a.data(), a.data() + a.size());
  };
  auto result = [](const AttnResult& r, int64_t L, int64_t H, int64_t D) {
    py::array_t<double> o({py::ssize_t(L), py::ssize_t(H), py::ssize_t(D)});
    py::array_t<double> lse({py::ssize_t(H), py::ssize_t(L)});
    if (!r.o.empty()) std::memcpy(o.mutable_data(), r.o.data(), r.o.size() * sizeof(double));
    if (!r.lse.empty()) std::memcpy(lse.mutable_data(), r.lse.data(), r.lse.size() * sizeof(double));
    return py::make_tuple(o, lse);
  };
  m.def("attention_f64", [vec3, result](const F64Arr& q, const F64Arr& k, const F64Arr& v, bool causal) {
    int64_t L, H, D, Lk, Hkv, Dk;
    auto qv = vec3(q, &L, &H, &D), kv = vec3(k, &Lk, &Hkv, &Dk), vv = vec3(v, &Lk, &Hkv, &Dk);
    return result(FullAttentionF64(qv, kv, vv, L, H, Hkv, D, causal), L, H, D);
  }, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("causal"));
  m.def("ring_attention_f64", [vec3, result](const F64Arr& q, const F64Arr& k, const F64Arr& v,
                                             const py::list& positions,
                                             const std::vector<int64_t>& block_sizes, bool causal) {
    int64_t L, H, D, Lk, Hkv, Dk;
    auto qv = vec3(q, &L, &H, &D), kv = vec3(k, &Lk, &Hkv, &Dk), vv = vec3(v, &Lk, &Hkv, &Dk);
    std::vector<std::vector<int64_t>> pos;
    for (const auto& p : positions) pos.push_back(ToVec(p));
    return result(RingAttentionF64(qv, kv, vv, L, H, Hkv, D, pos, block_sizes, causal), L, H, D);
  }, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("positions"), py::arg("block_sizes"),
     py::arg("causal"));

  // scheduler core
  py::class_<BatchSchedulerCore>(m, "BatchSchedulerCore")
      .def(py::init<int64_t>(), py::arg("max_batch_size"))
      .def("enqueue", &BatchSchedulerCore::Enqueue)
      .def("pop_pending",
           [](BatchSchedulerCore& s) -> py::object {
             auto v = s.PopPending();
             return v ? py::object(py::int_(*v)) : py::none();
           })
      .def("requeue_front", &BatchSchedulerCore::RequeueFront)
      .def("activate", &BatchSchedulerCore::Activate)
      .def("complete", &BatchSchedulerCore::Complete)
      .def("has_capacity", &BatchSchedulerCore::HasCapacity)
      .def("active", &BatchSchedulerCore::Active)
      .def_property_readonly("queued", &BatchSchedulerCore::Queued)
      .def_property_readonly("num_active", &BatchSchedulerCore::NumActive)
      .def_property_readonly("max_batch_size", &BatchSchedulerCore::MaxBatchSize)
      .def("wait_for_work", &BatchSchedulerCore::WaitForWork, py::arg("timeout_s"),
           py::call_guard<py::gil_scoped_release>());
}
