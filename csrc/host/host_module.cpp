// Python bindings of the native host cores (module lunaflux_b200._host).
//
//   PageAllocator  page_allocator.hpp  generational KV page allocator
//   BlockTables    block_table.hpp     per-request block tables + the dense page matrix
//   PrefixTree     prefix_tree.hpp     radix prefix cache over full KV pages
//   BpeEncoder     bpe.hpp             byte-level BPE merge loop
//   Channel        channel.hpp         framed supervisor <-> rank control channel
//   ApprovedRoot   approved_fs.hpp     no-follow file access under an approved root
//
// Blocking calls (channel I/O, file reads) release the GIL.  The cores are
// plain C++ with no Python dependency; csrc/host/selftest/ runs them under
// AddressSanitizer and UndefinedBehaviorSanitizer.
#include <pybind11/functional.h>
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "approved_fs.hpp"
#include "block_table.hpp"
#include "bpe.hpp"
#include "channel.hpp"
#include "page_allocator.hpp"
#include "prefix_tree.hpp"

namespace py = pybind11;

namespace {

// Page i of a token sequence given as a Python list / tuple of ints or as a
// buffer of int32: sequences are read one page at a time, so a prefix walk
// that stops at its first mismatch converts only the pages it compared.
class TokenPages {
 public:
  TokenPages(py::handle seq, int P) : P_(P), page_(P) {
    if (py::isinstance<py::array>(seq)) {
      arr_ = py::array_t<int32_t, py::array::c_style | py::array::forcecast>::ensure(seq);
      if (!arr_) throw py::type_error("tokens: int32 array expected");
      is_array_ = true;
      n_ = arr_.size();
    } else {
      fast_ = py::reinterpret_steal<py::object>(PySequence_Fast(seq.ptr(), "tokens: a sequence of ints"));
      if (!fast_) throw py::error_already_set();
      n_ = PySequence_Fast_GET_SIZE(fast_.ptr());
    }
  }
  int64_t size() const { return n_; }
  const int32_t* operator()(int64_t i) {
    if (is_array_) return arr_.data() + i * P_;
    PyObject** items = PySequence_Fast_ITEMS(fast_.ptr());
    for (int j = 0; j < P_; ++j) {
      const long v = PyLong_AsLong(items[i * P_ + j]);
      if (v == -1 && PyErr_Occurred()) throw py::error_already_set();
      page_[j] = (int32_t)v;
    }
    return page_.data();
  }

 private:
  int P_;
  std::vector<int32_t> page_;
  py::array_t<int32_t, py::array::c_style | py::array::forcecast> arr_;
  py::object fast_;
  bool is_array_ = false;  // (a default array_t is an empty array, not a null handle)
  int64_t n_ = 0;
};

py::tuple stamp_tuple(const lf_host::Stamp& s) {
  return py::make_tuple(s.dev, s.ino, s.size, s.mtime_ns, s.ctime_ns);
}

}  // namespace

PYBIND11_MODULE(_host, m) {
  using namespace lf_host;
  m.doc() = "LunaFlux native host cores";
  auto page_err = py::register_exception<PageError>(m, "PageError", PyExc_RuntimeError);
  py::register_exception<OutOfPages>(m, "OutOfPages", page_err.ptr());
  auto chan_closed = py::register_exception<ChannelClosed>(m, "ChannelClosed", PyExc_ConnectionError);
  py::register_exception<ChannelTimeout>(m, "ChannelTimeout", PyExc_TimeoutError);
  py::register_exception<ApprovedFsError>(m, "ApprovedFsError", PyExc_OSError);
  py::register_exception<BlockTableError>(m, "BlockTableError", PyExc_RuntimeError);
  py::register_exception<PrefixError>(m, "PrefixError", PyExc_RuntimeError);
  (void)chan_closed;

  py::class_<PageAllocator>(m, "PageAllocator")
      .def(py::init<int, int, int64_t, int, int>())
      .def("free_page_count", &PageAllocator::free_page_count)
      .def("allocated_page_count", &PageAllocator::allocated_page_count)
      .def("retired_page_count", &PageAllocator::retired_page_count)
      .def("capacity", &PageAllocator::capacity)
      .def("allocate_run", &PageAllocator::allocate_run)
      .def("retain_active", &PageAllocator::retain_active)
      .def("release_active", &PageAllocator::release_active)
      .def("check_release_active", &PageAllocator::check_release_active)
      .def("retain_cached", &PageAllocator::retain_cached)
      .def("release_cached", &PageAllocator::release_cached)
      .def("active_reference_count", &PageAllocator::active_reference_count)
      .def("cached_reference_count", &PageAllocator::cached_reference_count)
      .def("validate_active", &PageAllocator::validate_active)
      .def("checkpoint", &PageAllocator::checkpoint)
      .def("commit_checkpoint", &PageAllocator::commit_checkpoint)
      .def("rollback_to", &PageAllocator::rollback_to)
      .def("free_queue", &PageAllocator::free_queue)
      .def("debug_check_invariants", &PageAllocator::debug_check_invariants);

  py::class_<BlockTableArena>(m, "BlockTables")
      .def(py::init<int, int, int>())
      .def("free_table_count", &BlockTableArena::free_table_count)
      .def("allocated_table_count", &BlockTableArena::allocated_table_count)
      .def("allocate", &BlockTableArena::allocate)
      .def("release", &BlockTableArena::release)
      .def("page_count", &BlockTableArena::page_count)
      .def("pages", &BlockTableArena::pages)
      .def("append_pages", &BlockTableArena::append_pages)
      .def("page_at", &BlockTableArena::page_at)
      .def("resolve_token_position", &BlockTableArena::resolve_token_position)
      .def("truncate", &BlockTableArena::truncate, py::arg("idx"), py::arg("gen"), py::arg("keep"),
           py::arg("alloc").none(true))
      .def("reset_and_release", &BlockTableArena::reset_and_release, py::arg("idx"), py::arg("gen"),
           py::arg("alloc").none(true))
      .def("checkpoint", &BlockTableArena::checkpoint)
      .def("note", &BlockTableArena::note)
      .def("commit_checkpoint", &BlockTableArena::commit_checkpoint)
      .def("rollback", &BlockTableArena::rollback)
      .def("debug_check_invariants", &BlockTableArena::debug_check_invariants)
      // numpy view of the arena's own int32 [capacity, max_pages] matrix (no copy; keeps the arena alive)
      .def("matrix", [](py::object self) {
        auto& a = self.cast<BlockTableArena&>();
        return py::array_t<int32_t>({(py::ssize_t)a.capacity(), (py::ssize_t)a.max_pages()},
                                    {(py::ssize_t)(a.max_pages() * sizeof(int32_t)), (py::ssize_t)sizeof(int32_t)},
                                    a.matrix_data(), self);
      });

  py::class_<PrefixTree>(m, "PrefixTree")
      .def(py::init<PageAllocator&, int, int64_t>(), py::keep_alive<1, 2>())
      .def("new_root", &PrefixTree::new_root)
      .def("lookup",
           [](PrefixTree& t, int root, py::handle toks, int64_t max_pages) {
             TokenPages src(toks, t.tokens_per_page());
             return t.lookup_with(root, src.size(), max_pages, src);
           })
      .def("insert",
           [](PrefixTree& t, int root, py::handle toks, const std::vector<PrefixTree::Page>& pages) {
             TokenPages src(toks, t.tokens_per_page());
             return t.insert_with(root, src.size(), pages, src);
           })
      .def("retain", &PrefixTree::retain)
      .def("release", &PrefixTree::release)
      .def("evict", &PrefixTree::evict)
      .def("page", &PrefixTree::page)
      .def("pages_of", &PrefixTree::pages_of)
      .def("page_count", &PrefixTree::page_count)
      .def("evictable_pages", &PrefixTree::evictable_pages)
      .def("stats", [](const PrefixTree& t) {
        return py::make_tuple(t.hits(), t.lookups(), t.hit_tokens(), t.evicted_pages());
      })
      .def("debug_check_invariants", &PrefixTree::debug_check_invariants);

  py::class_<BpeEncoder>(m, "BpeEncoder")
      .def(py::init<const std::vector<std::tuple<int, int, int>>&>())
      .def("encode", &BpeEncoder::encode, py::call_guard<py::gil_scoped_release>());

  py::class_<Channel>(m, "Channel")
      .def(py::init<int, uint32_t, double>(), py::arg("fd"), py::arg("max_frame") = 64u << 20,
           py::arg("frame_timeout_s") = 10.0)
      .def("fileno", &Channel::fileno)
      .def_property_readonly("closed", &Channel::closed)
      .def("close", &Channel::close)
      .def(
          "send",
          [](Channel& c, const py::bytes& payload, double timeout_s) {
            std::string s = payload;
            py::gil_scoped_release nogil;
            c.send(s, timeout_s);
          },
          py::arg("payload"), py::arg("timeout_s") = 10.0)
      .def(
          "recv",
          [](Channel& c, double timeout_s) -> py::object {
            std::optional<std::string> got;
            {
              py::gil_scoped_release nogil;
              got = c.recv(timeout_s);
            }
            if (!got) return py::none();
            return py::bytes(*got);
          },
          py::arg("timeout_s"));

  py::class_<ApprovedRoot>(m, "ApprovedRoot")
      .def(py::init<const std::string&>())
      .def("close", &ApprovedRoot::close)
      .def("identity", [](const ApprovedRoot& r) { return stamp_tuple(r.identity()); })
      .def("stat", [](const ApprovedRoot& r, const std::string& loc) { return stamp_tuple(r.stat(loc)); })
      .def("read_snapshot",
           [](const ApprovedRoot& r, const std::string& loc, int64_t max_bytes) {
             PyObject* obj = nullptr;
             Stamp st;
             try {
               py::gil_scoped_release nogil;
               st = r.read_snapshot(loc, max_bytes, [&](int64_t n) -> uint8_t* {
                 py::gil_scoped_acquire gil;
                 obj = PyBytes_FromStringAndSize(nullptr, (Py_ssize_t)n);
                 if (obj == nullptr) throw std::bad_alloc();
                 return reinterpret_cast<uint8_t*>(PyBytes_AS_STRING(obj));
               });
             } catch (...) {
               Py_XDECREF(obj);
               throw;
             }
             return py::make_tuple(py::reinterpret_steal<py::bytes>(obj), stamp_tuple(st));
           })
      .def("read_into",
           [](const ApprovedRoot& r, const std::string& loc, py::buffer buf) {
             py::buffer_info info = buf.request(/*writable=*/true);
             const int64_t cap = info.size * info.itemsize;
             uint8_t* base = static_cast<uint8_t*>(info.ptr);
             Stamp st;
             {
               py::gil_scoped_release nogil;
               st = r.read_snapshot(loc, cap, [&](int64_t) { return base; });
             }
             return stamp_tuple(st);
           });
}
