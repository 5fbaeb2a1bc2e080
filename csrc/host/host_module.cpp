// Python bindings of the native host cores (module lunaflux_b200._host).
//
//   PageAllocator  page_allocator.hpp  generational KV page allocator
//   BpeEncoder     bpe.hpp             byte-level BPE merge loop
//   Channel        channel.hpp         framed supervisor <-> rank control channel
//   ApprovedRoot   approved_fs.hpp     no-follow file access under an approved root
//
// Blocking calls (channel I/O, file reads) release the GIL.  The cores are
// plain C++ with no Python dependency; csrc/host/selftest/ runs them under
// AddressSanitizer and UndefinedBehaviorSanitizer.
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "approved_fs.hpp"
#include "bpe.hpp"
#include "channel.hpp"
#include "page_allocator.hpp"

namespace py = pybind11;

namespace {

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
