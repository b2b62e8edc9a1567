// Python bindings of the host runtime (module vramancer_b200._runtime).  Every call
// that hashes, XORs, does file or socket I/O releases the GIL.  Memory crosses as
// Python buffers (bytes / bytearray / memoryview / numpy) or as raw (address, nbytes)
// pairs for pinned tensors.
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "runtime.h"

namespace py = pybind11;

namespace {

struct View {
  const uint8_t* p;
  size_t n;
};

View view_of(const py::buffer& b) {
  py::buffer_info info = b.request();
  return View{static_cast<const uint8_t*>(info.ptr), (size_t)(info.size * info.itemsize)};
}

py::bytes digest(const uint8_t d[32]) { return py::bytes(reinterpret_cast<const char*>(d), 32); }

}  // namespace

PYBIND11_MODULE(_runtime, m) {
  m.doc() = "vramancer_b200 host runtime: HMAC-SHA256, XOR parity, file spill, TCP tensor frames, page allocator";

  // ---- crypto
  m.def("sha256", [](py::buffer b) {
    View v = view_of(b);
    uint8_t d[32];
    {
      py::gil_scoped_release nogil;
      vrt::Sha256 s;
      s.update(v.p, v.n);
      s.finish(d);
    }
    return digest(d);
  });
  m.def("hmac_sha256", [](py::bytes key, py::buffer msg) {
    const std::string k = key;
    View v = view_of(msg);
    uint8_t d[32];
    {
      py::gil_scoped_release nogil;
      vrt::hmac_sha256(reinterpret_cast<const uint8_t*>(k.data()), k.size(), v.p, v.n, d);
    }
    return digest(d);
  });
  m.def("hmac_verify", [](py::bytes key, py::buffer msg, py::bytes tag) {
    const std::string k = key, t = tag;
    View v = view_of(msg);
    uint8_t d[32];
    {
      py::gil_scoped_release nogil;
      vrt::hmac_sha256(reinterpret_cast<const uint8_t*>(k.data()), k.size(), v.p, v.n, d);
    }
    return t.size() == 32 && vrt::ct_equal(d, reinterpret_cast<const uint8_t*>(t.data()), 32);
  });
  m.def("hmac_batch", [](py::bytes key, std::vector<py::buffer> msgs, int threads) {
    const std::string k = key;
    std::vector<std::pair<const uint8_t*, size_t>> ms;
    for (auto& b : msgs) {
      View v = view_of(b);
      ms.emplace_back(v.p, v.n);
    }
    std::vector<uint8_t> out(32 * ms.size());
    {
      py::gil_scoped_release nogil;
      vrt::hmac_batch(reinterpret_cast<const uint8_t*>(k.data()), k.size(), ms, out.data(), threads);
    }
    py::list res;
    for (size_t i = 0; i < ms.size(); ++i) res.append(digest(out.data() + 32 * i));
    return res;
  }, py::arg("key"), py::arg("msgs"), py::arg("threads") = 4);

  // ---- parity
  m.def("xor_parity", [](std::vector<py::buffer> shards, int threads) {
    std::vector<const uint8_t*> ps;
    size_t len = 0;
    for (size_t i = 0; i < shards.size(); ++i) {
      View v = view_of(shards[i]);
      if (i == 0) len = v.n;
      if (v.n != len) throw std::invalid_argument("xor_parity: shards must have equal length");
      ps.push_back(v.p);
    }
    py::bytearray out(std::string(len, '\0'));
    auto* o = reinterpret_cast<uint8_t*>(PyByteArray_AsString(out.ptr()));
    {
      py::gil_scoped_release nogil;
      vrt::xor_parity(ps, len, o, threads);
    }
    return out;
  }, py::arg("shards"), py::arg("threads") = 4);
  m.def("xor_parity_ptr", [](std::vector<uintptr_t> shards, size_t len, uintptr_t out, int threads) {
    std::vector<const uint8_t*> ps;
    for (auto a : shards) ps.push_back(reinterpret_cast<const uint8_t*>(a));
    py::gil_scoped_release nogil;
    vrt::xor_parity(ps, len, reinterpret_cast<uint8_t*>(out), threads);
  }, py::arg("shards"), py::arg("nbytes"), py::arg("out"), py::arg("threads") = 4);

  // ---- file spill
  m.def("file_write", [](const std::string& path, uintptr_t ptr, size_t n, size_t offset, bool direct, bool sync) {
    py::gil_scoped_release nogil;
    return vrt::file_write(path, reinterpret_cast<const void*>(ptr), n, offset, direct, sync);
  }, py::arg("path"), py::arg("ptr"), py::arg("nbytes"), py::arg("offset") = 0, py::arg("direct") = false,
        py::arg("sync") = false);
  m.def("file_read", [](const std::string& path, uintptr_t ptr, size_t n, size_t offset, bool direct) {
    py::gil_scoped_release nogil;
    return vrt::file_read(path, reinterpret_cast<void*>(ptr), n, offset, direct);
  }, py::arg("path"), py::arg("ptr"), py::arg("nbytes"), py::arg("offset") = 0, py::arg("direct") = false);
  py::class_<vrt::AsyncIO>(m, "AsyncIO")
      .def(py::init<int>(), py::arg("workers") = 4)
      .def("submit_write", [](vrt::AsyncIO& io, const std::string& path, uintptr_t ptr, size_t n, size_t off,
                              bool direct) { return io.submit_write(path, reinterpret_cast<const void*>(ptr), n, off, direct); },
           py::arg("path"), py::arg("ptr"), py::arg("nbytes"), py::arg("offset") = 0, py::arg("direct") = false)
      .def("submit_read", [](vrt::AsyncIO& io, const std::string& path, uintptr_t ptr, size_t n, size_t off,
                             bool direct) { return io.submit_read(path, reinterpret_cast<void*>(ptr), n, off, direct); },
           py::arg("path"), py::arg("ptr"), py::arg("nbytes"), py::arg("offset") = 0, py::arg("direct") = false)
      .def("wait", [](vrt::AsyncIO& io, int64_t t) {
        py::gil_scoped_release nogil;
        return io.wait(t);
      })
      .def("done", &vrt::AsyncIO::done)
      .def("pending", &vrt::AsyncIO::pending);

  // ---- transport
  py::class_<vrt::Connection>(m, "Connection")
      .def("send_frame", [](vrt::Connection& c, py::bytes header, uintptr_t ptr, uint64_t n, py::bytes key,
                            uint32_t chunk) {
        const std::string h = header, k = key;
        py::gil_scoped_release nogil;
        c.send_frame(h, reinterpret_cast<const uint8_t*>(ptr), n, k, chunk);
      }, py::arg("header"), py::arg("ptr"), py::arg("nbytes"), py::arg("key") = py::bytes(""),
           py::arg("chunk") = 16u << 20)
      .def("recv_frame", [](vrt::Connection& c, py::bytes key) {
        const std::string k = key;
        py::object holder;
        uint64_t n = 0;
        std::string header;
        {
          py::gil_scoped_release nogil;
          header = c.recv_frame(k, [&](uint64_t size) -> uint8_t* {
            py::gil_scoped_acquire gil;
            holder = py::bytearray(std::string((size_t)size, '\0'));
            return reinterpret_cast<uint8_t*>(PyByteArray_AsString(holder.ptr()));
          }, &n);
        }
        return py::make_tuple(py::bytes(header), holder);
      }, py::arg("key") = py::bytes(""))
      .def("close", &vrt::Connection::close)
      .def_property_readonly("fd", &vrt::Connection::fd);
  m.def("connect", [](const std::string& host, int port, double timeout) {
    py::gil_scoped_release nogil;
    return vrt::tcp_connect(host, port, timeout);
  }, py::arg("host"), py::arg("port"), py::arg("timeout") = 30.0, py::return_value_policy::take_ownership);
  py::class_<vrt::Listener>(m, "Listener")
      .def(py::init<const std::string&, int>(), py::arg("host") = "127.0.0.1", py::arg("port") = 0)
      .def("accept", [](vrt::Listener& l, double timeout) {
        py::gil_scoped_release nogil;
        return l.accept(timeout);
      }, py::arg("timeout") = -1.0, py::return_value_policy::take_ownership)
      .def_property_readonly("port", &vrt::Listener::port)
      .def("close", &vrt::Listener::close);

  // ---- pages
  py::class_<vrt::PageAllocator>(m, "PageAllocator")
      .def(py::init<int64_t>())
      .def("alloc", &vrt::PageAllocator::alloc)
      .def("incref", &vrt::PageAllocator::incref)
      .def("decref", &vrt::PageAllocator::decref)
      .def("free_all", &vrt::PageAllocator::free_all)
      .def("refcount", &vrt::PageAllocator::refcount)
      .def_property_readonly("num_free", &vrt::PageAllocator::num_free)
      .def_property_readonly("num_pages", &vrt::PageAllocator::num_pages);

  // ---- prompt-lookup drafts
  py::class_<vrt::NgramIndex>(m, "NgramIndex")
      .def(py::init<int, int>(), py::arg("max_n") = 3, py::arg("min_n") = 1)
      .def("extend", [](vrt::NgramIndex& ix, const std::vector<int32_t>& toks) { ix.extend(toks.data(), toks.size()); })
      .def("draft", &vrt::NgramIndex::draft, py::arg("num_draft"))
      .def("__len__", &vrt::NgramIndex::size);

  // ---- tokenizer
  m.def("basic_tokenize", [](const std::vector<std::string>& texts, int32_t vocab, int threads) {
    py::gil_scoped_release nogil;
    return vrt::basic_tokenize(texts, vocab, threads);
  }, py::arg("texts"), py::arg("vocab"), py::arg("threads") = 4);
}
