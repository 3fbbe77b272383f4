// Bindings of the stage-pack checkpoint layout (submodule `stagepack`). Data and
// destination buffers are integer addresses (a tensor's data_ptr()); the caller keeps
// them alive for the call. Reads release the interpreter lock.
#include "registry.h"
#include "stagepack.h"

namespace py = pybind11;
using namespace spc;

static void* ptr(uint64_t a) { return reinterpret_cast<void*>(uintptr_t(a)); }

static BindRegistrar reg([](py::module_& m) {
  auto s = m.def_submodule("stagepack", "checkpoint layout: index + aligned tensor regions");
  s.attr("INDEX_FILE") = pack::kIndexFile;
  s.attr("FORMAT") = pack::kFormat;
  s.attr("ALIGN") = pack::kAlign;
  s.def("fingerprint", [](uint64_t addr, uint64_t n) { return pack::fingerprint(ptr(addr), size_t(n)); });
  py::class_<pack::Region>(s, "Region")
      .def_readonly("file_path", &pack::Region::file_path)
      .def_readonly("file_offset", &pack::Region::file_offset)
      .def_readonly("tensor_bytes", &pack::Region::tensor_bytes);
  py::class_<pack::Writer>(s, "Writer")
      .def(py::init<const std::string&, const std::string&, const std::string&>(), py::arg("root"),
           py::arg("model_id"), py::arg("metadata_json") = "{}")
      .def("add",
           [](pack::Writer& w, const std::string& name, const std::string& dtype, const std::vector<uint64_t>& shape,
              uint64_t bpe, uint64_t addr, uint64_t bytes) {
             py::gil_scoped_release nogil;
             w.add(name, dtype, shape, bpe, ptr(addr), bytes);
           },
           py::arg("name"), py::arg("dtype"), py::arg("shape"), py::arg("bytes_per_element"), py::arg("address"),
           py::arg("bytes"))
      .def("finish", &pack::Writer::finish)
      .def_property_readonly("bytes_written", &pack::Writer::bytes_written);
  py::class_<pack::Pack>(s, "Pack")
      .def_static("open", &pack::Pack::open)
      .def_property_readonly("model_id", &pack::Pack::model_id)
      .def_property_readonly("metadata", &pack::Pack::metadata)
      .def("names", &pack::Pack::names)
      .def("entry",
           [](const pack::Pack& p, const std::string& name) {
             const pack::Entry& e = p.entry(name);
             py::dict d;
             d["name"] = e.name;
             d["dtype"] = e.dtype;
             d["shape"] = e.shape;
             d["bytes_per_element"] = e.bytes_per_element;
             d["file"] = e.file;
             d["offset"] = e.offset;
             d["bytes"] = e.bytes;
             d["fingerprint"] = e.fingerprint;
             return d;
           })
      .def("resolve", &pack::Pack::resolve, py::arg("name"), py::arg("dtype"), py::arg("shape"),
           py::arg("bytes_per_element"))
      .def("read",
           [](const pack::Pack& p, const std::string& name, uint64_t addr, uint64_t bytes, bool verify) {
             py::gil_scoped_release nogil;
             p.read(name, ptr(addr), bytes, verify);
           },
           py::arg("name"), py::arg("address"), py::arg("bytes"), py::arg("verify") = false)
      .def("read_rows",
           [](const pack::Pack& p, const std::string& name, uint64_t row0, uint64_t rows, uint64_t addr,
              uint64_t bytes) {
             py::gil_scoped_release nogil;
             p.read_rows(name, row0, rows, ptr(addr), bytes);
           })
      .def("read_shard",
           [](const pack::Pack& p, const std::string& name, const tp::Shape& shape, const tp::Geometry& g,
              uint64_t addr, uint64_t bytes) {
             tp::View v;
             {
               py::gil_scoped_release nogil;
               v = p.read_shard(name, shape, g, ptr(addr), bytes);
             }
             return py::make_tuple(uint32_t(v.shard_class), v.split_dimension, v.ranges, v.shard_bytes);
           });
});
