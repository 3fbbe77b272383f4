// Bindings of the text plane (tokenizer, chat templates) and the JSON DOM.
#include "json.h"
#include "registry.h"
#include "text.h"

namespace py = pybind11;
using namespace spc;

static BindRegistrar reg([](py::module_& m) {
  py::class_<Tokenizer, std::shared_ptr<Tokenizer>>(m, "Tokenizer")
      .def_static("from_hf_json", &Tokenizer::from_hf_json, py::arg("json_text"))
      .def_static("from_compiled", [](py::bytes b) { return Tokenizer::from_compiled(std::string(b)); })
      .def("to_compiled", [](const Tokenizer& t) { return py::bytes(t.to_compiled()); })
      .def("encode", [](const Tokenizer& t, py::object text, bool allow_special) {
        std::string s = py::isinstance<py::bytes>(text) ? std::string(text.cast<py::bytes>())
                                                        : text.cast<std::string>();
        py::gil_scoped_release rel;
        return t.encode(s, allow_special);
      }, py::arg("text"), py::arg("allow_special") = true)
      .def("encode_batch", [](const Tokenizer& t, const std::vector<std::string>& texts, int workers,
                              bool allow_special) {
        py::gil_scoped_release rel;
        return t.encode_batch(texts, workers, allow_special);
      }, py::arg("texts"), py::arg("workers") = 4, py::arg("allow_special") = true)
      .def("decode", [](const Tokenizer& t, const std::vector<uint32_t>& ids, bool skip_special) {
        const std::string s = t.decode(ids, skip_special);
        return py::str(PyUnicode_DecodeUTF8(s.data(), s.size(), "replace"));
      }, py::arg("ids"), py::arg("skip_special") = false)
      .def("decode_bytes", [](const Tokenizer& t, const std::vector<uint32_t>& ids, bool skip_special) {
        return py::bytes(t.decode(ids, skip_special));
      }, py::arg("ids"), py::arg("skip_special") = false)
      .def("token_bytes", [](const Tokenizer& t, uint32_t id) { return py::bytes(t.token_bytes(id)); })
      .def("token_to_id", &Tokenizer::token_to_id)
      .def("is_special", &Tokenizer::is_special)
      .def_property_readonly("vocab_size", &Tokenizer::vocab_size)
      .def_property_readonly("unk_id", &Tokenizer::unk_id)
      .def_property_readonly("cache_hits", &Tokenizer::cache_hits)
      .def_property_readonly("cache_misses", &Tokenizer::cache_misses)
      .def_static("split_pieces", [](py::bytes b) { return Tokenizer::split_pieces(std::string(b)); });
  m.attr("CHAT_ADD_GENERATION_PROMPT") = kChatAddGenerationPrompt;
  m.attr("CHAT_ENABLE_THINKING") = kChatEnableThinking;
  m.def("render_chat", [](const std::vector<std::pair<std::string, std::string>>& msgs, const std::string& style,
                          uint32_t flags, const std::string& effort, size_t capacity) {
    std::vector<ChatMessage> v;
    for (auto& p : msgs) v.push_back(ChatMessage{p.first, p.second});
    return render_chat(v, style, flags, effort, capacity);
  }, py::arg("messages"), py::arg("style") = "glm", py::arg("flags") = kChatAddGenerationPrompt,
     py::arg("reasoning_effort") = "", py::arg("capacity") = size_t(1) << 24);
  m.def("json_normalize", [](const std::string& text) { return Json::parse(text).dump(); });
});
