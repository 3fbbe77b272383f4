// Binding registry: each bind_*.cpp translation unit registers a function that
// adds its classes to the _sp_core module, so subsystems bind themselves
// without a central list (and without pulling torch headers into every unit).
#pragma once
#include <pybind11/functional.h>
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <functional>
#include <vector>

namespace spc {

using BindFn = std::function<void(pybind11::module_&)>;

inline std::vector<BindFn>& registry() {
  static std::vector<BindFn> fns;
  return fns;
}

struct BindRegistrar {
  explicit BindRegistrar(BindFn fn) { registry().push_back(std::move(fn)); }
};

}  // namespace spc
