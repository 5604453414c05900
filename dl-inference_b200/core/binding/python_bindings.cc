// pybind11 module `_dli_native` behind `import dli`: Graph, Engine and
// load_weights with the reference binding's Python surface
// (src/python_bindings.cc:49-85 of yncxcw/dl-inference). Tensors cross as
// torch.Tensor; Engine.run releases the GIL while the graph executes.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/csrc/utils/pybind.h>

#include <cstdint>
#include <string>
#include <utility>

#include "dli/engine.h"
#include "dli/graph.h"
#include "dli/profile.h"
#include "dli/weights.h"

namespace py = pybind11;

namespace {

dli::TensorMap fromPython(const py::dict& d) {
  dli::TensorMap out;
  for (const auto& item : d) {
    auto name = py::cast<std::string>(item.first);
    auto t = py::cast<at::Tensor>(item.second);
    out.emplace(std::move(name), dli::Tensor(std::move(t)));
  }
  return out;
}

py::dict toPython(const dli::TensorMap& m) {
  py::dict out;
  for (const auto& [name, t] : m) out[py::str(name)] = py::cast(t.torchTensor());
  return out;
}

std::pair<dli::DeviceType, int> parseDevice(const std::string& device) {
  const dli::DeviceType type = dli::deviceFromString(device);
  int index = 0;
  const auto colon = device.find(':');
  if (colon != std::string::npos) index = std::stoi(device.substr(colon + 1));
  return {type, index};
}

}  // namespace

PYBIND11_MODULE(_dli_native, m) {
  m.doc() = "dli graph engine with the sm_100a operator plugin";

  py::class_<dli::Graph>(m, "Graph")
      .def(py::init<>())
      .def_static("from_json", &dli::Graph::fromJson, py::arg("json"))
      .def_static("from_json_file", &dli::Graph::fromJsonFile, py::arg("path"))
      .def("to_json", &dli::Graph::toJson)
      .def_readwrite("format", &dli::Graph::format)
      .def_readwrite("model_type", &dli::Graph::model_type)
      .def_readwrite("weights", &dli::Graph::weights)
      .def_readwrite("inputs", &dli::Graph::inputs)
      .def_readwrite("outputs", &dli::Graph::outputs)
      .def_property_readonly("num_nodes", [](const dli::Graph& g) { return g.nodes.size(); })
      .def("node_ops", [](const dli::Graph& g) {
        std::vector<std::string> ops;
        for (const auto& n : g.nodes) ops.push_back(n.op_type);
        return ops;
      });

  py::class_<dli::Engine>(m, "Engine")
      .def(py::init<>())
      .def(
          "load_library",
          [](dli::Engine& e, const std::string& path) -> dli::Engine& {
            e.registry().loadLibrary(path);
            return e;
          },
          py::arg("path"), py::return_value_policy::reference_internal)
      .def(
          "run",
          [](dli::Engine& e, const dli::Graph& g, const py::dict& inputs, dli::ProfileSession* profile) {
            auto tensors = fromPython(inputs);
            dli::TensorMap out;
            dli::RunOptions options;
            options.profiler = profile;
            {
              py::gil_scoped_release release;
              out = e.run(g, std::move(tensors), options);
            }
            return toPython(out);
          },
          py::arg("graph"), py::arg("inputs"), py::arg("profile") = nullptr)
      .def(
          "set_constants",
          [](dli::Engine& e, const py::dict& tensors) { e.setConstants(fromPython(tensors)); },
          py::arg("tensors"))
      .def("clear_constants", &dli::Engine::clearConstants)
      .def("registered_operators", [](const dli::Engine& e) { return e.registry().types(); })
      .def("has_operator", [](const dli::Engine& e, const std::string& t) { return e.registry().contains(t); })
      .def("kv_cache_size", [](const dli::Engine& e) { return e.kvCache().size(); })
      .def("kv_cache_clear", [](dli::Engine& e) { e.kvCache().clear(); })
      .def("kv_cache_reset", [](dli::Engine& e) { e.kvCache().reset(); })
      .def("kv_cache_length",
           [](const dli::Engine& e, const std::string& name) -> std::int64_t {
             const auto* entry = e.kvCache().get(name);
             if (entry == nullptr) throw py::key_error(name);
             return entry->length;
           })
      .def("kv_cache_entry",
           [](const dli::Engine& e, const std::string& name) {
             const auto* entry = e.kvCache().get(name);
             if (entry == nullptr) throw py::key_error(name);
             return py::make_tuple(entry->key.torchTensor(), entry->value.torchTensor(), entry->length);
           })
      .def(
          "set_communicator",
          [](dli::Engine& e, std::uintptr_t comm, int rank, int size) {
            e.setCommunicator(reinterpret_cast<void*>(comm), rank, size);
          },
          py::arg("comm"), py::arg("rank"), py::arg("size"))
      .def("clear_plans", &dli::Engine::clearPlans);

  py::class_<dli::ProfileSession>(m, "ProfileSession")
      .def(py::init([](bool cpu, bool gpu, bool record_shapes, std::size_t max_events) {
             dli::ProfileConfig c;
             c.cpu = cpu;
             c.gpu = gpu;
             c.record_shapes = record_shapes;
             c.max_events = max_events;
             return std::make_unique<dli::ProfileSession>(c);
           }),
           py::arg("cpu") = true, py::arg("gpu") = true, py::arg("record_shapes") = false,
           py::arg("max_events") = 1000000)
      .def(
          "finalize",
          [](dli::ProfileSession& p) {
            py::gil_scoped_release release;
            p.finalize();
          })
      .def("reserve", &dli::ProfileSession::reserve, py::arg("pairs"))
      .def_property_readonly("finalized", &dli::ProfileSession::finalized)
      .def("to_json", &dli::ProfileSession::toJson)
      .def("write_json", &dli::ProfileSession::writeJson, py::arg("path"))
      .def_property_readonly("num_events", [](const dli::ProfileSession& p) { return p.events().size(); })
      .def_property_readonly("num_runs", [](const dli::ProfileSession& p) { return p.runs().size(); });

  m.def(
      "load_weights",
      [](const std::string& path, const std::string& device) {
        const auto [type, index] = parseDevice(device);
        dli::TensorMap out;
        {
          py::gil_scoped_release release;
          out = dli::loadWeights(path, type, index);
        }
        return toPython(out);
      },
      py::arg("path"), py::arg("device") = "cpu");
}
