#include "dli/engine.h"

#include "dli/profile.h"

#include <c10/cuda/CUDAStream.h>

#include <algorithm>
#include <stdexcept>
#include <unordered_map>

namespace dli {

struct Engine::Plan {
  struct Step {
    std::unique_ptr<Operator> op;
    const Node* node = nullptr;
    std::vector<int> in;
    std::vector<int> out;
    std::vector<int> release;  // slots whose last reader is this step (freed after it)
  };
  std::vector<Node> nodes;  // private copy: steps point into it
  std::vector<Step> steps;
  std::unordered_map<std::string, int> slot_of;
  std::vector<std::string> slot_names;
  std::vector<int> output_slots;
  std::vector<std::string> output_names;
  std::vector<std::pair<int, const Tensor*>> constant_slots;  // resolved Engine::constants_

  int slot(const std::string& name) {
    auto it = slot_of.find(name);
    if (it != slot_of.end()) return it->second;
    const int id = static_cast<int>(slot_names.size());
    slot_of.emplace(name, id);
    slot_names.push_back(name);
    return id;
  }
  bool matches(const Graph& g) const {
    if (g.nodes.size() != nodes.size()) return false;
    if (nodes.empty()) return true;
    return g.nodes.front().name == nodes.front().name && g.nodes.back().name == nodes.back().name &&
           g.nodes.back().op_type == nodes.back().op_type && g.outputs == output_names;
  }
};

Engine::Engine() = default;
Engine::~Engine() = default;

void Engine::clearPlans() { plans_.clear(); }

void Engine::setConstants(TensorMap constants) {
  constants_ = std::move(constants);
  plans_.clear();  // plans hold pointers into constants_
}

void Engine::clearConstants() {
  constants_.clear();
  plans_.clear();
}

void Engine::setCommunicator(void* comm, int rank, int size) {
  comm_ = comm;
  tp_rank_ = rank;
  tp_size_ = size;
}

Engine::Plan& Engine::planFor(const Graph& graph) {
  auto it = plans_.find(&graph);
  if (it != plans_.end() && it->second->matches(graph)) return *it->second;
  auto plan = std::make_unique<Plan>();
  plan->nodes = graph.nodes;
  plan->output_names = graph.outputs;
  for (const auto& name : graph.inputs) plan->slot(name);
  plan->steps.reserve(plan->nodes.size());
  for (const Node& n : plan->nodes) {
    Plan::Step s;
    s.op = registry_.create(n.op_type);
    s.node = &n;
    for (const auto& name : n.inputs) s.in.push_back(plan->slot(name));
    for (const auto& name : n.outputs) s.out.push_back(plan->slot(name));
    plan->steps.push_back(std::move(s));
  }
  for (const auto& name : graph.outputs) plan->output_slots.push_back(plan->slot(name));
  // Liveness: a slot is released after its last reader unless the graph returns it
  // (when the graph lists no outputs every tensor is returned, so nothing is freed).
  if (!graph.outputs.empty()) {
    std::vector<int> last(plan->slot_names.size(), -1);
    for (std::size_t i = 0; i < plan->steps.size(); ++i)
      for (const int s : plan->steps[i].in) last[s] = static_cast<int>(i);
    std::vector<bool> keep(plan->slot_names.size(), false);
    for (const int s : plan->output_slots) keep[s] = true;
    for (std::size_t s = 0; s < last.size(); ++s) {
      if (last[s] < 0 || keep[s]) continue;
      Plan::Step& st = plan->steps[last[s]];
      if (std::find(st.out.begin(), st.out.end(), static_cast<int>(s)) != st.out.end()) continue;
      st.release.push_back(static_cast<int>(s));
    }
  }
  for (const auto& [name, tensor] : constants_) {
    const auto s = plan->slot_of.find(name);
    if (s != plan->slot_of.end()) plan->constant_slots.emplace_back(s->second, &tensor);
  }
  Plan& ref = *plan;
  plans_[&graph] = std::move(plan);
  return ref;
}

TensorMap Engine::run(const Graph& graph, TensorMap inputs, const RunOptions& options) {
  Plan& plan = planFor(graph);
  std::vector<Tensor> slots(plan.slot_names.size());
  for (const auto& [slot, tensor] : plan.constant_slots) slots[slot] = *tensor;
  TensorMap extra;  // inputs the graph never references (returned when outputs are unlisted)
  int device = -1;
  for (auto& [name, tensor] : inputs) {
    if (device < 0 && tensor.isCuda()) device = tensor.deviceId();
    auto it = plan.slot_of.find(name);
    if (it == plan.slot_of.end()) extra.emplace(name, std::move(tensor));
    else slots[it->second] = std::move(tensor);
  }
  if (device < 0) {
    for (const auto& [slot, tensor] : plan.constant_slots)
      if (tensor->isCuda()) {
        device = tensor->deviceId();
        break;
      }
  }

  ExecutionContext ctx;
  ctx.kv_cache = &kv_cache_;
  ctx.device = device < 0 ? 0 : device;
  // Host-only runs (no CUDA tensor anywhere) never touch the CUDA runtime; their
  // operators reject the host inputs.
  ctx.cuda_stream = device < 0 ? nullptr : c10::cuda::getCurrentCUDAStream(device).stream();
  ctx.communicator = comm_;
  ctx.tp_rank = tp_rank_;
  ctx.tp_size = tp_size_;
  ProfileSession* prof = options.profiler;
  ctx.profiler = prof;
  const std::int64_t run_id = prof ? prof->beginRun() : -1;

  std::vector<const Tensor*> in;
  std::vector<Tensor> out_storage;
  std::vector<Tensor*> out;
  for (const auto& step : plan.steps) {
    in.clear();
    for (std::size_t i = 0; i < step.in.size(); ++i) {
      const Tensor& t = slots[step.in[i]];
      if (!t.defined())
        throw std::invalid_argument("node '" + step.node->name + "' missing input tensor: " +
                                    step.node->inputs[i]);
      in.push_back(&t);
    }
    out_storage.assign(step.out.size(), Tensor());
    out.clear();
    for (auto& t : out_storage) out.push_back(&t);
    if (prof == nullptr) {
      step.op->compute(in, out, step.node->attributes, ctx);
    } else {
      // a node is CUDA-backed when any of its inputs lives on the GPU
      const bool cuda = device >= 0 && std::any_of(in.begin(), in.end(), [](const Tensor* t) { return t->isCuda(); });
      const int node_index = static_cast<int>(&step - plan.steps.data());
      const std::int64_t ev = prof->beginOperator(run_id, node_index, *step.node, cuda, ctx.device, ctx.cuda_stream, in);
      try {
        step.op->compute(in, out, step.node->attributes, ctx);
      } catch (...) {
        prof->endOperator(ev, false, out);
        prof->endRun(run_id, false);
        throw;
      }
      prof->endOperator(ev, true, out);
    }
    for (std::size_t i = 0; i < step.out.size(); ++i) slots[step.out[i]] = std::move(out_storage[i]);
    for (const int s : step.release) slots[s] = Tensor();
  }

  if (prof != nullptr) prof->endRun(run_id, true);
  TensorMap result;
  if (graph.outputs.empty()) {
    for (std::size_t i = 0; i < slots.size(); ++i)
      if (slots[i].defined()) result.emplace(plan.slot_names[i], std::move(slots[i]));
    for (auto& kv : extra) result.emplace(kv.first, std::move(kv.second));
    return result;
  }
  for (std::size_t i = 0; i < plan.output_slots.size(); ++i) {
    const Tensor& t = slots[plan.output_slots[i]];
    if (!t.defined()) throw std::invalid_argument("graph output tensor was not produced: " + graph.outputs[i]);
    result.emplace(graph.outputs[i], t);
  }
  return result;
}

}  // namespace dli
