// Graph executor.
//
// Same entry point as the reference runtime (include/dli/engine.h:14-28 of
// yncxcw/dl-inference): Engine::run(graph, inputs) walks the nodes in order and
// returns the graph outputs (or every tensor when the graph lists none). The
// reference re-creates each operator, re-resolves every tensor name in a
// std::map and formats log strings per node per run (src/engine.cc:13-52); this
// engine compiles a graph once into a static plan (operators instantiated once,
// names resolved to slot indices) and replays it, so a run costs one virtual
// call per node. All launches of a run go to the current ATen CUDA stream of the
// inputs' device, which makes a run capturable into a CUDA graph by the caller.
#pragma once

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "dli/graph.h"
#include "dli/operator.h"
#include "dli/tensor.h"

namespace dli {

using TensorMap = std::map<std::string, Tensor>;

class ProfileSession;

// Per-run options (the reference's profiling design, .codex/profiling_design.md:141-160).
struct RunOptions {
  ProfileSession* profiler = nullptr;  // non-owning; times every node of the run when set
};

class Engine {
 public:
  Engine();
  ~Engine();
  Engine(const Engine&) = delete;
  Engine& operator=(const Engine&) = delete;

  OperatorRegistry& registry() { return registry_; }
  const OperatorRegistry& registry() const { return registry_; }
  KVCache& kvCache() { return kv_cache_; }
  const KVCache& kvCache() const { return kv_cache_; }

  TensorMap run(const Graph& graph, TensorMap inputs, const RunOptions& options = {});

  // Tensors bound to graph input names for every later run (e.g. weights), so a
  // run only passes what changes per call. Inputs passed to run() win.
  void setConstants(TensorMap constants);
  void clearConstants();

  // Tensor-parallel communicator used by `all_reduce` nodes (opaque ncclComm_t).
  void setCommunicator(void* comm, int rank, int size);
  // Drops cached plans (needed only if a Graph object is mutated after a run).
  void clearPlans();

 private:
  struct Plan;
  Plan& planFor(const Graph& graph);

  OperatorRegistry registry_;
  KVCache kv_cache_;
  std::map<const Graph*, std::unique_ptr<Plan>> plans_;
  TensorMap constants_;
  void* comm_ = nullptr;
  int tp_rank_ = 0;
  int tp_size_ = 1;
};

}  // namespace dli
