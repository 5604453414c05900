// Operator plugin boundary: the interface a dlopen'ed operator library
// implements and the registry it registers into. Same shape as the reference
// runtime (include/dli/operator.h:15-41 of yncxcw/dl-inference): a plugin
// exports `extern "C" bool dli_register_operators(dli::OperatorRegistry*)`,
// which calls registerFactory(type, factory) once per operator string.
//
// ExecutionContext keeps the reference's `kv_cache` member first and appends the
// stream / device / tensor-parallel fields the sm_100a plugin needs.
#pragma once

#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "dli/attributes.h"
#include "dli/kv_cache.h"
#include "dli/tensor.h"

namespace dli {

class ProfileSession;

struct ExecutionContext {
  KVCache* kv_cache = nullptr;
  void* cuda_stream = nullptr;   // cudaStream_t every launch of this run goes to
  int device = 0;                // CUDA device ordinal of the run
  void* communicator = nullptr;  // tensor-parallel communicator (ncclComm_t) or null
  int tp_rank = 0;
  int tp_size = 1;
  ProfileSession* profiler = nullptr;  // the run's profiling session, if any
};

class Operator {
 public:
  virtual ~Operator() = default;
  virtual std::string type() const = 0;
  virtual void compute(const std::vector<const Tensor*>& inputs, const std::vector<Tensor*>& outputs,
                       const Attributes& attrs, ExecutionContext& context) const = 0;
};

class OperatorRegistry {
 public:
  using Factory = std::function<std::unique_ptr<Operator>()>;
  void registerFactory(std::string type, Factory factory);
  bool contains(const std::string& type) const;
  std::unique_ptr<Operator> create(const std::string& type) const;
  // dlopen(path, RTLD_NOW | RTLD_LOCAL) + dlsym("dli_register_operators"); throws
  // std::runtime_error when the library, the symbol or the registration fails.
  void loadLibrary(const std::string& path);
  std::vector<std::string> types() const;

 private:
  std::map<std::string, Factory> factories_;
  std::vector<void*> library_handles_;
};

using RegisterOperatorsFn = bool (*)(OperatorRegistry*);

}  // namespace dli
