#include <dlfcn.h>

#include <stdexcept>

#include "dli/operator.h"

namespace dli {

void OperatorRegistry::registerFactory(std::string type, Factory factory) {
  factories_[std::move(type)] = std::move(factory);
}

bool OperatorRegistry::contains(const std::string& type) const { return factories_.count(type) != 0; }

std::unique_ptr<Operator> OperatorRegistry::create(const std::string& type) const {
  const auto it = factories_.find(type);
  if (it == factories_.end()) throw std::invalid_argument("operator is not registered: " + type);
  return it->second();
}

std::vector<std::string> OperatorRegistry::types() const {
  std::vector<std::string> out;
  out.reserve(factories_.size());
  for (const auto& kv : factories_) out.push_back(kv.first);
  return out;
}

void OperatorRegistry::loadLibrary(const std::string& path) {
  void* handle = dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL);
  if (handle == nullptr) {
    const char* err = dlerror();
    throw std::runtime_error("failed to load operator library: " + path + ": " +
                             (err ? err : "unknown error"));
  }
  void* sym = dlsym(handle, "dli_register_operators");
  if (sym == nullptr) {
    dlclose(handle);
    throw std::runtime_error("operator library is missing dli_register_operators: " + path);
  }
  if (!reinterpret_cast<RegisterOperatorsFn>(sym)(this)) {
    dlclose(handle);
    throw std::runtime_error("operator library registration failed: " + path);
  }
  library_handles_.push_back(handle);  // kept for the registry's lifetime
}

}  // namespace dli
