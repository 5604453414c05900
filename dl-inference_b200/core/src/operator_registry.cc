#include <dlfcn.h>

#include <memory>
#include <stdexcept>

#include "dli/operator.h"

namespace dli {

namespace {

// Owns a dlopen handle until released; closes it when a load step fails.
struct DlCloser {
  void operator()(void* handle) const {
    if (handle != nullptr) dlclose(handle);
  }
};
using LibraryHandle = std::unique_ptr<void, DlCloser>;

std::string dlErrorText() {
  const char* text = dlerror();
  return text != nullptr ? text : "unknown error";
}

}  // namespace

void OperatorRegistry::registerFactory(std::string type, Factory factory) {
  factories_.insert_or_assign(std::move(type), std::move(factory));
}

bool OperatorRegistry::contains(const std::string& type) const { return factories_.find(type) != factories_.end(); }

std::unique_ptr<Operator> OperatorRegistry::create(const std::string& type) const {
  const auto found = factories_.find(type);
  if (found == factories_.end()) throw std::invalid_argument("operator is not registered: " + type);
  return found->second();
}

std::vector<std::string> OperatorRegistry::types() const {
  std::vector<std::string> names;
  names.reserve(factories_.size());
  for (const auto& entry : factories_) names.push_back(entry.first);
  return names;
}

// The plugin contract: RTLD_NOW | RTLD_LOCAL, an extern "C" registration entry
// point that returns false on failure, and a handle kept for the registry's
// lifetime once registration succeeded (the factories point into the library).
void OperatorRegistry::loadLibrary(const std::string& path) {
  LibraryHandle library(dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL));
  if (!library) throw std::runtime_error("failed to load operator library: " + path + ": " + dlErrorText());
  const auto entry = reinterpret_cast<RegisterOperatorsFn>(dlsym(library.get(), "dli_register_operators"));
  if (entry == nullptr) throw std::runtime_error("operator library is missing dli_register_operators: " + path);
  if (!entry(this)) throw std::runtime_error("operator library registration failed: " + path);
  library_handles_.push_back(library.release());
}

}  // namespace dli
