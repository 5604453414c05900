// Library-wide state of libdli_sm100.so: last-error text, device error word,
// device properties.
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "common.cuh"

namespace dli_sm100 {

__device__ unsigned g_device_error = 0;

namespace {
thread_local std::string t_last_error;

const char* device_error_name(unsigned code) {
  switch (code) {
    case kDevErrGemmTimeout: return "tcgen05 GEMM pipeline wait exceeded its iteration limit";
    case kDevErrEmbeddingIndex: return "embedding id outside [0, vocab)";
    case kDevErrRotaryPosition: return "rotary position outside the cos/sin table";
    case kDevErrAttentionTimeout: return "attention pipeline wait exceeded its iteration limit";
    case kDevErrKvCapacity: return "KV-cache position outside the cache capacity";
    case kDevErrExchangeTimeout: return "tensor-parallel exchange: a peer's rows did not arrive within the wait limit";
    default: return "unknown device error";
  }
}
}  // namespace

dli_status fail(dli_status status, const std::string& msg) {
  t_last_error = msg;
  return status;
}

dli_status ok() {
  t_last_error.clear();
  return DLI_OK;
}

std::atomic<uint64_t> g_launches{0};

dli_status check_launch(const char* what, int launches) {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return fail(DLI_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
  }
  g_launches.fetch_add(static_cast<uint64_t>(launches), std::memory_order_relaxed);
  return ok();
}

unsigned* device_error_word() {
  static std::mutex mu;
  static std::vector<unsigned*> words;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(words.size()) <= dev) words.resize(dev + 1, nullptr);
  if (words[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    words[dev] = static_cast<unsigned*>(p);
  }
  return words[dev];
}

dli_status ensure_smem(const void* kernel, int bytes, const char* what) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(DLI_ERR_CUDA, std::string(what) + ": no device");
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({dev, kernel})) return DLI_OK;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    return fail(DLI_ERR_CUDA, std::string(what) + " shared-memory attribute: " + cudaGetErrorString(e));
  done.insert({dev, kernel});
  return DLI_OK;
}

int tuning_knob(const char* name, int fallback) {
  const std::string var = std::string("DLI_SM100_") + name;
  const char* v = std::getenv(var.c_str());
  if (v == nullptr || *v == '\0') return fallback;
  return std::atoi(v);
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> counts;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(counts.size()) <= dev) counts.resize(dev + 1, 0);
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

}  // namespace dli_sm100

using namespace dli_sm100;

extern "C" int dli_sm100_abi_version(void) { return DLI_SM100_ABI_VERSION; }

extern "C" uint64_t dli_sm100_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" const char* dli_sm100_last_error(void) { return t_last_error.c_str(); }

extern "C" dli_status dli_sm100_check_device_error(void* stream) {
  cudaError_t err = cudaStreamSynchronize(as_stream(stream));
  if (err != cudaSuccess) return fail(DLI_ERR_CUDA, std::string("stream sync: ") + cudaGetErrorString(err));
  unsigned code = 0;
  err = cudaMemcpyFromSymbol(&code, g_device_error, sizeof(code));
  if (err != cudaSuccess) return fail(DLI_ERR_CUDA, std::string("read device error: ") + cudaGetErrorString(err));
  if (code == 0) return ok();
  const unsigned zero = 0;
  err = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  if (err != cudaSuccess) return fail(DLI_ERR_CUDA, std::string("clear device error: ") + cudaGetErrorString(err));
  return fail(DLI_ERR_DEVICE, std::string("device error ") + std::to_string(code) + ": " +
                                  device_error_name(code));
}
