#include "dli/kv_cache.h"

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>

#include "dli_sm100.h"

namespace dli {
namespace {

dli_dtype cDtype(DType d) {
  switch (d) {
    case DType::Float32: return DLI_DTYPE_F32;
    case DType::BFloat16: return DLI_DTYPE_BF16;
    case DType::Float16: return DLI_DTYPE_F16;
    default: break;
  }
  throw std::invalid_argument("KV cache expects float32/bfloat16/float16 tensors");
}

void check(dli_status st, const char* what) {
  if (st == DLI_OK) return;
  const std::string msg = std::string(what) + ": " + dli_sm100_last_error();
  if (st == DLI_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

}  // namespace

void KVCache::append(const std::string& name, const Tensor& key, const Tensor& value, void* stream) {
  if (!key.isCuda() || !value.isCuda()) throw std::invalid_argument("KV cache expects CUDA tensors");
  if (key.rank() != 4 || value.rank() != 4) throw std::invalid_argument("KV cache expects rank-4 tensors");
  if (key.shape() != value.shape()) throw std::invalid_argument("KV key/value shape mismatch");
  if (key.dtype() != value.dtype()) throw std::invalid_argument("KV key/value dtype mismatch");
  const dli_dtype dt = cDtype(key.dtype());
  const std::int64_t b = key.dim(0), h = key.dim(1), s = key.dim(2), d = key.dim(3);
  c10::cuda::CUDAGuard guard(key.deviceId());
  if (stream == nullptr) stream = c10::cuda::getCurrentCUDAStream(key.deviceId()).stream();

  auto it = entries_.find(name);
  if (it != entries_.end()) {
    const KVCacheEntry& e = it->second;
    if (e.key.dim(0) != b || e.key.dim(1) != h || e.key.dim(3) != d || e.key.dtype() != key.dtype())
      throw std::invalid_argument("KV cache append shape mismatch");
  }
  if (it == entries_.end() || it->second.length + s > it->second.capacity()) {
    const std::int64_t old_len = it == entries_.end() ? 0 : it->second.length;
    const std::int64_t old_cap = it == entries_.end() ? 0 : it->second.capacity();
    std::int64_t cap = std::max<std::int64_t>({old_len + s, 2 * old_cap, 64});
    cap = (cap + 63) / 64 * 64;
    KVCacheEntry grown;
    grown.key = Tensor::cuda(key.dtype(), {b, h, cap, d}, key.deviceId());
    grown.value = Tensor::cuda(key.dtype(), {b, h, cap, d}, key.deviceId());
    grown.length = 0;
    if (old_len > 0) {
      // Move the valid rows: one pitched copy, a row block of old_len*D elements per (b, h).
      const KVCacheEntry& e = it->second;
      const std::size_t elt = byteSize(key.dtype());
      const std::size_t width = static_cast<std::size_t>(old_len * d) * elt;
      const std::size_t spitch = static_cast<std::size_t>(old_cap * d) * elt;
      const std::size_t dpitch = static_cast<std::size_t>(cap * d) * elt;
      const auto cs = static_cast<cudaStream_t>(stream);
      for (int which = 0; which < 2; ++which) {
        const Tensor& src = which ? e.value : e.key;
        Tensor& dst = which ? grown.value : grown.key;
        const cudaError_t err = cudaMemcpy2DAsync(dst.deviceData(), dpitch, src.deviceData(), spitch,
                                                  width, static_cast<std::size_t>(b * h),
                                                  cudaMemcpyDeviceToDevice, cs);
        if (err != cudaSuccess)
          throw std::runtime_error(std::string("kv cache grow: ") + cudaGetErrorString(err));
      }
      grown.length = old_len;
    }
    entries_[name] = std::move(grown);
    it = entries_.find(name);
  }
  KVCacheEntry& e = it->second;
  check(dli_sm100_kv_append(e.key.deviceData(), e.value.deviceData(), key.deviceData(), value.deviceData(),
                            b, h, e.capacity(), e.length, s, d, dt, stream),
        "kv cache append");
  e.length += s;
}

const KVCacheEntry* KVCache::get(const std::string& name) const {
  const auto it = entries_.find(name);
  return it == entries_.end() ? nullptr : &it->second;
}

KVCacheEntry* KVCache::getMutable(const std::string& name) {
  const auto it = entries_.find(name);
  return it == entries_.end() ? nullptr : &it->second;
}

KVCacheEntry& KVCache::reserve(const std::string& name, std::int64_t batch, std::int64_t heads,
                               std::int64_t capacity, std::int64_t head_dim, DType dtype, int device_id) {
  auto it = entries_.find(name);
  if (it != entries_.end()) {
    const KVCacheEntry& e = it->second;
    if (e.key.dim(0) == batch && e.key.dim(1) == heads && e.key.dim(3) == head_dim &&
        e.key.dtype() == dtype && e.capacity() >= capacity)
      return it->second;
  }
  KVCacheEntry e;
  e.key = Tensor(at::zeros({batch, heads, capacity, head_dim},
                           at::TensorOptions().dtype(torchDType(dtype)).device(at::kCUDA, device_id)));
  e.value = Tensor(at::zeros({batch, heads, capacity, head_dim},
                             at::TensorOptions().dtype(torchDType(dtype)).device(at::kCUDA, device_id)));
  e.length = 0;
  entries_[name] = std::move(e);
  return entries_[name];
}

void KVCache::reset() {
  for (auto& kv : entries_) kv.second.length = 0;
}

}  // namespace dli
