// Per-layer key/value cache.
//
// Keeps the reference's API (include/dli/kv_cache.h:10-24 of yncxcw/dl-inference:
// append(name, key, value), get(name), size(), clear()) but stores each entry in
// preallocated [B, H, capacity, D] device buffers with a row count `length`.
// append() writes the new rows in place with a strided copy kernel (the
// reference reallocates and copies the whole cache with four flat memcpys per
// call, src/kv_cache.cc:33-42, which is also only a sequence concatenation when
// B*H == 1); when capacity runs out the buffers grow geometrically.
//
// reserve() creates an entry of a fixed capacity for graphs that address rows by
// position (the fused qkv_rotary_cache / attention_kvcache operators): those
// write rows positions[b] + s themselves and leave `length` untouched.
#pragma once

#include <cstdint>
#include <map>
#include <string>

#include "dli/tensor.h"

namespace dli {

struct KVCacheEntry {
  Tensor key;    // [B, H, capacity, D]
  Tensor value;  // [B, H, capacity, D]
  std::int64_t length = 0;
  std::int64_t capacity() const { return key.rank() == 4 ? key.dim(2) : 0; }
};

class KVCache {
 public:
  // Appends key/value [B, H, S_new, D] (CUDA, float dtype) on `stream`
  // (cudaStream_t; null = the current ATen stream of the tensors' device).
  void append(const std::string& name, const Tensor& key, const Tensor& value,
              void* stream = nullptr);
  const KVCacheEntry* get(const std::string& name) const;
  KVCacheEntry* getMutable(const std::string& name);
  // Creates (or returns, if shape-compatible) a zero-filled entry of the given capacity.
  KVCacheEntry& reserve(const std::string& name, std::int64_t batch, std::int64_t heads,
                        std::int64_t capacity, std::int64_t head_dim, DType dtype, int device_id);
  std::size_t size() const { return entries_.size(); }
  void clear() { entries_.clear(); }
  // Sets every entry's length to 0 without releasing memory.
  void reset();

 private:
  std::map<std::string, KVCacheEntry> entries_;
};

}  // namespace dli
