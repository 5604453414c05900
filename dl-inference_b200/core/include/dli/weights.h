// dli.weights.v1 loader: a JSON manifest {"format", "data", "tensors": {name:
// {dtype, shape, offset, nbytes}}} plus one binary payload, the format the
// reference exporter writes (python/dli_export/weights.py:21-65) and reads
// (src/weights.cc:242-272 of yncxcw/dl-inference). The payload is memory-mapped.
// The reference reads the whole file into a vector, copies each tensor into a
// pageable host tensor and then to the device (src/weights.cc:228-238); here a
// CUDA destination is filled straight from the mapping through a ring of
// pinned staging buffers (file reads overlap the DMA; one cudaMemcpyAsync per
// 32 MB chunk), and a CPU destination gets one copy out of the mapping. Dtype
// strings: float32, int64 (reference) and bfloat16, float16, int32 (additive).
#pragma once

#include <string>

#include "dli/engine.h"

namespace dli {

TensorMap loadWeights(const std::string& manifest_path, DeviceType device, int device_id = 0);

}  // namespace dli
