// Small helpers the operator implementations share: shape arithmetic, input
// validation that throws the same exception types the reference operators do
// (std::invalid_argument), and typed attribute access with defaults.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "dli/attributes.h"
#include "dli/tensor.h"

namespace dli {

// Product of shape[begin, end) (the whole shape by default); 1 for an empty range.
std::int64_t product(const std::vector<std::int64_t>& shape, std::size_t begin = 0,
                     std::size_t end = static_cast<std::size_t>(-1));
// "[d0, d1, ...]" for error messages.
std::string formatShape(const std::vector<std::int64_t>& shape);
// Throws std::invalid_argument unless every input is a CUDA tensor.
void requireCudaInputs(const std::vector<const Tensor*>& inputs, const std::string& op);
// Throws unless the tensor holds float32, bfloat16 or float16.
void requireFloat(const Tensor& tensor, const std::string& op);
// Throws unless both tensors have one dtype.
void requireSameDtype(const Tensor& a, const Tensor& b, const std::string& op);
// A numeric attribute (an integer literal in the graph reads as a double) or `fallback`.
double attrDouble(const Attributes& attrs, const std::string& name, double fallback);
// An integer-list attribute or `fallback`.
std::vector<std::int64_t> attrInts(const Attributes& attrs, const std::string& name,
                                   std::vector<std::int64_t> fallback);
// Device pointer of a (const) tensor, for C-ABI calls that take void*.
void* ptr(const Tensor& tensor);
// The target shape of a reshape with at most one -1 entry resolved from the
// element count of `input`; throws when the counts cannot match. The rules are
// the reference's reshape contract (src/utils.cc:54-76), which exported graphs
// depend on.
std::vector<std::int64_t> reshapeShape(const std::vector<std::int64_t>& input,
                                       std::vector<std::int64_t> target);

}  // namespace dli
