// dli::Tensor — the tensor handed across the operator boundary.
//
// Same contract as the reference runtime's tensor (include/dli/tensor.h:14-73 of
// yncxcw/dl-inference): dense row-major storage owned by an at::Tensor (the
// PyTorch caching allocator provides device memory), or a non-owning external
// CUDA pointer; `deviceData()` returns the raw device pointer and throws
// std::logic_error for host tensors. DType keeps the reference's Float32 = 0 and
// Int64 = 1 and appends BFloat16, Float16 and Int32.
#pragma once

#include <ATen/ATen.h>

#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace dli {

enum class DeviceType { Cpu, Cuda };
enum class DType { Float32, Int64, BFloat16, Float16, Int32 };

std::string toString(DeviceType device);
DeviceType deviceFromString(const std::string& device);
std::string toString(DType dtype);
DType dtypeFromString(const std::string& dtype);
std::size_t byteSize(DType dtype);
bool isFloating(DType dtype);
at::ScalarType torchDType(DType dtype);
DType dtypeFromTorch(at::ScalarType dtype);

class Tensor {
 public:
  Tensor() = default;
  Tensor(DType dtype, std::vector<std::int64_t> shape);  // zero-filled host tensor
  explicit Tensor(at::Tensor tensor);                       // made contiguous

  static Tensor zeros(DType dtype, std::vector<std::int64_t> shape);
  static Tensor cuda(DType dtype, std::vector<std::int64_t> shape, int device_id = 0);
  static Tensor externalCuda(DType dtype, std::vector<std::int64_t> shape, void* data,
                             int device_id = 0);

  DType dtype() const { return dtype_; }
  DeviceType device() const { return device_; }
  int deviceId() const { return device_id_; }
  bool isCpu() const { return device_ == DeviceType::Cpu; }
  bool isCuda() const { return device_ == DeviceType::Cuda; }
  bool defined() const { return static_cast<bool>(impl_) || external_device_ptr_ != nullptr; }
  const std::vector<std::int64_t>& shape() const { return shape_; }
  std::size_t rank() const { return shape_.size(); }
  std::int64_t dim(std::size_t index) const;
  std::size_t numel() const;
  std::size_t nbytes() const;
  void* deviceData();
  const void* deviceData() const;
  Tensor withShape(std::vector<std::int64_t> shape) const;
  at::Tensor& torchTensor();
  const at::Tensor& torchTensor() const;

  template <typename T>
  T* data();
  template <typename T>
  const T* data() const;

 private:
  struct Impl;
  explicit Tensor(std::shared_ptr<Impl> impl);
  const Impl& impl() const;
  Impl& impl();

  DType dtype_ = DType::Float32;
  DeviceType device_ = DeviceType::Cpu;
  int device_id_ = 0;
  std::vector<std::int64_t> shape_;
  std::shared_ptr<Impl> impl_;
  void* external_device_ptr_ = nullptr;
};

bool sameShape(const Tensor& lhs, const Tensor& rhs);
std::size_t contiguousOffset(const std::vector<std::int64_t>& shape,
                             const std::vector<std::int64_t>& indices);

}  // namespace dli
