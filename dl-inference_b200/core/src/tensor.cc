#include "dli/tensor.h"

#include <limits>
#include <utility>

namespace dli {

struct Tensor::Impl {
  explicit Impl(at::Tensor t) : tensor(std::move(t)) {}
  at::Tensor tensor;
};

namespace {

at::TensorOptions optionsFor(DType dtype, DeviceType device, int device_id) {
  auto options = at::TensorOptions().dtype(torchDType(dtype));
  return device == DeviceType::Cpu ? options.device(at::kCPU)
                                   : options.device(at::Device(at::kCUDA, device_id));
}

void checkShape(const std::vector<std::int64_t>& shape) {
  for (const auto d : shape)
    if (d < 0) throw std::invalid_argument("negative tensor dimension");
}

template <typename T>
void checkHost(const Tensor& t, DType want) {
  if (!t.isCpu()) throw std::logic_error("host data access requested for non-CPU tensor");
  if (t.dtype() != want) throw std::logic_error("tensor dtype does not match requested host type");
}

}  // namespace

std::string toString(DeviceType device) { return device == DeviceType::Cpu ? "cpu" : "cuda"; }

DeviceType deviceFromString(const std::string& device) {
  if (device == "cpu") return DeviceType::Cpu;
  if (device == "cuda" || device.rfind("cuda:", 0) == 0) return DeviceType::Cuda;
  throw std::invalid_argument("unknown device: " + device);
}

std::string toString(DType dtype) {
  switch (dtype) {
    case DType::Float32: return "float32";
    case DType::Int64: return "int64";
    case DType::BFloat16: return "bfloat16";
    case DType::Float16: return "float16";
    case DType::Int32: return "int32";
  }
  throw std::invalid_argument("unknown dtype");
}

DType dtypeFromString(const std::string& dtype) {
  if (dtype == "float32") return DType::Float32;
  if (dtype == "int64") return DType::Int64;
  if (dtype == "bfloat16") return DType::BFloat16;
  if (dtype == "float16") return DType::Float16;
  if (dtype == "int32") return DType::Int32;
  throw std::invalid_argument("unknown dtype: " + dtype);
}

std::size_t byteSize(DType dtype) {
  switch (dtype) {
    case DType::Float32: return 4;
    case DType::Int64: return 8;
    case DType::BFloat16: return 2;
    case DType::Float16: return 2;
    case DType::Int32: return 4;
  }
  throw std::invalid_argument("unknown dtype");
}

bool isFloating(DType dtype) {
  return dtype == DType::Float32 || dtype == DType::BFloat16 || dtype == DType::Float16;
}

at::ScalarType torchDType(DType dtype) {
  switch (dtype) {
    case DType::Float32: return at::kFloat;
    case DType::Int64: return at::kLong;
    case DType::BFloat16: return at::kBFloat16;
    case DType::Float16: return at::kHalf;
    case DType::Int32: return at::kInt;
  }
  throw std::invalid_argument("unknown dtype");
}

DType dtypeFromTorch(at::ScalarType dtype) {
  switch (dtype) {
    case at::kFloat: return DType::Float32;
    case at::kLong: return DType::Int64;
    case at::kBFloat16: return DType::BFloat16;
    case at::kHalf: return DType::Float16;
    case at::kInt: return DType::Int32;
    default: break;
  }
  throw std::invalid_argument("unsupported torch tensor dtype");
}

Tensor::Tensor(std::shared_ptr<Impl> impl) : impl_(std::move(impl)) {
  const auto& t = impl_->tensor;
  dtype_ = dtypeFromTorch(t.scalar_type());
  if (t.device().is_cpu()) {
    device_ = DeviceType::Cpu;
    device_id_ = 0;
  } else if (t.device().is_cuda()) {
    device_ = DeviceType::Cuda;
    device_id_ = t.device().index();
  } else {
    throw std::invalid_argument("unsupported torch tensor device");
  }
  shape_.assign(t.sizes().begin(), t.sizes().end());
  if (shape_.empty()) shape_.push_back(1);
}

Tensor::Tensor(at::Tensor tensor) : Tensor(std::make_shared<Impl>(tensor.contiguous())) {}

Tensor::Tensor(DType dtype, std::vector<std::int64_t> shape) {
  if (shape.empty()) shape.push_back(1);
  checkShape(shape);
  *this = Tensor(std::make_shared<Impl>(at::zeros(shape, optionsFor(dtype, DeviceType::Cpu, 0))));
}

Tensor Tensor::zeros(DType dtype, std::vector<std::int64_t> shape) {
  return Tensor(dtype, std::move(shape));
}

Tensor Tensor::cuda(DType dtype, std::vector<std::int64_t> shape, int device_id) {
  if (shape.empty()) shape.push_back(1);
  checkShape(shape);
  return Tensor(std::make_shared<Impl>(at::empty(shape, optionsFor(dtype, DeviceType::Cuda, device_id))));
}

Tensor Tensor::externalCuda(DType dtype, std::vector<std::int64_t> shape, void* data, int device_id) {
  if (data == nullptr) throw std::invalid_argument("external CUDA tensor pointer is null");
  if (shape.empty()) shape.push_back(1);
  checkShape(shape);
  Tensor t;
  t.dtype_ = dtype;
  t.device_ = DeviceType::Cuda;
  t.device_id_ = device_id;
  t.shape_ = std::move(shape);
  t.external_device_ptr_ = data;
  return t;
}

const Tensor::Impl& Tensor::impl() const {
  if (!impl_) throw std::logic_error("tensor is uninitialized");
  return *impl_;
}

Tensor::Impl& Tensor::impl() {
  if (!impl_) throw std::logic_error("tensor is uninitialized");
  return *impl_;
}

std::int64_t Tensor::dim(std::size_t index) const {
  if (index >= shape_.size()) throw std::out_of_range("tensor dimension out of range");
  return shape_[index];
}

std::size_t Tensor::numel() const {
  std::size_t n = 1;
  for (const auto d : shape_) {
    if (d == 0) return 0;
    if (static_cast<std::uint64_t>(d) > std::numeric_limits<std::size_t>::max() / n)
      throw std::overflow_error("tensor shape is too large");
    n *= static_cast<std::size_t>(d);
  }
  return n;
}

std::size_t Tensor::nbytes() const { return numel() * byteSize(dtype_); }

void* Tensor::deviceData() {
  if (device_ != DeviceType::Cuda) throw std::logic_error("tensor is not on CUDA");
  return impl_ ? impl_->tensor.data_ptr() : external_device_ptr_;
}

const void* Tensor::deviceData() const {
  if (device_ != DeviceType::Cuda) throw std::logic_error("tensor is not on CUDA");
  return impl_ ? impl_->tensor.data_ptr() : external_device_ptr_;
}

Tensor Tensor::withShape(std::vector<std::int64_t> shape) const {
  if (shape.empty()) shape.push_back(1);
  checkShape(shape);
  std::size_t n = 1;
  for (const auto d : shape) n *= static_cast<std::size_t>(d);
  if (n != numel()) throw std::invalid_argument("tensor view changes element count");
  if (!impl_) {
    Tensor view = *this;
    view.shape_ = std::move(shape);
    return view;
  }
  return Tensor(std::make_shared<Impl>(impl_->tensor.view(shape)));
}

at::Tensor& Tensor::torchTensor() { return impl().tensor; }
const at::Tensor& Tensor::torchTensor() const { return impl().tensor; }

template <> float* Tensor::data<float>() { checkHost<float>(*this, DType::Float32); return impl().tensor.data_ptr<float>(); }
template <> const float* Tensor::data<float>() const { checkHost<float>(*this, DType::Float32); return impl().tensor.data_ptr<float>(); }
template <> std::int64_t* Tensor::data<std::int64_t>() { checkHost<std::int64_t>(*this, DType::Int64); return impl().tensor.data_ptr<std::int64_t>(); }
template <> const std::int64_t* Tensor::data<std::int64_t>() const { checkHost<std::int64_t>(*this, DType::Int64); return impl().tensor.data_ptr<std::int64_t>(); }

bool sameShape(const Tensor& lhs, const Tensor& rhs) { return lhs.shape() == rhs.shape(); }

std::size_t contiguousOffset(const std::vector<std::int64_t>& shape,
                             const std::vector<std::int64_t>& indices) {
  if (shape.size() != indices.size()) throw std::invalid_argument("rank mismatch in contiguousOffset");
  std::size_t offset = 0, stride = 1;
  for (std::size_t r = shape.size(); r-- > 0;) {
    if (indices[r] < 0 || indices[r] >= shape[r]) throw std::out_of_range("tensor index out of range");
    offset += static_cast<std::size_t>(indices[r]) * stride;
    stride *= static_cast<std::size_t>(shape[r]);
  }
  return offset;
}

}  // namespace dli
