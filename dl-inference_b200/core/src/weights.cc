#include "dli/weights.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <filesystem>
#include <fstream>
#include <cstring>
#include <sstream>
#include <stdexcept>

#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>

#include "json.h"

namespace dli {
namespace {

struct Mapping {
  void* base = MAP_FAILED;
  std::size_t size = 0;
  int fd = -1;
  explicit Mapping(const std::string& path) {
    fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("failed to open weights data: " + path);
    struct stat st {};
    if (::fstat(fd, &st) != 0) throw std::runtime_error("failed to stat weights data: " + path);
    size = static_cast<std::size_t>(st.st_size);
    if (size > 0) {
      base = ::mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
      if (base == MAP_FAILED) throw std::runtime_error("failed to map weights data: " + path);
    }
  }
  ~Mapping() {
    if (base != MAP_FAILED) ::munmap(base, size);
    if (fd >= 0) ::close(fd);
  }
};

void cudaCheck(cudaError_t err, const char* what) {
  if (err != cudaSuccess) throw std::runtime_error(std::string("weights: ") + what + ": " + cudaGetErrorString(err));
}

// Host-to-device upload through a ring of pinned staging buffers: the mapped
// file pages are copied into one buffer while the DMA engine drains the
// previous ones (one cudaMemcpyAsync per chunk on a private stream), so file
// reads and PCIe/C2C transfers overlap and every byte crosses host memory once.
class DeviceUploader {
 public:
  static constexpr std::size_t kChunk = std::size_t(32) << 20;
  static constexpr int kSlots = 4;

  explicit DeviceUploader(int device) : guard_(static_cast<c10::DeviceIndex>(device)) {
    cudaCheck(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    for (int i = 0; i < kSlots; ++i) {
      cudaCheck(cudaHostAlloc(&slot_[i], kChunk, cudaHostAllocDefault), "cudaHostAlloc");
      cudaCheck(cudaEventCreateWithFlags(&done_[i], cudaEventDisableTiming), "cudaEventCreate");
    }
  }
  ~DeviceUploader() {
    if (stream_) cudaStreamSynchronize(stream_);
    for (int i = 0; i < kSlots; ++i) {
      if (done_[i]) cudaEventDestroy(done_[i]);
      if (slot_[i]) cudaFreeHost(slot_[i]);
    }
    if (stream_) cudaStreamDestroy(stream_);
  }
  DeviceUploader(const DeviceUploader&) = delete;
  DeviceUploader& operator=(const DeviceUploader&) = delete;

  void upload(void* dst, const char* src, std::size_t n) {
    for (std::size_t off = 0; off < n; off += kChunk) {
      const std::size_t len = std::min(kChunk, n - off);
      const int s = next_++ % kSlots;
      if (used_[s]) cudaCheck(cudaEventSynchronize(done_[s]), "cudaEventSynchronize");  // slot drained
      std::memcpy(slot_[s], src + off, len);
      cudaCheck(cudaMemcpyAsync(static_cast<char*>(dst) + off, slot_[s], len, cudaMemcpyHostToDevice, stream_),
                "cudaMemcpyAsync");
      cudaCheck(cudaEventRecord(done_[s], stream_), "cudaEventRecord");
      used_[s] = true;
      bytes_ += len;
    }
  }
  void finish() { cudaCheck(cudaStreamSynchronize(stream_), "cudaStreamSynchronize"); }
  std::size_t bytes() const { return bytes_; }

 private:
  c10::cuda::CUDAGuard guard_;
  cudaStream_t stream_ = nullptr;
  std::array<void*, kSlots> slot_{};
  std::array<cudaEvent_t, kSlots> done_{};
  std::array<bool, kSlots> used_{};
  unsigned next_ = 0;
  std::size_t bytes_ = 0;
};

}  // namespace

TensorMap loadWeights(const std::string& manifest_path, DeviceType device, int device_id) {
  const std::filesystem::path manifest(manifest_path);
  std::ifstream f(manifest);
  if (!f) throw std::runtime_error("failed to open weights manifest: " + manifest_path);
  std::ostringstream buf;
  buf << f.rdbuf();
  const json::Value root = json::parse(buf.str());
  if (root.type != json::Value::Type::Object)
    throw std::invalid_argument("weights manifest root must be an object");
  const std::string format = json::asString(root.at("format"), "format");
  if (format != "dli.weights.v1") throw std::invalid_argument("unsupported weights format: " + format);
  std::filesystem::path data = json::asString(root.at("data"), "data");
  if (data.is_relative()) data = manifest.parent_path() / data;
  const json::Value& tensors = root.at("tensors");
  if (tensors.type != json::Value::Type::Object) throw std::invalid_argument("weights tensors must be an object");

  Mapping map(data.string());
  TensorMap result;
  // declared after `result`: on an error the uploader drains its stream before
  // the tensors it writes into are released
  std::unique_ptr<DeviceUploader> uploader;
  if (device != DeviceType::Cpu) uploader = std::make_unique<DeviceUploader>(device_id);
  for (const auto& [name, meta] : tensors.o) {
    if (meta.type != json::Value::Type::Object)
      throw std::invalid_argument("weights tensor metadata must be an object: " + name);
    const DType dtype = dtypeFromString(json::asString(meta.at("dtype"), "dtype"));
    const std::vector<std::int64_t> shape = json::asIntArray(meta.at("shape"), "shape");
    const auto offset = static_cast<std::size_t>(json::asInt(meta.at("offset"), "offset"));
    const auto nbytes = static_cast<std::size_t>(json::asInt(meta.at("nbytes"), "nbytes"));
    if (offset > map.size || nbytes > map.size - offset)
      throw std::invalid_argument("weights tensor range exceeds data file: " + name);
    std::size_t expect = byteSize(dtype);
    for (const auto d : shape) {
      if (d < 0) throw std::invalid_argument("negative dimension in weights tensor: " + name);
      expect *= static_cast<std::size_t>(d);
    }
    if (expect != nbytes)
      throw std::invalid_argument("weights tensor byte count does not match dtype and shape: " + name);
    const char* src = static_cast<const char*>(map.base) + offset;
    if (device == DeviceType::Cpu) {
      at::Tensor host = at::empty(shape, at::TensorOptions().dtype(torchDType(dtype)).device(at::kCPU));
      if (nbytes) std::memcpy(host.data_ptr(), src, nbytes);
      result.emplace(name, Tensor(host));
    } else {
      // straight from the mapped file to the device tensor, no pageable copy
      at::Tensor dev = at::empty(shape, at::TensorOptions().dtype(torchDType(dtype)).device(at::kCUDA, device_id));
      if (nbytes) uploader->upload(dev.data_ptr(), src, nbytes);
      result.emplace(name, Tensor(dev));
    }
  }
  // the device tensors are complete before they are returned (the caching
  // allocator's streams never saw the private upload stream)
  if (uploader) uploader->finish();
  return result;
}

}  // namespace dli
