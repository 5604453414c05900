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
    const auto opts = at::TensorOptions().dtype(torchDType(dtype)).device(at::kCPU);
    at::Tensor host = at::empty(shape, opts);
    if (nbytes) std::memcpy(host.data_ptr(), static_cast<const char*>(map.base) + offset, nbytes);
    if (device == DeviceType::Cpu) result.emplace(name, Tensor(host));
    else result.emplace(name, Tensor(host.to(at::Device(at::kCUDA, device_id))));
  }
  return result;
}

}  // namespace dli
