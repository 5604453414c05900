#include "dli/profile.h"

#include <cuda_runtime.h>
#include <unistd.h>

#include <chrono>
#include <ctime>
#include <fstream>
#include <functional>
#include <sstream>
#include <stdexcept>
#include <thread>

#include "dli/graph.h"

namespace dli {

namespace {

std::int64_t steadyNs() {
  return std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

void cudaCheck(cudaError_t err, const char* what) {
  if (err != cudaSuccess) throw std::runtime_error(std::string("profile: ") + what + ": " + cudaGetErrorString(err));
}

std::string jsonEscape(const std::string& s) {
  std::string out;
  out.reserve(s.size() + 2);
  for (const char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\t': out += "\\t"; break;
      default:
        if (static_cast<unsigned char>(c) < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof(buf), "\\u%04x", c);
          out += buf;
        } else {
          out += c;
        }
    }
  }
  return out;
}

std::string shapeText(const Tensor& t) {
  std::string s = toString(t.dtype()) + (t.isCuda() ? "@cuda:" + std::to_string(t.deviceId()) : "@cpu") + "[";
  for (std::size_t i = 0; i < t.shape().size(); ++i) s += (i ? "," : "") + std::to_string(t.shape()[i]);
  return s + "]";
}

std::string utcNow() {
  const std::time_t t = std::time(nullptr);
  std::tm tm{};
  gmtime_r(&t, &tm);
  char buf[32];
  std::strftime(buf, sizeof(buf), "%Y-%m-%dT%H:%M:%SZ", &tm);
  return buf;
}

}  // namespace

// A start/end event pair on one stream. `captured` pairs were recorded into a
// CUDA graph under capture: they hold a time only once the graph has replayed.
struct ProfileSession::EventPair {
  cudaEvent_t start = nullptr;
  cudaEvent_t end = nullptr;
  bool captured = false;
  EventPair() {
    cudaCheck(cudaEventCreate(&start), "cudaEventCreate");
    cudaCheck(cudaEventCreate(&end), "cudaEventCreate");
  }
  ~EventPair() {
    if (start) cudaEventDestroy(start);
    if (end) cudaEventDestroy(end);
  }
};

ProfileSession::ProfileSession(ProfileConfig config) : config_(config), origin_ns_(steadyNs()) {}

ProfileSession::~ProfileSession() = default;

std::int64_t ProfileSession::nowNs() const { return steadyNs() - origin_ns_; }

std::int64_t ProfileSession::beginRun() {
  std::lock_guard<std::mutex> lock(mu_);
  if (finalized_) throw std::logic_error("profile: session already finalized");
  ProfileRunRecord r;
  r.run_id = static_cast<std::int64_t>(runs_.size());
  r.start_ns = nowNs();
  runs_.push_back(r);
  return r.run_id;
}

void ProfileSession::endRun(std::int64_t run_id, bool ok) {
  std::lock_guard<std::mutex> lock(mu_);
  ProfileRunRecord& r = runs_.at(static_cast<std::size_t>(run_id));
  r.duration_ns = nowNs() - r.start_ns;
  r.status = ok ? "ok" : "error";
}

std::int64_t ProfileSession::beginOperator(std::int64_t run_id, int node_index, const Node& node, bool cuda,
                                           int device, void* stream, const std::vector<const Tensor*>& inputs) {
  std::lock_guard<std::mutex> lock(mu_);
  if (events_.size() >= config_.max_events) {
    ++dropped_;
    return -1;
  }
  ProfileEventRecord e;
  e.event_id = static_cast<std::int64_t>(events_.size());
  e.run_id = run_id;
  e.node_index = node_index;
  e.node_name = node.name;
  e.op_type = node.op_type;
  e.host_thread_id = std::hash<std::thread::id>()(std::this_thread::get_id());
  e.device = cuda ? device : -1;
  e.stream = cuda ? reinterpret_cast<std::uintptr_t>(stream) : 0;
  if (config_.record_shapes)
    for (const Tensor* t : inputs)
      if (t != nullptr) e.shapes.push_back("in:" + shapeText(*t));
  std::unique_ptr<EventPair> pair;
  if (config_.gpu && cuda) {
    if (!pool_.empty()) {
      pair = std::move(pool_.back());
      pool_.pop_back();
    } else {
      pair = std::make_unique<EventPair>();
    }
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    cudaCheck(cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &capture), "cudaStreamIsCapturing");
    pair->captured = capture == cudaStreamCaptureStatusActive;
    // start marker before the host clock starts: the node's launches follow it
    cudaCheck(pair->captured ? cudaEventRecordWithFlags(pair->start, static_cast<cudaStream_t>(stream),
                                                        cudaEventRecordExternal)
                             : cudaEventRecord(pair->start, static_cast<cudaStream_t>(stream)),
              "cudaEventRecord");
  }
  e.cpu_start_ns = nowNs();
  events_.push_back(std::move(e));
  pairs_.push_back(std::move(pair));
  open_start_.push_back(steadyNs());
  return static_cast<std::int64_t>(events_.size()) - 1;
}

void ProfileSession::endOperator(std::int64_t index, bool ok, const std::vector<Tensor*>& outputs) {
  if (index < 0) return;
  const std::int64_t end = steadyNs();
  std::lock_guard<std::mutex> lock(mu_);
  const auto i = static_cast<std::size_t>(index);
  ProfileEventRecord& e = events_.at(i);
  if (config_.cpu) e.cpu_duration_ns = end - open_start_.at(i);
  if (!ok) e.status = "error";
  if (config_.record_shapes)
    for (const Tensor* t : outputs)
      if (t != nullptr && t->defined()) e.shapes.push_back("out:" + shapeText(*t));
  EventPair* pair = pairs_.at(i).get();
  if (pair == nullptr) return;
  if (!ok) {  // a failed node may not have reached its stream: no GPU time
    pool_.push_back(std::move(pairs_[i]));
    return;
  }
  const auto stream = reinterpret_cast<cudaStream_t>(e.stream);
  cudaCheck(pair->captured ? cudaEventRecordWithFlags(pair->end, stream, cudaEventRecordExternal)
                           : cudaEventRecord(pair->end, stream),
            "cudaEventRecord");
}

void ProfileSession::reserve(std::size_t pairs) {
  std::lock_guard<std::mutex> lock(mu_);
  while (pool_.size() < pairs) pool_.push_back(std::make_unique<EventPair>());
}

void ProfileSession::finalize() {
  std::lock_guard<std::mutex> lock(mu_);
  if (finalized_) return;
  for (std::size_t i = 0; i < events_.size(); ++i) {
    EventPair* pair = pairs_[i].get();
    if (pair == nullptr) continue;
    // a captured pair that was never replayed holds no time: it reports unmeasured
    if (cudaEventSynchronize(pair->end) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, pair->start, pair->end) == cudaSuccess)
      events_[i].gpu_duration_ns = static_cast<std::int64_t>(static_cast<double>(ms) * 1e6 + 0.5);
    else
      cudaGetLastError();
  }
  pairs_.clear();
  pool_.clear();
  finalized_ = true;
}

std::string ProfileSession::toJson() const {
  std::lock_guard<std::mutex> lock(mu_);
  if (!finalized_) throw std::logic_error("profile: finalize() before reading the report");
  int driver = 0;
  if (cudaDriverGetVersion(&driver) != cudaSuccess) {
    cudaGetLastError();
    driver = 0;
  }
  std::ostringstream o;
  o << "{\n \"schema\": \"dli.profile.v1\",\n \"clock\": \"steady_clock\",\n \"metadata\": {"
    << "\"created_utc\": \"" << utcNow() << "\", \"process_id\": " << ::getpid()
    << ", \"runtime_version\": \"dli-sm100\", \"cuda_driver_version\": \"" << driver / 1000 << "."
    << (driver % 1000) / 10 << "\", \"cuda_timing\": " << (config_.gpu ? "true" : "false")
    << ", \"record_shapes\": " << (config_.record_shapes ? "true" : "false") << ", \"dropped_events\": " << dropped_
    << "},\n \"runs\": [";
  for (std::size_t i = 0; i < runs_.size(); ++i) {
    const auto& r = runs_[i];
    o << (i ? ",\n  " : "\n  ") << "{\"run_id\": " << r.run_id << ", \"start_ns\": " << r.start_ns
      << ", \"duration_ns\": " << r.duration_ns << ", \"status\": \"" << r.status << "\"}";
  }
  o << "],\n \"events\": [";
  for (std::size_t i = 0; i < events_.size(); ++i) {
    const auto& e = events_[i];
    o << (i ? ",\n  " : "\n  ") << "{\"event_id\": " << e.event_id << ", \"run_id\": " << e.run_id
      << ", \"parent_id\": null, \"category\": \"graph_operator\", \"node_index\": " << e.node_index
      << ", \"node_name\": \"" << jsonEscape(e.node_name) << "\", \"op_type\": \"" << jsonEscape(e.op_type)
      << "\", \"host_thread_id\": " << e.host_thread_id << ", \"cpu_start_ns\": " << e.cpu_start_ns
      << ", \"cpu_duration_ns\": ";
    if (e.cpu_duration_ns >= 0) o << e.cpu_duration_ns;
    else o << "null";
    o << ", \"gpu_duration_ns\": ";
    if (e.gpu_duration_ns >= 0) o << e.gpu_duration_ns;
    else o << "null";
    o << ", \"device\": ";
    if (e.device >= 0) o << e.device;
    else o << "null";
    char sbuf[32];
    std::snprintf(sbuf, sizeof(sbuf), "0x%llx", static_cast<unsigned long long>(e.stream));
    o << ", \"stream\": " << (e.device >= 0 ? "\"" + std::string(sbuf) + "\"" : std::string("null"))
      << ", \"status\": \"" << e.status << "\"";
    if (!e.shapes.empty()) {
      o << ", \"shapes\": [";
      for (std::size_t k = 0; k < e.shapes.size(); ++k) o << (k ? ", " : "") << "\"" << jsonEscape(e.shapes[k]) << "\"";
      o << "]";
    }
    o << "}";
  }
  o << "]\n}\n";
  return o.str();
}

void ProfileSession::writeJson(const std::string& path) const {
  const std::string text = toJson();
  std::ofstream f(path, std::ios::binary | std::ios::trunc);
  if (!f) throw std::runtime_error("profile: cannot write " + path);
  f << text;
}

}  // namespace dli
