// Per-operator profiling of Engine::run, written as `dli.profile.v1` JSON.
//
// This is the profiling session the reference designs but does not build
// (.codex/profiling_design.md of yncxcw/dl-inference: ProfileSession at :141,
// the schema at :224-270, the stream contract at :185-213). For every graph
// node the session records the host time spent inside Operator::compute
// (steady_clock) and, for nodes with CUDA tensors, the device time between a
// pair of CUDA events recorded on the run's stream before and after the node.
// Nothing synchronises per node: event pairs are resolved in finalize(), the
// only call that may wait for the GPU. CPU and GPU durations are kept apart and
// never added.
//
// Inside stream capture the events are recorded as external event-record nodes
// of the CUDA graph, so replaying the graph times every captured node; finalize()
// then reads the durations of the latest replay.
#pragma once

#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "dli/tensor.h"

namespace dli {

struct Node;

struct ProfileConfig {
  bool cpu = true;             // host time inside Operator::compute
  bool gpu = true;             // CUDA-event time of nodes with CUDA tensors
  bool record_shapes = false;  // dtype and dims of every input and output
  std::size_t max_events = 1000000;  // later events are counted as dropped
};

struct ProfileEventRecord {
  std::int64_t event_id = 0;
  std::int64_t run_id = 0;
  int node_index = 0;
  std::string node_name;
  std::string op_type;
  std::uint64_t host_thread_id = 0;
  std::int64_t cpu_start_ns = 0;     // relative to the session's creation
  std::int64_t cpu_duration_ns = -1;  // -1: not recorded
  std::int64_t gpu_duration_ns = -1;  // -1: not measured (host node, timing off, capture not replayed)
  int device = -1;
  std::uintptr_t stream = 0;
  std::string status = "ok";  // "ok" or "error"
  std::vector<std::string> shapes;
};

struct ProfileRunRecord {
  std::int64_t run_id = 0;
  std::int64_t start_ns = 0;
  std::int64_t duration_ns = 0;
  std::string status = "running";
};

class ProfileSession {
 public:
  explicit ProfileSession(ProfileConfig config = {});
  ~ProfileSession();
  ProfileSession(const ProfileSession&) = delete;
  ProfileSession& operator=(const ProfileSession&) = delete;

  const ProfileConfig& config() const { return config_; }
  bool finalized() const { return finalized_; }

  // Engine hooks. beginOperator returns an event index (or -1 when dropped)
  // that endOperator closes. `cuda` marks a node with CUDA tensors, whose
  // markers go to `stream` (a cudaStream_t).
  std::int64_t beginRun();
  void endRun(std::int64_t run_id, bool ok);
  std::int64_t beginOperator(std::int64_t run_id, int node_index, const Node& node, bool cuda, int device,
                             void* stream, const std::vector<const Tensor*>& inputs);
  void endOperator(std::int64_t index, bool ok, const std::vector<Tensor*>& outputs);

  // Creates `pairs` CUDA event pairs ahead of use, so that timing nodes inside
  // a stream capture creates no events while the capture is open.
  void reserve(std::size_t pairs);
  // Waits for the recorded CUDA events and resolves their durations. Further
  // runs are an error; a second call does nothing.
  void finalize();
  // The dli.profile.v1 document (finalize() first).
  std::string toJson() const;
  void writeJson(const std::string& path) const;
  const std::vector<ProfileEventRecord>& events() const { return events_; }
  const std::vector<ProfileRunRecord>& runs() const { return runs_; }

 private:
  struct EventPair;
  std::int64_t nowNs() const;

  ProfileConfig config_;
  std::int64_t origin_ns_ = 0;
  bool finalized_ = false;
  std::uint64_t dropped_ = 0;
  std::vector<ProfileEventRecord> events_;
  std::vector<ProfileRunRecord> runs_;
  std::vector<std::unique_ptr<EventPair>> pairs_;  // parallel to events_ (null when not timed)
  std::vector<std::unique_ptr<EventPair>> pool_;   // released pairs, reused by later events
  std::vector<std::int64_t> open_start_;           // host start of each event (steady clock)
  mutable std::mutex mu_;
};

}  // namespace dli
