// Observability: Profiler (CPU spans + CUDA event pairs + NVTX3 ranges),
// TensorBoardWriter (TFRecord event files), PrometheusWriter (text
// exposition) and a levelled logger.
//
// Parity with the reference's turbol_vllm/include/turbol/profiler/profiler.hpp:
// same config fields, Span/AggregatedStats records, Begin/EndSpan,
// Begin/EndEvent, Mark, Chrome-trace/JSON export and summary.  Behavioural
// fixes over the reference (turbol_vllm/src/profiler/profiler.cpp):
//   * EndSpan(id) ends the span with that id (the reference pops the most
//     recently opened span whatever id it is given);
//   * EndEvent records the end event and returns; event pairs are resolved
//     lazily (only at GetStats / export) instead of blocking per event;
//   * exports take the lock once (the reference's ExportJSON locks a mutex it
//     then locks again through GetStats and deadlocks);
//   * NVTX ranges are really emitted when enable_nvtx is set;
//   * Mark records a zero-length span.
// TensorBoard files follow the TFRecord framing (length, masked CRC32C of the
// length, payload, masked CRC32C of the payload) and the tensorflow Event /
// Summary protobuf wire format; the reference writes neither CRCs nor valid
// field wire types (turbol_vllm/src/profiler/tensorboard_writer.cpp:41-105).
#pragma once

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "turbol/common.hpp"

namespace turbol {

struct SpanID {
  uint64_t id = 0;
};
struct EventID {
  uint64_t id = 0;
};

struct ProfilerConfig {
  bool enable_nvtx = true;
  bool enable_cuda_timing = true;
  bool enable_memory = false;
  bool enable_cpu = true;
  int cuda_device_id = 0;
  int rank = 0;  // Chrome-trace pid
  std::string export_dir = "/tmp/turbol_profiler";
};

struct Span {
  uint64_t id = 0;
  uint64_t parent = 0;
  std::string name;
  std::string category;
  int device_id = -1;
  int64_t start_ns = 0;
  int64_t end_ns = 0;
  int64_t duration_ns() const { return end_ns - start_ns; }
  std::map<std::string, std::string> metadata;
};

struct AggregatedStats {
  std::string name;
  int64_t count = 0;
  int64_t total_ns = 0;
  int64_t min_ns = INT64_MAX;
  int64_t max_ns = 0;
  double avg_ns() const { return count ? static_cast<double>(total_ns) / static_cast<double>(count) : 0.0; }
};

// Per-collective record: bytes moved and device time, for bandwidth reports.
struct CommRecord {
  std::string name;
  int64_t bytes = 0;
  double ms = 0.0;
  double gbps() const { return ms > 0 ? static_cast<double>(bytes) / (ms * 1e6) : 0.0; }
};

class Profiler {
 public:
  explicit Profiler(const ProfilerConfig& cfg = {});
  ~Profiler();
  Profiler(const Profiler&) = delete;
  Profiler& operator=(const Profiler&) = delete;

  void Enable();
  void Disable();
  bool IsEnabled() const { return enabled_; }

  SpanID BeginSpan(const std::string& name, const std::string& category = "compute", int device_id = -1);
  void EndSpan(SpanID id);

  class Guard {
   public:
    Guard(Profiler* p, const std::string& name, const std::string& category = "compute", int device_id = -1)
        : p_(p), id_(p->BeginSpan(name, category, device_id)) {}
    Guard(const Guard&) = delete;
    Guard& operator=(const Guard&) = delete;
    Guard(Guard&& o) noexcept : p_(o.p_), id_(o.id_) { o.p_ = nullptr; }
    ~Guard() { End(); }
    void End() {
      if (p_) p_->EndSpan(id_);
      p_ = nullptr;
    }

   private:
    Profiler* p_;
    SpanID id_;
  };

  // CUDA event pair on the current torch stream of `device_id`.
  EventID BeginEvent(const std::string& name, int device_id = 0);
  void EndEvent(EventID id);
  void Mark(const std::string& name);
  void RecordComm(const std::string& name, int64_t bytes, double ms);

  std::vector<Span> GetAllSpans() const;
  std::vector<AggregatedStats> GetStats() const;
  std::vector<CommRecord> GetCommRecords() const;
  Status ExportChromeTrace(const std::string& path) const;
  Status ExportJSON(const std::string& path) const;
  std::string Summary() const;
  void PrintSummary() const;
  void Clear();

 private:
  struct EventPair {
    uint64_t id;
    std::string name;
    int device_id;
    cudaEvent_t start = nullptr, end = nullptr;
    int64_t cpu_start_ns = 0;
    bool ended = false;
  };
  int64_t NowNs() const;
  void ResolveEventsLocked() const;
  std::vector<AggregatedStats> StatsLocked() const;

  ProfilerConfig cfg_;
  bool enabled_ = false;
  uint64_t next_id_ = 1;
  std::chrono::steady_clock::time_point t0_;
  mutable std::vector<Span> spans_;  // completed (resolved events are appended lazily)
  std::unordered_map<uint64_t, Span> open_;
  std::vector<uint64_t> stack_;
  mutable std::vector<EventPair> events_;
  std::vector<CommRecord> comms_;
  mutable std::mutex mu_;
};

// ---------------------------------------------------------------------------
class TensorBoardWriter {
 public:
  explicit TensorBoardWriter(const std::string& log_dir);
  ~TensorBoardWriter();
  TensorBoardWriter(const TensorBoardWriter&) = delete;
  TensorBoardWriter& operator=(const TensorBoardWriter&) = delete;

  void AddScalar(const std::string& tag, float value, int64_t step);
  void AddHistogram(const std::string& tag, const float* values, int64_t n, int64_t step);
  void AddText(const std::string& tag, const std::string& text, int64_t step);
  void Flush();
  const std::string& path() const { return path_; }

 private:
  void WriteRecord(const std::string& payload);
  std::string path_;
  std::FILE* f_ = nullptr;
  std::mutex mu_;
};

// CRC32C (Castagnoli) and the TFRecord mask; exposed for tests.
uint32_t Crc32c(const void* data, size_t n);
uint32_t MaskedCrc32c(const void* data, size_t n);

// ---------------------------------------------------------------------------
struct Labels {
  std::map<std::string, std::string> kv;
};

class PrometheusWriter {
 public:
  explicit PrometheusWriter(const std::string& path);
  void Write(const std::string& name, double value, const Labels& labels = {});         // untyped
  void WriteCounter(const std::string& name, double inc, const Labels& labels = {});   // accumulates
  void WriteGauge(const std::string& name, double value, const Labels& labels = {});   // sets
  void ObserveHistogram(const std::string& name, double value, const std::vector<double>& buckets,
                        const Labels& labels = {});
  Status Flush();
  std::string Render() const;

 private:
  struct Hist {
    std::vector<double> bounds;
    std::vector<uint64_t> counts;  // cumulative at render time
    double sum = 0;
    uint64_t count = 0;
  };
  static std::string Key(const Labels& l);
  std::string path_;
  std::map<std::string, std::string> type_;
  std::map<std::string, std::map<std::string, double>> values_;
  std::map<std::string, std::map<std::string, Hist>> hists_;
  mutable std::mutex mu_;
};

// ---------------------------------------------------------------------------
enum class LogLevel { kDebug = 0, kInfo = 1, kWarning = 2, kError = 3, kOff = 4 };
void SetLogLevel(LogLevel l);
LogLevel GetLogLevel();
void Log(LogLevel l, const std::string& msg);

}  // namespace turbol
