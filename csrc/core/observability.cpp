#include "turbol/observability.hpp"

#if TURBOL_CUDA
#include <nvtx3/nvToolsExt.h>
#else  // CPU-only build: no NVTX (it ships with the CUDA toolkit)
#define nvtxRangePushA(name) ((void)(name))
#define nvtxRangePop() ((void)0)
#define nvtxMarkA(name) ((void)(name))
#endif
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <fstream>
#include <iostream>
#include <sstream>

namespace turbol {
namespace {

std::string json_escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\t': o += "\\t"; break;
      default:
        if (static_cast<unsigned char>(c) < 0x20) {
          char b[8];
          std::snprintf(b, sizeof(b), "\\u%04x", c);
          o += b;
        } else {
          o += c;
        }
    }
  }
  return o;
}

void mkdirs(const std::string& dir) {
  std::string cur;
  for (size_t i = 0; i < dir.size(); ++i) {
    cur += dir[i];
    if (dir[i] == '/' || i + 1 == dir.size()) ::mkdir(cur.c_str(), 0755);
  }
}

}  // namespace

// ============================================================================
// Profiler
// ============================================================================
Profiler::Profiler(const ProfilerConfig& cfg) : cfg_(cfg), t0_(std::chrono::steady_clock::now()) {}

Profiler::~Profiler() {
  std::lock_guard<std::mutex> g(mu_);
  for (auto& e : events_) {
    if (e.start) cudaEventDestroy(e.start);
    if (e.end) cudaEventDestroy(e.end);
  }
}

int64_t Profiler::NowNs() const {
  return std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0_).count();
}

void Profiler::Enable() {
  std::lock_guard<std::mutex> g(mu_);
  if (!enabled_) {
    enabled_ = true;
    if (spans_.empty() && open_.empty()) t0_ = std::chrono::steady_clock::now();
  }
}

void Profiler::Disable() {
  std::lock_guard<std::mutex> g(mu_);
  enabled_ = false;
}

SpanID Profiler::BeginSpan(const std::string& name, const std::string& category, int device_id) {
  std::lock_guard<std::mutex> g(mu_);
  if (!enabled_) return SpanID{0};
  Span s;
  s.id = next_id_++;
  s.parent = stack_.empty() ? 0 : stack_.back();
  s.name = name;
  s.category = category;
  s.device_id = device_id;
  s.start_ns = NowNs();
  if (cfg_.enable_nvtx) nvtxRangePushA(name.c_str());
  stack_.push_back(s.id);
  const uint64_t id = s.id;
  open_.emplace(id, std::move(s));
  return SpanID{id};
}

void Profiler::EndSpan(SpanID id) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = open_.find(id.id);
  if (it == open_.end()) return;
  Span s = std::move(it->second);
  open_.erase(it);
  s.end_ns = NowNs();
  if (cfg_.enable_nvtx) nvtxRangePop();
  auto pos = std::find(stack_.begin(), stack_.end(), id.id);
  if (pos != stack_.end()) stack_.erase(pos);
  spans_.push_back(std::move(s));
}

EventID Profiler::BeginEvent(const std::string& name, int device_id) {
  std::lock_guard<std::mutex> g(mu_);
  if (!enabled_ || !cfg_.enable_cuda_timing || GetCudaDeviceCount() == 0) return EventID{0};
  EventPair e;
  e.id = next_id_++;
  e.name = name;
  e.device_id = device_id;
  cudaEventCreate(&e.start);
  cudaEventCreate(&e.end);
  cudaStream_t st = CurrentStream(device_id);
  cudaEventRecord(e.start, st);
  e.cpu_start_ns = NowNs();
  events_.push_back(e);
  return EventID{e.id};
}

void Profiler::EndEvent(EventID id) {
  std::lock_guard<std::mutex> g(mu_);
  for (auto& e : events_) {
    if (e.id == id.id && !e.ended) {
      cudaStream_t st = CurrentStream(e.device_id);
      cudaEventRecord(e.end, st);
      e.ended = true;
      return;
    }
  }
}

void Profiler::Mark(const std::string& name) {
  std::lock_guard<std::mutex> g(mu_);
  if (!enabled_) return;
  Span s;
  s.id = next_id_++;
  s.parent = stack_.empty() ? 0 : stack_.back();
  s.name = name;
  s.category = "mark";
  s.start_ns = s.end_ns = NowNs();
  if (cfg_.enable_nvtx) nvtxMarkA(name.c_str());
  spans_.push_back(std::move(s));
}

void Profiler::RecordComm(const std::string& name, int64_t bytes, double ms) {
  std::lock_guard<std::mutex> g(mu_);
  comms_.push_back(CommRecord{name, bytes, ms});
}

// Turns ended CUDA event pairs into spans (device time anchored at the CPU
// time of BeginEvent).  Synchronizes only on those events.
void Profiler::ResolveEventsLocked() const {
  std::vector<EventPair> keep;
  for (auto& e : events_) {
    if (!e.ended) {
      keep.push_back(e);
      continue;
    }
    float ms = 0.f;
    cudaEventSynchronize(e.end);
    cudaEventElapsedTime(&ms, e.start, e.end);
    Span s;
    s.id = e.id;
    s.name = e.name;
    s.category = "cuda";
    s.device_id = e.device_id;
    s.start_ns = e.cpu_start_ns;
    s.end_ns = e.cpu_start_ns + static_cast<int64_t>(std::llround(static_cast<double>(ms) * 1e6));
    spans_.push_back(std::move(s));
    cudaEventDestroy(e.start);
    cudaEventDestroy(e.end);
  }
  events_.swap(keep);
}

std::vector<Span> Profiler::GetAllSpans() const {
  std::lock_guard<std::mutex> g(mu_);
  ResolveEventsLocked();
  return spans_;
}

std::vector<AggregatedStats> Profiler::StatsLocked() const {
  ResolveEventsLocked();
  std::map<std::string, AggregatedStats> m;
  for (const auto& s : spans_) {
    if (s.category == "mark") continue;
    auto& a = m[s.name];
    a.name = s.name;
    const int64_t d = s.duration_ns();
    a.count++;
    a.total_ns += d;
    a.min_ns = std::min(a.min_ns, d);
    a.max_ns = std::max(a.max_ns, d);
  }
  std::vector<AggregatedStats> out;
  for (auto& kv : m) out.push_back(kv.second);
  return out;
}

std::vector<AggregatedStats> Profiler::GetStats() const {
  std::lock_guard<std::mutex> g(mu_);
  return StatsLocked();
}

std::vector<CommRecord> Profiler::GetCommRecords() const {
  std::lock_guard<std::mutex> g(mu_);
  return comms_;
}

Status Profiler::ExportChromeTrace(const std::string& path) const {
  std::lock_guard<std::mutex> g(mu_);
  ResolveEventsLocked();
  std::ofstream f(path);
  if (!f) return Status::InvalidArgument("cannot write " + path);
  f << "[";
  bool first = true;
  for (const auto& s : spans_) {
    if (!first) f << ",";
    first = false;
    const bool instant = s.category == "mark";
    f << "\n{\"name\":\"" << json_escape(s.name) << "\",\"cat\":\"" << json_escape(s.category) << "\",\"ph\":\""
      << (instant ? "i" : "X") << "\",\"ts\":" << (static_cast<double>(s.start_ns) / 1000.0);
    if (!instant) f << ",\"dur\":" << (static_cast<double>(s.duration_ns()) / 1000.0);
    f << ",\"pid\":" << cfg_.rank << ",\"tid\":" << s.device_id << ",\"args\":{\"id\":" << s.id
      << ",\"parent\":" << s.parent << "}}";
  }
  f << "\n]\n";
  return f.good() ? Status::Ok() : Status::InternalError("write failed: " + path);
}

Status Profiler::ExportJSON(const std::string& path) const {
  std::lock_guard<std::mutex> g(mu_);
  const auto stats = StatsLocked();
  std::ofstream f(path);
  if (!f) return Status::InvalidArgument("cannot write " + path);
  f << "{\"stats\":[";
  for (size_t i = 0; i < stats.size(); ++i) {
    const auto& a = stats[i];
    f << (i ? "," : "") << "\n{\"name\":\"" << json_escape(a.name) << "\",\"count\":" << a.count
      << ",\"total_ns\":" << a.total_ns << ",\"min_ns\":" << a.min_ns << ",\"max_ns\":" << a.max_ns
      << ",\"avg_ns\":" << a.avg_ns() << "}";
  }
  f << "],\"comms\":[";
  for (size_t i = 0; i < comms_.size(); ++i) {
    const auto& c = comms_[i];
    f << (i ? "," : "") << "\n{\"name\":\"" << json_escape(c.name) << "\",\"bytes\":" << c.bytes
      << ",\"ms\":" << c.ms << ",\"gbps\":" << c.gbps() << "}";
  }
  f << "]}\n";
  return f.good() ? Status::Ok() : Status::InternalError("write failed: " + path);
}

std::string Profiler::Summary() const {
  std::lock_guard<std::mutex> g(mu_);
  auto stats = StatsLocked();
  std::sort(stats.begin(), stats.end(), [](const auto& a, const auto& b) { return a.total_ns > b.total_ns; });
  std::ostringstream o;
  char line[256];
  std::snprintf(line, sizeof(line), "%-32s %8s %12s %12s %12s %12s\n", "name", "count", "total_ms", "avg_ms",
                "min_ms", "max_ms");
  o << line;
  for (const auto& a : stats) {
    std::snprintf(line, sizeof(line), "%-32s %8lld %12.3f %12.3f %12.3f %12.3f\n", a.name.c_str(),
                  static_cast<long long>(a.count), a.total_ns / 1e6, a.avg_ns() / 1e6, a.min_ns / 1e6,
                  a.max_ns / 1e6);
    o << line;
  }
  return o.str();
}

void Profiler::PrintSummary() const { std::cout << Summary() << std::flush; }

void Profiler::Clear() {
  std::lock_guard<std::mutex> g(mu_);
  spans_.clear();
  comms_.clear();
}

// ============================================================================
// CRC32C (Castagnoli, reflected polynomial 0x82F63B78), table driven.
// ============================================================================
namespace {
struct Crc32cTable {
  uint32_t t[256];
  Crc32cTable() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1) ? (c >> 1) ^ 0x82F63B78u : (c >> 1);
      t[i] = c;
    }
  }
};
const Crc32cTable& crc_table() {
  static Crc32cTable tab;
  return tab;
}

// protobuf wire-format helpers
void put_varint(std::string& o, uint64_t v) {
  while (v >= 0x80) {
    o.push_back(static_cast<char>((v & 0x7f) | 0x80));
    v >>= 7;
  }
  o.push_back(static_cast<char>(v));
}
void put_tag(std::string& o, int field, int wire) { put_varint(o, (static_cast<uint64_t>(field) << 3) | wire); }
void put_fixed64(std::string& o, uint64_t v) {
  for (int i = 0; i < 8; ++i) o.push_back(static_cast<char>((v >> (8 * i)) & 0xff));
}
void put_fixed32(std::string& o, uint32_t v) {
  for (int i = 0; i < 4; ++i) o.push_back(static_cast<char>((v >> (8 * i)) & 0xff));
}
void put_double(std::string& o, int field, double d) {
  uint64_t b;
  std::memcpy(&b, &d, 8);
  put_tag(o, field, 1);
  put_fixed64(o, b);
}
void put_float(std::string& o, int field, float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  put_tag(o, field, 5);
  put_fixed32(o, b);
}
void put_bytes(std::string& o, int field, const std::string& s) {
  put_tag(o, field, 2);
  put_varint(o, s.size());
  o += s;
}
void put_int(std::string& o, int field, int64_t v) {
  put_tag(o, field, 0);
  put_varint(o, static_cast<uint64_t>(v));
}

double wall_time() {
  timespec ts;
  clock_gettime(CLOCK_REALTIME, &ts);
  return static_cast<double>(ts.tv_sec) + static_cast<double>(ts.tv_nsec) * 1e-9;
}

// tensorflow.Event: wall_time=1 (double), step=2 (int64), file_version=3 (string), summary=5
std::string event_bytes(int64_t step, const std::string* summary, const std::string* file_version) {
  std::string e;
  put_double(e, 1, wall_time());
  if (step != 0) put_int(e, 2, step);
  if (file_version) put_bytes(e, 3, *file_version);
  if (summary) put_bytes(e, 5, *summary);
  return e;
}
}  // namespace

uint32_t Crc32c(const void* data, size_t n) {
  const auto& t = crc_table().t;
  uint32_t c = 0xFFFFFFFFu;
  const auto* p = static_cast<const uint8_t*>(data);
  for (size_t i = 0; i < n; ++i) c = t[(c ^ p[i]) & 0xff] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

uint32_t MaskedCrc32c(const void* data, size_t n) {
  const uint32_t c = Crc32c(data, n);
  return ((c >> 15) | (c << 17)) + 0xa282ead8u;
}

// ============================================================================
// TensorBoardWriter
// ============================================================================
TensorBoardWriter::TensorBoardWriter(const std::string& log_dir) {
  mkdirs(log_dir);
  char host[256] = {0};
  gethostname(host, sizeof(host) - 1);
  std::ostringstream p;
  p << log_dir << "/events.out.tfevents." << static_cast<long long>(wall_time()) << "." << host << "." << getpid();
  path_ = p.str();
  f_ = std::fopen(path_.c_str(), "wb");
  if (f_) {
    const std::string fv = "brain.Event:2";
    WriteRecord(event_bytes(0, nullptr, &fv));
  }
}

TensorBoardWriter::~TensorBoardWriter() {
  if (f_) {
    std::fflush(f_);
    std::fclose(f_);
  }
}

void TensorBoardWriter::WriteRecord(const std::string& payload) {
  if (!f_) return;
  std::string hdr;
  put_fixed64(hdr, payload.size());
  std::string rec = hdr;
  put_fixed32(rec, MaskedCrc32c(hdr.data(), hdr.size()));
  rec += payload;
  put_fixed32(rec, MaskedCrc32c(payload.data(), payload.size()));
  std::fwrite(rec.data(), 1, rec.size(), f_);
}

void TensorBoardWriter::AddScalar(const std::string& tag, float value, int64_t step) {
  std::string v;  // Summary.Value: tag=1, simple_value=2
  put_bytes(v, 1, tag);
  put_float(v, 2, value);
  std::string s;  // Summary: value=1
  put_bytes(s, 1, v);
  std::lock_guard<std::mutex> g(mu_);
  WriteRecord(event_bytes(step, &s, nullptr));
}

void TensorBoardWriter::AddHistogram(const std::string& tag, const float* values, int64_t n, int64_t step) {
  // HistogramProto: min=1 max=2 num=3 sum=4 sum_squares=5 bucket_limit=6 (packed) bucket=7 (packed)
  double mn = 0, mx = 0, sum = 0, sq = 0;
  if (n > 0) {
    mn = mx = values[0];
    for (int64_t i = 0; i < n; ++i) {
      const double x = values[i];
      mn = std::min(mn, x);
      mx = std::max(mx, x);
      sum += x;
      sq += x * x;
    }
  }
  const int nb = 30;
  std::vector<double> limits, counts(nb, 0.0);
  const double width = (mx > mn) ? (mx - mn) / nb : 1.0;
  for (int b = 0; b < nb; ++b) limits.push_back(b + 1 == nb ? mx + 1e-12 : mn + width * (b + 1));
  for (int64_t i = 0; i < n; ++i) {
    int b = width > 0 ? static_cast<int>((values[i] - mn) / width) : 0;
    counts[std::min(std::max(b, 0), nb - 1)] += 1.0;
  }
  std::string h;
  put_double(h, 1, mn);
  put_double(h, 2, mx);
  put_double(h, 3, static_cast<double>(n));
  put_double(h, 4, sum);
  put_double(h, 5, sq);
  std::string lim, cnt;
  for (double x : limits) {
    uint64_t b;
    std::memcpy(&b, &x, 8);
    put_fixed64(lim, b);
  }
  for (double x : counts) {
    uint64_t b;
    std::memcpy(&b, &x, 8);
    put_fixed64(cnt, b);
  }
  put_bytes(h, 6, lim);
  put_bytes(h, 7, cnt);
  std::string v;
  put_bytes(v, 1, tag);
  put_bytes(v, 5, h);  // Summary.Value.histo = 5
  std::string s;
  put_bytes(s, 1, v);
  std::lock_guard<std::mutex> g(mu_);
  WriteRecord(event_bytes(step, &s, nullptr));
}

void TensorBoardWriter::AddText(const std::string& tag, const std::string& text, int64_t step) {
  // Summary.Value{tag=1, metadata=9{plugin_data=1{plugin_name=1:"text"}}, tensor=8{dtype=1:DT_STRING(7),
  // tensor_shape=2{}, string_val=8}}
  std::string plugin;
  put_bytes(plugin, 1, "text");
  std::string meta;
  put_bytes(meta, 1, plugin);
  std::string tensor;
  put_int(tensor, 1, 7);
  put_bytes(tensor, 2, std::string());
  put_bytes(tensor, 8, text);
  std::string v;
  put_bytes(v, 1, tag);
  put_bytes(v, 9, meta);
  put_bytes(v, 8, tensor);
  std::string s;
  put_bytes(s, 1, v);
  std::lock_guard<std::mutex> g(mu_);
  WriteRecord(event_bytes(step, &s, nullptr));
}

void TensorBoardWriter::Flush() {
  std::lock_guard<std::mutex> g(mu_);
  if (f_) std::fflush(f_);
}

// ============================================================================
// PrometheusWriter
// ============================================================================
PrometheusWriter::PrometheusWriter(const std::string& path) : path_(path) {}

std::string PrometheusWriter::Key(const Labels& l) {
  if (l.kv.empty()) return "";
  std::string k = "{";
  bool first = true;
  for (const auto& kv : l.kv) {
    if (!first) k += ",";
    first = false;
    k += kv.first + "=\"" + json_escape(kv.second) + "\"";
  }
  return k + "}";
}

void PrometheusWriter::Write(const std::string& name, double value, const Labels& labels) {
  std::lock_guard<std::mutex> g(mu_);
  if (!type_.count(name)) type_[name] = "untyped";
  values_[name][Key(labels)] = value;
}

void PrometheusWriter::WriteCounter(const std::string& name, double inc, const Labels& labels) {
  std::lock_guard<std::mutex> g(mu_);
  type_[name] = "counter";
  values_[name][Key(labels)] += inc;
}

void PrometheusWriter::WriteGauge(const std::string& name, double value, const Labels& labels) {
  std::lock_guard<std::mutex> g(mu_);
  type_[name] = "gauge";
  values_[name][Key(labels)] = value;
}

void PrometheusWriter::ObserveHistogram(const std::string& name, double value, const std::vector<double>& buckets,
                                        const Labels& labels) {
  std::lock_guard<std::mutex> g(mu_);
  type_[name] = "histogram";
  auto& h = hists_[name][Key(labels)];
  if (h.bounds.empty()) {
    h.bounds = buckets;
    std::sort(h.bounds.begin(), h.bounds.end());
    h.counts.assign(h.bounds.size(), 0);
  }
  for (size_t i = 0; i < h.bounds.size(); ++i)
    if (value <= h.bounds[i]) h.counts[i]++;
  h.sum += value;
  h.count++;
}

std::string PrometheusWriter::Render() const {
  std::lock_guard<std::mutex> g(mu_);
  std::ostringstream o;
  o.precision(17);
  for (const auto& t : type_) {
    const std::string& name = t.first;
    o << "# TYPE " << name << " " << t.second << "\n";
    if (t.second == "histogram") {
      auto it = hists_.find(name);
      if (it == hists_.end()) continue;
      for (const auto& kh : it->second) {
        std::string lab = kh.first;
        auto with_le = [&](const std::string& le) {
          if (lab.empty()) return "{le=\"" + le + "\"}";
          return lab.substr(0, lab.size() - 1) + ",le=\"" + le + "\"}";
        };
        const Hist& h = kh.second;
        for (size_t i = 0; i < h.bounds.size(); ++i) {
          std::ostringstream b;
          b << h.bounds[i];
          o << name << "_bucket" << with_le(b.str()) << " " << h.counts[i] << "\n";
        }
        o << name << "_bucket" << with_le("+Inf") << " " << h.count << "\n";
        o << name << "_sum" << lab << " " << h.sum << "\n";
        o << name << "_count" << lab << " " << h.count << "\n";
      }
    } else {
      auto it = values_.find(name);
      if (it == values_.end()) continue;
      for (const auto& kv : it->second) o << name << kv.first << " " << kv.second << "\n";
    }
  }
  return o.str();
}

Status PrometheusWriter::Flush() {
  const std::string text = Render();
  const std::string tmp = path_ + ".tmp";
  {
    std::ofstream f(tmp, std::ios::trunc);
    if (!f) return Status::InvalidArgument("cannot write " + tmp);
    f << text;
  }
  if (std::rename(tmp.c_str(), path_.c_str()) != 0) return Status::InternalError("rename failed: " + path_);
  return Status::Ok();
}

// ============================================================================
// Logger (level from TURBOL_LOG_LEVEL = debug|info|warning|error|off)
// ============================================================================
namespace {
std::atomic<int>& log_level_ref() {
  static std::atomic<int> lvl([] {
    const char* e = std::getenv("TURBOL_LOG_LEVEL");
    if (!e) return 1;
    std::string s(e);
    if (s == "debug") return 0;
    if (s == "info") return 1;
    if (s == "warning" || s == "warn") return 2;
    if (s == "error") return 3;
    if (s == "off") return 4;
    return 1;
  }());
  return lvl;
}
std::mutex& log_mu() {
  static std::mutex m;
  return m;
}
}  // namespace

void SetLogLevel(LogLevel l) { log_level_ref() = static_cast<int>(l); }
LogLevel GetLogLevel() { return static_cast<LogLevel>(log_level_ref().load()); }

void Log(LogLevel l, const std::string& msg) {
  if (static_cast<int>(l) < log_level_ref().load()) return;
  static const char* names[] = {"DEBUG", "INFO", "WARNING", "ERROR"};
  std::lock_guard<std::mutex> g(log_mu());
  std::cerr << "[turbol " << names[static_cast<int>(l)] << "] " << msg << std::endl;
}

}  // namespace turbol
