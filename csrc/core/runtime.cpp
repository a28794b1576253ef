#include "turbol/runtime.hpp"

#include <ATen/ATen.h>
#include <arpa/inet.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <fstream>
#include <numeric>
#include <random>

#include "kernels.h"

namespace turbol {

// ============================================================================
// CoreEngine
// ============================================================================
CoreEngine& CoreEngine::Instance() {
  static CoreEngine e;
  return e;
}

Status CoreEngine::Initialize(int device_id, int streams_per_device) {
  std::lock_guard<std::mutex> g(mu_);
  device_id_ = device_id;
  if (GetCudaDeviceCount() > device_id && streams_.find(device_id) == streams_.end()) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device_id);
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    std::vector<cudaStream_t> v;
    for (int i = 0; i < streams_per_device; ++i) {
      cudaStream_t s;
      cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, i == 0 ? hi : lo);
      v.push_back(s);
    }
    streams_[device_id] = v;
    cudaSetDevice(prev);
  }
  initialized_ = true;
  return Status::Ok();
}

Status CoreEngine::Shutdown() {
  std::lock_guard<std::mutex> g(mu_);
  for (auto& kv : streams_)
    for (auto s : kv.second) cudaStreamDestroy(s);
  streams_.clear();
  modules_.clear();
  initialized_ = false;
  return Status::Ok();
}

Status CoreEngine::Synchronize() {
  if (GetCudaDeviceCount() == 0) return Status::Ok();
  return FromCuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
}

std::vector<std::string> CoreEngine::ListModules() const {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<std::string> v;
  for (auto& kv : modules_) v.push_back(kv.first);
  return v;
}

cudaStream_t CoreEngine::GetStream(int device_id, int index) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = streams_.find(device_id);
  if (it == streams_.end() || it->second.empty()) return nullptr;
  return it->second[static_cast<size_t>(index) % it->second.size()];
}

// ============================================================================
// TensorUtils
// ============================================================================
namespace {
Status ew(Tensor* out, const Tensor* x, const Tensor* y, float a, int op) {
  if (!out || !out->defined()) return Status::InvalidArgument("null/empty output");
  if (out->dtype() != DataType::kFloat32) return Status::InvalidArgument("TensorUtils supports float32 only");
  const int64_t n = out->numel();
  if ((x && x->numel() != n) || (y && y->numel() != n)) return Status::InvalidArgument("numel mismatch");
  if ((x && x->device() != out->device()) || (y && y->device() != out->device()))
    return Status::InvalidArgument("device mismatch");
  float* o = out->data<float>();
  const float* xp = x ? x->data<float>() : nullptr;
  const float* yp = y ? y->data<float>() : nullptr;
  if (out->is_cuda())
    return FromCuda(tb_elementwise(o, xp, yp, n, a, op, StreamFor(out->torch())), "elementwise");
  for (int64_t i = 0; i < n; ++i) {
    switch (op) {
      case 0: o[i] = a; break;
      case 1: o[i] = xp[i] + a; break;
      case 2: o[i] = xp[i] * a; break;
      case 3: o[i] = xp[i] + yp[i]; break;
      case 4: o[i] = xp[i] - yp[i]; break;
      default: o[i] = xp[i]; break;
    }
  }
  return Status::Ok();
}
}  // namespace

Status TensorUtils::Fill(Tensor* t, float v) { return ew(t, nullptr, nullptr, v, 0); }
Status TensorUtils::AddScalar(Tensor* t, float v) { return ew(t, t, nullptr, v, 1); }
Status TensorUtils::Scale(Tensor* t, float v) { return ew(t, t, nullptr, v, 2); }
Status TensorUtils::Add(const Tensor& a, const Tensor& b, Tensor* out) {
  if (!SameLayout(a, b)) return Status::InvalidArgument("Add: layout mismatch");
  if (!out->defined() || !SameLayout(a, *out)) *out = Tensor(a.shape(), DataType::kFloat32, a.device());
  return ew(out, &a, &b, 0.f, 3);
}
Status TensorUtils::Sub(const Tensor& a, const Tensor& b, Tensor* out) {
  if (!SameLayout(a, b)) return Status::InvalidArgument("Sub: layout mismatch");
  if (!out->defined() || !SameLayout(a, *out)) *out = Tensor(a.shape(), DataType::kFloat32, a.device());
  return ew(out, &a, &b, 0.f, 4);
}
Status TensorUtils::Copy(const Tensor& src, Tensor* dst) {
  if (!dst->defined() || !SameLayout(src, *dst)) *dst = Tensor(src.shape(), DataType::kFloat32, src.device());
  return ew(dst, &src, nullptr, 0.f, 5);
}
bool TensorUtils::SameLayout(const Tensor& a, const Tensor& b) {
  return a.defined() && b.defined() && a.shape() == b.shape() && a.dtype() == b.dtype() && a.device() == b.device();
}

// ============================================================================
// ByteTokenizer
// ============================================================================
std::vector<int> ByteTokenizer::Encode(const std::string& s, bool add_bos, bool add_eos) const {
  std::vector<int> ids;
  ids.reserve(s.size() + 2);
  if (add_bos) ids.push_back(kBos);
  for (unsigned char c : s) ids.push_back(static_cast<int>(c));
  if (add_eos) ids.push_back(kEos);
  return ids;
}

std::string ByteTokenizer::Decode(const std::vector<int>& ids, bool skip_special) const {
  std::string s;
  for (int id : ids) {
    if (id >= 0 && id < 256) s.push_back(static_cast<char>(id));
    else if (!skip_special) s += id == kPad ? "<pad>" : id == kBos ? "<bos>" : id == kEos ? "<eos>" : "<unk>";
  }
  return s;
}

// ============================================================================
// Dataset
// ============================================================================
namespace {

void append_utf8(std::string& o, uint32_t cp) {
  if (cp < 0x80) {
    o.push_back(static_cast<char>(cp));
  } else if (cp < 0x800) {
    o.push_back(static_cast<char>(0xC0 | (cp >> 6)));
    o.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    o.push_back(static_cast<char>(0xE0 | (cp >> 12)));
    o.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    o.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else {
    o.push_back(static_cast<char>(0xF0 | (cp >> 18)));
    o.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
    o.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    o.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  }
}

// Minimal JSON scanner for one flat object: string, number, bool and null
// values; nested objects/arrays are skipped.
struct JsonScan {
  const std::string& s;
  size_t i = 0;
  explicit JsonScan(const std::string& str) : s(str) {}
  void ws() {
    while (i < s.size() && std::isspace(static_cast<unsigned char>(s[i]))) ++i;
  }
  bool str(std::string* out) {
    if (i >= s.size() || s[i] != '"') return false;
    ++i;
    std::string o;
    while (i < s.size()) {
      char c = s[i++];
      if (c == '"') {
        if (out) *out = o;
        return true;
      }
      if (c != '\\') {
        o.push_back(c);
        continue;
      }
      if (i >= s.size()) return false;
      char e = s[i++];
      switch (e) {
        case '"': o.push_back('"'); break;
        case '\\': o.push_back('\\'); break;
        case '/': o.push_back('/'); break;
        case 'b': o.push_back('\b'); break;
        case 'f': o.push_back('\f'); break;
        case 'n': o.push_back('\n'); break;
        case 'r': o.push_back('\r'); break;
        case 't': o.push_back('\t'); break;
        case 'u': {
          if (i + 4 > s.size()) return false;
          uint32_t cp = static_cast<uint32_t>(std::stoul(s.substr(i, 4), nullptr, 16));
          i += 4;
          if (cp >= 0xD800 && cp < 0xDC00 && i + 6 <= s.size() && s[i] == '\\' && s[i + 1] == 'u') {
            const uint32_t lo = static_cast<uint32_t>(std::stoul(s.substr(i + 2, 4), nullptr, 16));
            if (lo >= 0xDC00 && lo < 0xE000) {
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
              i += 6;
            }
          }
          append_utf8(o, cp);
          break;
        }
        default: return false;
      }
    }
    return false;
  }
  bool skip_value(std::string* scalar) {
    ws();
    if (i >= s.size()) return false;
    if (s[i] == '"') return str(scalar);
    if (s[i] == '{' || s[i] == '[') {
      int depth = 0;
      bool in_str = false;
      for (; i < s.size(); ++i) {
        char c = s[i];
        if (in_str) {
          if (c == '\\') ++i;
          else if (c == '"') in_str = false;
          continue;
        }
        if (c == '"') in_str = true;
        else if (c == '{' || c == '[') ++depth;
        else if (c == '}' || c == ']') {
          if (--depth == 0) {
            ++i;
            return true;
          }
        }
      }
      return false;
    }
    size_t b = i;
    while (i < s.size() && s[i] != ',' && s[i] != '}' && !std::isspace(static_cast<unsigned char>(s[i]))) ++i;
    if (scalar) *scalar = s.substr(b, i - b);
    return i > b;
  }
};

}  // namespace

Status Dataset::ParseLine(const std::string& line, DataSample* out) {
  JsonScan js(line);
  js.ws();
  if (js.i >= line.size() || line[js.i] != '{') return Status::InvalidArgument("JSONL line is not an object");
  ++js.i;
  DataSample d;
  while (true) {
    js.ws();
    if (js.i < line.size() && line[js.i] == '}') break;
    std::string key, val;
    if (!js.str(&key)) return Status::InvalidArgument("bad JSON key");
    js.ws();
    if (js.i >= line.size() || line[js.i] != ':') return Status::InvalidArgument("expected ':'");
    ++js.i;
    if (!js.skip_value(&val)) return Status::InvalidArgument("bad JSON value for key " + key);
    if (key == "prompt" || key == "question" || key == "instruction") d.prompt = val;
    else if (key == "chosen" || key == "response" || key == "answer" || key == "output") d.chosen = val;
    else if (key == "rejected") d.rejected = val;
    else if (key == "source") d.source = val;
    else if (key == "reward") {
      try {
        d.reward = std::stof(val);
      } catch (...) {
      }
    }
    js.ws();
    if (js.i < line.size() && line[js.i] == ',') {
      ++js.i;
      continue;
    }
    if (js.i < line.size() && line[js.i] == '}') break;
    return Status::InvalidArgument("expected ',' or '}'");
  }
  *out = d;
  return Status::Ok();
}

Status Dataset::Initialize() {
  entries_.clear();
  for (size_t f = 0; f < cfg_.data_paths.size(); ++f) {
    std::ifstream in(cfg_.data_paths[f], std::ios::binary);
    if (!in) return Status::NotFound("cannot open " + cfg_.data_paths[f]);
    std::string line;
    size_t off = 0;
    while (std::getline(in, line)) {
      bool blank = std::all_of(line.begin(), line.end(), [](unsigned char c) { return std::isspace(c); });
      if (!blank) entries_.push_back(Entry{f, off});
      off += line.size() + 1;
    }
  }
  initialized_ = true;
  epoch_ = 0;
  Reset();
  return Status::Ok();
}

Status Dataset::Shutdown() {
  entries_.clear();
  order_.clear();
  initialized_ = false;
  return Status::Ok();
}

void Dataset::Reset() {
  order_.resize(entries_.size());
  std::iota(order_.begin(), order_.end(), 0);
  if (cfg_.shuffle) {
    std::mt19937_64 g(cfg_.seed + 0x9E3779B97F4A7C15ull * epoch_);
    std::shuffle(order_.begin(), order_.end(), g);
  }
  ++epoch_;
  cursor_ = 0;
}

Status Dataset::Seek(size_t index) {
  if (index > order_.size()) return Status::InvalidArgument("seek past end");
  cursor_ = index;
  return Status::Ok();
}

Status Dataset::GetSample(size_t i, DataSample* out) const {
  if (i >= entries_.size()) return Status::InvalidArgument("sample index out of range");
  const Entry& e = entries_[i];
  std::ifstream in(cfg_.data_paths[e.file], std::ios::binary);
  if (!in) return Status::NotFound("cannot open " + cfg_.data_paths[e.file]);
  in.seekg(static_cast<std::streamoff>(e.offset));
  std::string line;
  std::getline(in, line);
  TURBOL_RETURN_IF_ERROR(ParseLine(line, out));
  out->index = static_cast<int64_t>(i);
  return Status::Ok();
}

Status Dataset::NextBatch(PreprocessedBatch* batch) {
  if (!initialized_) return Status::InvalidArgument("Dataset not initialized");
  if (!HasNext()) return Status::NotFound("end of dataset");
  const int B = static_cast<int>(std::min<size_t>(cfg_.batch_size, order_.size() - cursor_));
  const int L = cfg_.max_seq_length;
  at::Tensor ids = at::full({B, L}, ByteTokenizer::kPad, at::kInt);
  at::Tensor mask = at::zeros({B, L}, at::kInt);
  at::Tensor labels = at::full({B, L}, -100, at::kInt);
  at::Tensor plen = at::zeros({B}, at::kInt);
  batch->sample_indices.clear();
  for (int b = 0; b < B; ++b) {
    DataSample s;
    const size_t idx = order_[cursor_++];
    TURBOL_RETURN_IF_ERROR(GetSample(idx, &s));
    batch->sample_indices.push_back(static_cast<int64_t>(idx));
    std::vector<int> p = tok_.Encode(s.prompt, true, false);
    std::vector<int> r = tok_.Encode(s.chosen, false, true);
    if (!cfg_.truncate && static_cast<int>(p.size() + r.size()) > L)
      return Status::InvalidArgument("sample longer than max_seq_length");
    const int np = std::min<int>(static_cast<int>(p.size()), L);
    const int nr = std::min<int>(static_cast<int>(r.size()), L - np);
    for (int t = 0; t < np; ++t) {
      ids[b][t] = p[t];
      mask[b][t] = 1;
    }
    for (int t = 0; t < nr; ++t) {
      ids[b][np + t] = r[t];
      mask[b][np + t] = 1;
      labels[b][np + t] = r[t];
    }
    plen[b] = np;
  }
  const at::Device dev = cfg_.prefetch_device.torch();
  batch->input_ids = Tensor(ids.to(dev));
  batch->attention_mask = Tensor(mask.to(dev));
  batch->labels = Tensor(labels.to(dev));
  batch->prompt_lens = Tensor(plen.to(dev));
  return Status::Ok();
}

// ============================================================================
// TcpStore.  Wire format: request = op(1) klen(4) key vlen(4) val; reply =
// status(1) vlen(4) val.  Ops: S set, G get (waits server-side up to the
// timeout carried in val), A add (val = decimal delta).
// ============================================================================
namespace {
using Clock = std::chrono::steady_clock;

bool send_all(int fd, const void* p, size_t n) {
  const char* c = static_cast<const char*>(p);
  while (n) {
    ssize_t k = ::send(fd, c, n, MSG_NOSIGNAL);
    if (k <= 0) return false;
    c += k;
    n -= static_cast<size_t>(k);
  }
  return true;
}

// Receives exactly n bytes or fails once the deadline passes (-1 = none).
bool recv_all(int fd, void* p, size_t n, int timeout_ms) {
  char* c = static_cast<char*>(p);
  const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms < 0 ? 0 : timeout_ms);
  while (n) {
    int wait = -1;
    if (timeout_ms >= 0) {
      auto left = std::chrono::duration_cast<std::chrono::milliseconds>(deadline - Clock::now()).count();
      if (left <= 0) return false;
      wait = static_cast<int>(left);
    }
    pollfd pf{fd, POLLIN, 0};
    int r = ::poll(&pf, 1, wait);
    if (r <= 0) return false;
    ssize_t k = ::recv(fd, c, n, 0);
    if (k <= 0) return false;
    c += k;
    n -= static_cast<size_t>(k);
  }
  return true;
}

bool send_msg(int fd, char op, const std::string& a, const std::string& b) {
  uint32_t la = htonl(static_cast<uint32_t>(a.size())), lb = htonl(static_cast<uint32_t>(b.size()));
  std::string buf;
  buf.push_back(op);
  buf.append(reinterpret_cast<char*>(&la), 4);
  buf += a;
  buf.append(reinterpret_cast<char*>(&lb), 4);
  buf += b;
  return send_all(fd, buf.data(), buf.size());
}

bool recv_str(int fd, std::string* s, int timeout_ms) {
  uint32_t l;
  if (!recv_all(fd, &l, 4, timeout_ms)) return false;
  l = ntohl(l);
  s->resize(l);
  return l == 0 || recv_all(fd, &(*s)[0], l, timeout_ms);
}
}  // namespace

TcpStore::TcpStore(const std::string& host, int port, bool is_server, int timeout_ms)
    : host_(host), port_(port), server_(is_server), timeout_ms_(timeout_ms) {
  if (server_) {
    listen_fd_ = ::socket(AF_INET, SOCK_STREAM, 0);
    int one = 1;
    ::setsockopt(listen_fd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_addr.s_addr = htonl(INADDR_ANY);
    a.sin_port = htons(static_cast<uint16_t>(port));
    if (::bind(listen_fd_, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0 || ::listen(listen_fd_, 256) != 0) {
      ::close(listen_fd_);
      throw std::runtime_error("TcpStore: cannot listen on port " + std::to_string(port));
    }
    socklen_t len = sizeof(a);
    ::getsockname(listen_fd_, reinterpret_cast<sockaddr*>(&a), &len);
    port_ = ntohs(a.sin_port);
    accept_thread_ = std::thread([this] { ServeLoop(); });
  }
  // connect with retries until the deadline
  const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms_);
  while (true) {
    addrinfo hints{}, *res = nullptr;
    hints.ai_family = AF_INET;
    hints.ai_socktype = SOCK_STREAM;
    if (::getaddrinfo(host_.c_str(), std::to_string(port_).c_str(), &hints, &res) == 0 && res) {
      int fd = ::socket(res->ai_family, res->ai_socktype, res->ai_protocol);
      if (fd >= 0 && ::connect(fd, res->ai_addr, res->ai_addrlen) == 0) {
        int one = 1;
        ::setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
        fd_ = fd;
        ::freeaddrinfo(res);
        break;
      }
      if (fd >= 0) ::close(fd);
      ::freeaddrinfo(res);
    }
    if (Clock::now() > deadline) {
      stop_ = true;
      if (listen_fd_ >= 0) ::shutdown(listen_fd_, SHUT_RDWR);
      if (accept_thread_.joinable()) accept_thread_.join();
      if (listen_fd_ >= 0) ::close(listen_fd_);
      throw std::runtime_error("TcpStore: timed out connecting to " + host_ + ":" + std::to_string(port_));
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(20));
  }
}

TcpStore::~TcpStore() {
  stop_ = true;
  if (fd_ >= 0) ::close(fd_);
  if (listen_fd_ >= 0) {
    ::shutdown(listen_fd_, SHUT_RDWR);
    ::close(listen_fd_);
  }
  data_cv_.notify_all();
  if (accept_thread_.joinable()) accept_thread_.join();
  for (auto& t : client_threads_)
    if (t.joinable()) t.join();
}

void TcpStore::ServeLoop() {
  while (!stop_) {
    pollfd pf{listen_fd_, POLLIN, 0};
    if (::poll(&pf, 1, 100) <= 0) continue;
    int c = ::accept(listen_fd_, nullptr, nullptr);
    if (c < 0) continue;
    int one = 1;
    ::setsockopt(c, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
    client_threads_.emplace_back([this, c] { ServeClient(c); });
  }
}

void TcpStore::ServeClient(int fd) {
  while (!stop_) {
    pollfd pf{fd, POLLIN, 0};
    int r = ::poll(&pf, 1, 100);
    if (r == 0) continue;
    if (r < 0) break;
    char op;
    if (!recv_all(fd, &op, 1, 5000)) break;
    std::string key, val;
    if (!recv_str(fd, &key, 5000) || !recv_str(fd, &val, 5000)) break;
    std::string reply;
    char status = 0;
    if (op == 'S') {
      std::lock_guard<std::mutex> g(data_mu_);
      data_[key] = val;
      data_cv_.notify_all();
    } else if (op == 'A') {
      std::lock_guard<std::mutex> g(data_mu_);
      int64_t cur = 0;
      auto it = data_.find(key);
      if (it != data_.end()) cur = std::stoll(it->second);
      cur += std::stoll(val);
      data_[key] = std::to_string(cur);
      reply = data_[key];
      data_cv_.notify_all();
    } else if (op == 'G') {
      const int tmo = std::stoi(val);
      std::unique_lock<std::mutex> g(data_mu_);
      const bool ok = data_cv_.wait_for(g, std::chrono::milliseconds(tmo),
                                        [&] { return stop_ || data_.count(key) != 0; });
      if (ok && data_.count(key)) reply = data_[key];
      else status = 1;  // timeout
    } else {
      status = 2;
    }
    std::string buf(1, status);
    uint32_t l = htonl(static_cast<uint32_t>(reply.size()));
    buf.append(reinterpret_cast<char*>(&l), 4);
    buf += reply;
    if (!send_all(fd, buf.data(), buf.size())) break;
  }
  ::close(fd);
}

Status TcpStore::Request(char op, const std::string& key, const std::string& val, int timeout_ms, std::string* reply) {
  std::lock_guard<std::mutex> g(req_mu_);
  if (fd_ < 0) return Status::Unavailable("TcpStore not connected");
  if (!send_msg(fd_, op, key, val)) return Status::Unavailable("TcpStore: send failed");
  char status;
  const int wait = timeout_ms + 5000;
  if (!recv_all(fd_, &status, 1, wait) || !recv_str(fd_, reply, wait))
    return Status::Timeout("TcpStore: no reply for key " + key);
  if (status == 1) return Status::Timeout("TcpStore: timed out waiting for key " + key);
  if (status != 0) return Status::InternalError("TcpStore: bad request");
  return Status::Ok();
}

Status TcpStore::Set(const std::string& key, const std::string& value) {
  std::string r;
  return Request('S', key, value, timeout_ms_, &r);
}

Status TcpStore::Get(const std::string& key, std::string* value, int timeout_ms) {
  const int t = timeout_ms < 0 ? timeout_ms_ : timeout_ms;
  return Request('G', key, std::to_string(t), t, value);
}

Status TcpStore::Add(const std::string& key, int64_t delta, int64_t* result) {
  std::string r;
  TURBOL_RETURN_IF_ERROR(Request('A', key, std::to_string(delta), timeout_ms_, &r));
  if (result) *result = std::stoll(r);
  return Status::Ok();
}

Status TcpStore::Wait(const std::vector<std::string>& keys, int timeout_ms) {
  const int t = timeout_ms < 0 ? timeout_ms_ : timeout_ms;
  const auto deadline = Clock::now() + std::chrono::milliseconds(t);
  for (const auto& k : keys) {
    const auto left = std::chrono::duration_cast<std::chrono::milliseconds>(deadline - Clock::now()).count();
    if (left <= 0) return Status::Timeout("TcpStore: wait deadline passed at key " + k);
    std::string v;
    TURBOL_RETURN_IF_ERROR(Get(k, &v, static_cast<int>(left)));
  }
  return Status::Ok();
}

Status TcpStore::Barrier(const std::string& name, int world, int timeout_ms) {
  int64_t n = 0;
  TURBOL_RETURN_IF_ERROR(Add("__barrier__/" + name, 1, &n));
  if (n == world) TURBOL_RETURN_IF_ERROR(Set("__barrier__/" + name + "/done", "1"));
  return Wait({"__barrier__/" + name + "/done"}, timeout_ms);
}

// ============================================================================
// PipelineSchedule
// ============================================================================
std::vector<PipeOp> PipelineSchedule::OneFOneB(int P, int s, int M) {
  std::vector<PipeOp> ops;
  const int warm = std::min(P - s - 1, M);
  int f = 0, b = 0;
  for (int i = 0; i < warm; ++i) ops.push_back({'F', f++});
  while (f < M) {
    ops.push_back({'F', f++});
    ops.push_back({'B', b++});
  }
  while (b < M) ops.push_back({'B', b++});
  return ops;
}

std::vector<PipeOp> PipelineSchedule::GPipe(int P, int s, int M) {
  (void)P;
  (void)s;
  std::vector<PipeOp> ops;
  for (int i = 0; i < M; ++i) ops.push_back({'F', i});
  for (int i = M - 1; i >= 0; --i) ops.push_back({'B', i});
  return ops;
}

int PipelineSchedule::PeakActivations(const std::vector<PipeOp>& ops) {
  int cur = 0, peak = 0;
  for (const auto& o : ops) {
    cur += o.kind == 'F' ? 1 : -1;
    peak = std::max(peak, cur);
  }
  return peak;
}

// ============================================================================
// KVBlockManager
// ============================================================================
KVBlockManager::KVBlockManager(int num_blocks, int block_size) : num_blocks_(num_blocks), block_size_(block_size) {
  if (num_blocks <= 0 || block_size <= 0) throw std::invalid_argument("KVBlockManager: sizes must be positive");
  Reset();
}

void KVBlockManager::Reset() {
  seqs_.clear();
  free_.resize(num_blocks_);
  // hand out low block ids first
  for (int i = 0; i < num_blocks_; ++i) free_[i] = num_blocks_ - 1 - i;
}

Status KVBlockManager::Allocate(int64_t seq_id, int num_tokens) {
  if (seqs_.count(seq_id)) return Status::AlreadyExists("sequence already allocated");
  const int need = BlocksFor(std::max(num_tokens, 1));
  if (need > static_cast<int>(free_.size())) return Status::OutOfMemory("KV cache out of blocks");
  Seq s;
  for (int i = 0; i < need; ++i) {
    s.blocks.push_back(free_.back());
    free_.pop_back();
  }
  s.len = num_tokens;
  seqs_.emplace(seq_id, std::move(s));
  return Status::Ok();
}

Status KVBlockManager::AppendToken(int64_t seq_id) {
  auto it = seqs_.find(seq_id);
  if (it == seqs_.end()) return Status::NotFound("unknown sequence");
  Seq& s = it->second;
  if (s.len + 1 > static_cast<int>(s.blocks.size()) * block_size_) {
    if (free_.empty()) return Status::OutOfMemory("KV cache out of blocks");
    s.blocks.push_back(free_.back());
    free_.pop_back();
  }
  s.len++;
  return Status::Ok();
}

Status KVBlockManager::Free(int64_t seq_id) {
  auto it = seqs_.find(seq_id);
  if (it == seqs_.end()) return Status::NotFound("unknown sequence");
  for (int b : it->second.blocks) free_.push_back(b);
  seqs_.erase(it);
  return Status::Ok();
}

std::vector<int> KVBlockManager::BlockTable(int64_t seq_id) const {
  auto it = seqs_.find(seq_id);
  return it == seqs_.end() ? std::vector<int>{} : it->second.blocks;
}

int KVBlockManager::SeqLen(int64_t seq_id) const {
  auto it = seqs_.find(seq_id);
  return it == seqs_.end() ? -1 : it->second.len;
}

}  // namespace turbol
