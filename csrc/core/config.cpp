#include "turbol/config.hpp"

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cstdlib>
#include <cstdio>
#include <fstream>
#include <sstream>

namespace turbol {
namespace {

std::string trim(const std::string& s) {
  size_t b = 0, e = s.size();
  while (b < e && std::isspace(static_cast<unsigned char>(s[b]))) ++b;
  while (e > b && std::isspace(static_cast<unsigned char>(s[e - 1]))) --e;
  return s.substr(b, e - b);
}

}  // namespace

Status Config::Load(const std::string& path) {
  std::ifstream in(path);
  if (!in) return Status::NotFound("Cannot open config file: " + path);
  std::string line;
  int n = 0;
  while (std::getline(in, line)) {
    ++n;
    const std::string t = trim(line);
    if (t.empty() || t[0] == '#') continue;
    const auto eq = t.find('=');
    if (eq == std::string::npos)
      return Status::InvalidArgument("Malformed config line " + std::to_string(n) + ": " + t);
    const std::string k = trim(t.substr(0, eq));
    if (k.empty()) return Status::InvalidArgument("Empty key on config line " + std::to_string(n));
    data_[k] = trim(t.substr(eq + 1));
  }
  return Status::Ok();
}

Status Config::Save(const std::string& path) const {
  std::ofstream out(path, std::ios::trunc);
  if (!out) return Status::InvalidArgument("Cannot write config file: " + path);
  for (const auto& kv : data_) out << kv.first << "=" << kv.second << "\n";
  out.flush();
  return out.good() ? Status::Ok() : Status::InternalError("Failed writing config: " + path);
}

std::vector<std::string> Config::Keys() const {
  std::vector<std::string> k;
  for (const auto& kv : data_) k.push_back(kv.first);
  return k;
}

void Config::SetFloat(const std::string& key, double v, bool single_precision) {
  char buf[64];
  std::snprintf(buf, sizeof(buf), single_precision ? "%.9g" : "%.17g", v);
  data_[key] = buf;
}

std::string Config::GetString(const std::string& key, const std::string& def) const {
  auto it = data_.find(key);
  return it == data_.end() ? def : it->second;
}

long long Config::GetInt(const std::string& key, long long def) const {
  auto it = data_.find(key);
  if (it == data_.end()) return def;
  const std::string v = trim(it->second);
  if (v.empty()) return def;
  char* end = nullptr;
  errno = 0;
  const long long r = std::strtoll(v.c_str(), &end, 10);
  if (errno != 0 || end != v.c_str() + v.size()) return def;
  return r;
}

double Config::GetFloat(const std::string& key, double def) const {
  auto it = data_.find(key);
  if (it == data_.end()) return def;
  const std::string v = trim(it->second);
  if (v.empty()) return def;
  char* end = nullptr;
  errno = 0;
  const double r = std::strtod(v.c_str(), &end);
  if (errno != 0 || end != v.c_str() + v.size()) return def;
  return r;
}

bool Config::GetBool(const std::string& key, bool def) const {
  auto it = data_.find(key);
  if (it == data_.end()) return def;
  std::string v = trim(it->second);
  std::transform(v.begin(), v.end(), v.begin(), [](unsigned char c) { return std::tolower(c); });
  if (v == "true" || v == "1" || v == "yes" || v == "on") return true;
  if (v == "false" || v == "0" || v == "no" || v == "off") return false;
  return def;
}

}  // namespace turbol
