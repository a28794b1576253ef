// Config: a typed key -> string store persisted as "key=value" text.
//
// Parity: same file format and API as the reference
// (turbol_vllm/include/turbol/core/config.hpp:12-79, src/core/config.cpp:19-108):
// '#' comment lines and blank lines are skipped, keys and values are trimmed,
// Save writes the entries sorted by key, booleans accept true/1/yes/on and
// false/0/no/off, floats are written with 9 significant digits (exact round
// trip), a missing file is kNotFound and a line without '=' is
// kInvalidArgument.  Keeping the format identical lets checkpoints written here
// be read by the reference's Config::Load and vice versa.
#pragma once

#include <map>
#include <string>
#include <vector>

#include "turbol/common.hpp"

namespace turbol {

class Config {
 public:
  Status Load(const std::string& path);
  Status Save(const std::string& path) const;

  bool Has(const std::string& key) const { return data_.count(key) != 0; }
  void Erase(const std::string& key) { data_.erase(key); }
  void Clear() { data_.clear(); }
  size_t size() const { return data_.size(); }
  std::vector<std::string> Keys() const;

  void SetString(const std::string& key, const std::string& v) { data_[key] = v; }
  void SetInt(const std::string& key, long long v) { data_[key] = std::to_string(v); }
  void SetFloat(const std::string& key, double v, bool single_precision = true);
  void SetBool(const std::string& key, bool v) { data_[key] = v ? "true" : "false"; }

  std::string GetString(const std::string& key, const std::string& def) const;
  long long GetInt(const std::string& key, long long def) const;
  double GetFloat(const std::string& key, double def) const;
  bool GetBool(const std::string& key, bool def) const;

 private:
  std::map<std::string, std::string> data_;  // ordered: Save is sorted by key
};

}  // namespace turbol
