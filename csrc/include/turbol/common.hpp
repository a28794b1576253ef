// Foundation types of the turbol_b200 host runtime: Status, Shape, Device,
// DataType and Tensor.
//
// Parity: the error model and value types follow the reference's
// turbol_vllm/include/turbol/common.hpp:97-381 (StatusCode values, Device
// "CPU"/"CUDA:n" strings, the nine dtypes).  Two behaviours differ on purpose:
//   * kInt32 is 4 bytes (the reference's CPU tree reports 8, a bug).
//   * Tensor storage comes from the PyTorch allocators (the CUDA caching
//     allocator on the device), is zero-initialised, and is shared zero-copy
//     with torch through Tensor::torch().  The reference mallocs/cudaMallocs per
//     tensor and leaves memory uninitialised.
#pragma once

#include <ATen/ATen.h>

#include "turbol/cuda_compat.hpp"

#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace turbol {

enum class StatusCode : int {
  kOk = 0,
  kInvalidArgument = 1,
  kNotFound = 2,
  kAlreadyExists = 3,
  kResourceExhausted = 4,
  kUnimplemented = 5,
  kInternalError = 6,
  kUnavailable = 7,
  kTimeout = 8,
  kCudaError = 100,
  // Older names of this library, kept as aliases of the same values.
  kOutOfMemory = kResourceExhausted,
  kNotImplemented = kUnimplemented,
};

class Status {
 public:
  Status() = default;
  Status(StatusCode c, std::string m) : code_(c), msg_(std::move(m)) {}
  static Status Ok() { return {}; }
  static Status InvalidArgument(const std::string& m) { return {StatusCode::kInvalidArgument, m}; }
  static Status NotFound(const std::string& m) { return {StatusCode::kNotFound, m}; }
  static Status AlreadyExists(const std::string& m) { return {StatusCode::kAlreadyExists, m}; }
  static Status ResourceExhausted(const std::string& m) { return {StatusCode::kResourceExhausted, m}; }
  static Status OutOfMemory(const std::string& m) { return ResourceExhausted(m); }
  static Status Unimplemented(const std::string& m) { return {StatusCode::kUnimplemented, m}; }
  static Status NotImplemented(const std::string& m) { return Unimplemented(m); }
  static Status InternalError(const std::string& m) { return {StatusCode::kInternalError, m}; }
  static Status Unavailable(const std::string& m) { return {StatusCode::kUnavailable, m}; }
  static Status Timeout(const std::string& m) { return {StatusCode::kTimeout, m}; }
  static Status CudaError(const std::string& m) { return {StatusCode::kCudaError, m}; }

  bool ok() const { return code_ == StatusCode::kOk; }
  StatusCode code() const { return code_; }
  const std::string& message() const { return msg_; }
  std::string ToString() const;

 private:
  StatusCode code_ = StatusCode::kOk;
  std::string msg_;
};

#define TURBOL_RETURN_IF_ERROR(expr)   \
  do {                                 \
    ::turbol::Status _st = (expr);     \
    if (!_st.ok()) return _st;         \
  } while (0)

// Converts a cudaError_t (returned as int by the kernel launchers) to a Status.
inline Status FromCuda(int err, const char* what) {
  if (err == 0) return Status::Ok();
  return Status::CudaError(std::string(what) + ": " + cudaGetErrorString(static_cast<cudaError_t>(err)));
}

struct Shape {
  std::vector<int64_t> dims;
  Shape() = default;
  explicit Shape(std::vector<int64_t> d) : dims(std::move(d)) {}
  Shape(std::initializer_list<int64_t> d) : dims(d) {}
  size_t size() const { return dims.size(); }
  int64_t operator[](size_t i) const { return dims[i]; }
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
  }
  bool operator==(const Shape& o) const { return dims == o.dims; }
  std::string ToString() const;
};

struct Device {
  enum class Type { kCPU, kCUDA };
  Type type = Type::kCPU;
  int id = 0;
  static Device CPU() { return {Type::kCPU, 0}; }
  static Device CUDA(int i = 0) { return {Type::kCUDA, i}; }
  bool is_cuda() const { return type == Type::kCUDA; }
  bool is_cpu() const { return type == Type::kCPU; }
  bool operator==(const Device& o) const { return type == o.type && (type == Type::kCPU || id == o.id); }
  bool operator!=(const Device& o) const { return !(*this == o); }
  std::string ToString() const { return is_cuda() ? "CUDA:" + std::to_string(id) : "CPU"; }
  at::Device torch() const { return is_cuda() ? at::Device(at::kCUDA, id) : at::Device(at::kCPU); }
  static Device FromTorch(const at::Device& d) { return d.is_cuda() ? CUDA(d.index() < 0 ? 0 : d.index()) : CPU(); }
  // Accepts "cpu", "cuda", "cuda:N", "CPU", "CUDA:N".
  static Device Parse(const std::string& s);
};

enum class DataType { kFloat32, kFloat16, kBFloat16, kInt32, kInt64, kInt16, kInt8, kUInt8, kBool };

size_t GetDataTypeSize(DataType t);
std::string DataTypeName(DataType t);
DataType ParseDataType(const std::string& s);
at::ScalarType ToTorch(DataType t);
DataType FromTorch(at::ScalarType t);

// Owning, contiguous tensor.  Copy construction/assignment deep-copy (the
// reference's semantics); moves transfer ownership.  `torch()` exposes the
// storage zero-copy as an at::Tensor.
class Tensor {
 public:
  Tensor() = default;
  Tensor(const Shape& shape, DataType dtype, Device device);
  explicit Tensor(at::Tensor t);  // adopts t (made contiguous), no copy when already contiguous

  Tensor(const Tensor& o) : t_(o.t_.defined() ? o.t_.clone() : at::Tensor()) {}
  Tensor& operator=(const Tensor& o) {
    if (this != &o) t_ = o.t_.defined() ? o.t_.clone() : at::Tensor();
    return *this;
  }
  Tensor(Tensor&&) noexcept = default;
  Tensor& operator=(Tensor&&) noexcept = default;

  bool defined() const { return t_.defined(); }
  int64_t numel() const { return t_.defined() ? t_.numel() : 0; }
  Shape shape() const;
  DataType dtype() const { return t_.defined() ? FromTorch(t_.scalar_type()) : DataType::kFloat32; }
  Device device() const { return t_.defined() ? Device::FromTorch(t_.device()) : Device::CPU(); }
  bool is_cuda() const { return t_.defined() && t_.is_cuda(); }
  size_t size_bytes() const { return t_.defined() ? t_.nbytes() : 0; }

  void* data() { return t_.defined() ? t_.data_ptr() : nullptr; }
  const void* data() const { return t_.defined() ? t_.data_ptr() : nullptr; }
  template <typename T> T* data() { return static_cast<T*>(data()); }
  template <typename T> const T* data() const { return static_cast<const T*>(data()); }

  Tensor Clone() const { return Tensor(t_.clone()); }
  // Moves the storage to `device` in place (the reference's ToDevice contract).
  Status ToDevice(const Device& device);
  // Copies from `src` (same numel; dtype converted) into this tensor.
  Status CopyFrom(const Tensor& src);
  Status Reshape(const Shape& shape);

  at::Tensor& torch() { return t_; }
  const at::Tensor& torch() const { return t_; }

 private:
  at::Tensor t_;
};

// CUDA helpers (reference common.hpp:386-428 equivalents).
int GetCudaDeviceCount();
Status SetCudaDevice(int id);
struct CudaMemoryInfo {
  size_t total = 0, free = 0;
  size_t used() const { return total - free; }
  double utilization() const { return total ? static_cast<double>(used()) / static_cast<double>(total) : 0.0; }
};
CudaMemoryInfo GetCudaMemoryInfo(int device_id);

// Current torch CUDA stream of the tensor's device (kernels launch there).
inline cudaStream_t StreamFor(const at::Tensor& t) { return CurrentStream(t.device().index()); }

}  // namespace turbol
