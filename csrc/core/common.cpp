// Implementation of the foundation types declared in turbol/common.hpp.
#include "turbol/common.hpp"


#include <algorithm>
#include <cctype>
#include <sstream>
#include <stdexcept>

namespace turbol {

std::string Status::ToString() const {
  if (ok()) return "OK";
  const char* name = "Unknown";
  switch (code_) {
    case StatusCode::kOk: name = "OK"; break;
    case StatusCode::kInvalidArgument: name = "InvalidArgument"; break;
    case StatusCode::kNotFound: name = "NotFound"; break;
    case StatusCode::kAlreadyExists: name = "AlreadyExists"; break;
    case StatusCode::kResourceExhausted: name = "ResourceExhausted"; break;
    case StatusCode::kUnimplemented: name = "Unimplemented"; break;
    case StatusCode::kInternalError: name = "InternalError"; break;
    case StatusCode::kUnavailable: name = "Unavailable"; break;
    case StatusCode::kTimeout: name = "Timeout"; break;
    case StatusCode::kCudaError: name = "CudaError"; break;
  }
  return std::string(name) + ": " + msg_;
}

std::string Shape::ToString() const {
  std::ostringstream o;
  o << "Shape(";
  for (size_t i = 0; i < dims.size(); ++i) o << (i ? ", " : "") << dims[i];
  o << ")";
  return o.str();
}

Device Device::Parse(const std::string& raw) {
  std::string s = raw;
  std::transform(s.begin(), s.end(), s.begin(), [](unsigned char c) { return std::tolower(c); });
  if (s.rfind("cuda", 0) == 0) {
    int id = 0;
    auto pos = s.find(':');
    if (pos != std::string::npos) id = std::stoi(s.substr(pos + 1));
    return CUDA(id);
  }
  if (s.empty() || s == "cpu") return CPU();
  throw std::invalid_argument("unknown device string: " + raw);
}

size_t GetDataTypeSize(DataType t) {
  switch (t) {
    case DataType::kFloat32: return 4;
    case DataType::kFloat16: return 2;
    case DataType::kBFloat16: return 2;
    case DataType::kInt32: return 4;
    case DataType::kInt64: return 8;
    case DataType::kInt16: return 2;
    case DataType::kInt8: return 1;
    case DataType::kUInt8: return 1;
    case DataType::kBool: return 1;
  }
  return 0;
}

std::string DataTypeName(DataType t) {
  switch (t) {
    case DataType::kFloat32: return "float32";
    case DataType::kFloat16: return "float16";
    case DataType::kBFloat16: return "bfloat16";
    case DataType::kInt32: return "int32";
    case DataType::kInt64: return "int64";
    case DataType::kInt16: return "int16";
    case DataType::kInt8: return "int8";
    case DataType::kUInt8: return "uint8";
    case DataType::kBool: return "bool";
  }
  return "unknown";
}

DataType ParseDataType(const std::string& s) {
  if (s == "float32" || s == "float" || s == "f32") return DataType::kFloat32;
  if (s == "float16" || s == "half" || s == "f16") return DataType::kFloat16;
  if (s == "bfloat16" || s == "bf16") return DataType::kBFloat16;
  if (s == "int32" || s == "i32") return DataType::kInt32;
  if (s == "int64" || s == "i64") return DataType::kInt64;
  if (s == "int16") return DataType::kInt16;
  if (s == "int8") return DataType::kInt8;
  if (s == "uint8") return DataType::kUInt8;
  if (s == "bool") return DataType::kBool;
  throw std::invalid_argument("unknown dtype: " + s);
}

at::ScalarType ToTorch(DataType t) {
  switch (t) {
    case DataType::kFloat32: return at::kFloat;
    case DataType::kFloat16: return at::kHalf;
    case DataType::kBFloat16: return at::kBFloat16;
    case DataType::kInt32: return at::kInt;
    case DataType::kInt64: return at::kLong;
    case DataType::kInt16: return at::kShort;
    case DataType::kInt8: return at::kChar;
    case DataType::kUInt8: return at::kByte;
    case DataType::kBool: return at::kBool;
  }
  return at::kFloat;
}

DataType FromTorch(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return DataType::kFloat32;
    case at::kHalf: return DataType::kFloat16;
    case at::kBFloat16: return DataType::kBFloat16;
    case at::kInt: return DataType::kInt32;
    case at::kLong: return DataType::kInt64;
    case at::kShort: return DataType::kInt16;
    case at::kChar: return DataType::kInt8;
    case at::kByte: return DataType::kUInt8;
    case at::kBool: return DataType::kBool;
    default: throw std::invalid_argument("unsupported torch dtype");
  }
}

Tensor::Tensor(const Shape& shape, DataType dtype, Device device) {
  for (auto d : shape.dims)
    if (d < 0) throw std::invalid_argument("Tensor: negative dimension");
  t_ = at::zeros(shape.dims, at::TensorOptions().dtype(ToTorch(dtype)).device(device.torch()));
}

Tensor::Tensor(at::Tensor t) : t_(t.defined() ? t.contiguous() : t) {}

Shape Tensor::shape() const {
  if (!t_.defined()) return Shape();
  return Shape(std::vector<int64_t>(t_.sizes().begin(), t_.sizes().end()));
}

Status Tensor::ToDevice(const Device& device) {
  if (!t_.defined()) return Status::InvalidArgument("ToDevice on an empty tensor");
  if (device.is_cuda() && device.id >= GetCudaDeviceCount())
    return Status::InvalidArgument("no such CUDA device: " + device.ToString());
  if (Device::FromTorch(t_.device()) == device) return Status::Ok();
  t_ = t_.to(device.torch()).contiguous();
  return Status::Ok();
}

Status Tensor::CopyFrom(const Tensor& src) {
  if (!t_.defined() || !src.defined()) return Status::InvalidArgument("CopyFrom with an empty tensor");
  if (src.numel() != numel()) return Status::InvalidArgument("CopyFrom: numel mismatch");
  t_.view(-1).copy_(src.torch().reshape(-1));
  return Status::Ok();
}

Status Tensor::Reshape(const Shape& shape) {
  if (shape.numel() != numel()) return Status::InvalidArgument("Reshape: numel mismatch");
  t_ = t_.view(shape.dims);
  return Status::Ok();
}

int GetCudaDeviceCount() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

Status SetCudaDevice(int id) { return FromCuda(cudaSetDevice(id), "cudaSetDevice"); }

CudaMemoryInfo GetCudaMemoryInfo(int device_id) {
  CudaMemoryInfo info;
  if (device_id < 0 || device_id >= GetCudaDeviceCount()) return info;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device_id);
  size_t f = 0, t = 0;
  if (cudaMemGetInfo(&f, &t) == cudaSuccess) {
    info.free = f;
    info.total = t;
  } else {
    cudaGetLastError();
  }
  cudaSetDevice(prev);
  return info;
}

}  // namespace turbol
