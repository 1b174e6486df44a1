// Read-only memory-mapped safetensors file: an 8-byte little-endian header
// length, a JSON header mapping tensor names to dtype / shape /
// data_offsets, then the raw tensor bytes.  The generator only needs float32
// tensors with exact shapes, as the reference's SafetensorsFile::Expect
// (safetensors.hpp:36-65, safetensors.cpp:156-247).
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace ovb {

struct TensorInfo {
  std::string dtype;
  std::vector<uint64_t> shape;
  uint64_t begin = 0;  // byte offsets into the data section
  uint64_t end = 0;
};

class SafetensorsFile {
 public:
  explicit SafetensorsFile(const std::string& path);
  ~SafetensorsFile();
  SafetensorsFile(const SafetensorsFile&) = delete;
  SafetensorsFile& operator=(const SafetensorsFile&) = delete;

  // The float32 tensor `name` with exactly `shape`; throws ovb::Error
  // (OV_ERR_IO) naming the tensor otherwise.
  const float* ExpectF32(const std::string& name, const std::vector<uint64_t>& shape) const;
  bool Has(const std::string& name) const { return tensors_.count(name) != 0; }

 private:
  void Parse(const char* json, size_t size);

  int fd_ = -1;
  const uint8_t* map_ = nullptr;
  size_t size_ = 0;
  const uint8_t* data_ = nullptr;
  size_t data_size_ = 0;
  std::map<std::string, TensorInfo> tensors_;
  std::string path_;
};

}  // namespace ovb
