// Minimal safetensors reader for float32 checkpoints (see safetensors.hpp).
#include "safetensors.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cstring>

#include "internal.hpp"

namespace ovb {
namespace {

// A small recursive-descent reader for the header's JSON subset: objects,
// arrays, strings without escapes other than \" and \\, and integers.
class JsonCursor {
 public:
  JsonCursor(const char* p, size_t n) : p_(p), end_(p + n) {}
  void Skip() {
    while (p_ < end_ && std::isspace(static_cast<unsigned char>(*p_))) ++p_;
  }
  bool Eat(char c) {
    Skip();
    if (p_ < end_ && *p_ == c) {
      ++p_;
      return true;
    }
    return false;
  }
  void Expect(char c) {
    if (!Eat(c)) throw Error(OV_ERR_IO, std::string("safetensors header: expected '") + c + "'");
  }
  std::string String() {
    Expect('"');
    std::string out;
    while (p_ < end_ && *p_ != '"') {
      if (*p_ == '\\' && p_ + 1 < end_) ++p_;
      out.push_back(*p_++);
    }
    Expect('"');
    return out;
  }
  uint64_t Integer() {
    Skip();
    uint64_t v = 0;
    bool any = false;
    while (p_ < end_ && std::isdigit(static_cast<unsigned char>(*p_))) {
      v = v * 10 + static_cast<uint64_t>(*p_++ - '0');
      any = true;
    }
    if (!any) throw Error(OV_ERR_IO, "safetensors header: expected an integer");
    return v;
  }
  std::vector<uint64_t> IntegerArray() {
    std::vector<uint64_t> out;
    Expect('[');
    if (Eat(']')) return out;
    do out.push_back(Integer());
    while (Eat(','));
    Expect(']');
    return out;
  }
  // Skips any JSON value (used for __metadata__).
  void Value() {
    Skip();
    if (p_ >= end_) throw Error(OV_ERR_IO, "safetensors header: truncated");
    if (*p_ == '"') {
      (void)String();
    } else if (*p_ == '{') {
      ++p_;
      if (Eat('}')) return;
      do {
        (void)String();
        Expect(':');
        Value();
      } while (Eat(','));
      Expect('}');
    } else if (*p_ == '[') {
      ++p_;
      if (Eat(']')) return;
      do Value();
      while (Eat(','));
      Expect(']');
    } else {
      while (p_ < end_ && *p_ != ',' && *p_ != '}' && *p_ != ']') ++p_;
    }
  }

 private:
  const char* p_;
  const char* end_;
};

}  // namespace

SafetensorsFile::SafetensorsFile(const std::string& path) : path_(path) {
  fd_ = ::open(path.c_str(), O_RDONLY);
  if (fd_ < 0) throw Error(OV_ERR_IO, "cannot open " + path);
  struct stat st {};
  if (::fstat(fd_, &st) != 0 || st.st_size < 8) throw Error(OV_ERR_IO, path + ": too small");
  size_ = static_cast<size_t>(st.st_size);
  void* m = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
  if (m == MAP_FAILED) throw Error(OV_ERR_IO, "cannot map " + path);
  map_ = static_cast<const uint8_t*>(m);
  uint64_t header = 0;
  std::memcpy(&header, map_, 8);
  if (header > size_ - 8) throw Error(OV_ERR_IO, path + ": header length out of range");
  Parse(reinterpret_cast<const char*>(map_ + 8), static_cast<size_t>(header));
  data_ = map_ + 8 + header;
  data_size_ = size_ - 8 - static_cast<size_t>(header);
  for (const auto& [name, t] : tensors_)
    if (t.begin > t.end || t.end > data_size_)
      throw Error(OV_ERR_IO, path + ": tensor " + name + " lies outside the file");
}

SafetensorsFile::~SafetensorsFile() {
  if (map_ != nullptr) ::munmap(const_cast<uint8_t*>(map_), size_);
  if (fd_ >= 0) ::close(fd_);
}

void SafetensorsFile::Parse(const char* json, size_t size) {
  JsonCursor c(json, size);
  c.Expect('{');
  if (c.Eat('}')) return;
  do {
    const std::string name = c.String();
    c.Expect(':');
    if (name == "__metadata__") {
      c.Value();
      continue;
    }
    TensorInfo info;
    c.Expect('{');
    do {
      const std::string key = c.String();
      c.Expect(':');
      if (key == "dtype") {
        info.dtype = c.String();
      } else if (key == "shape") {
        info.shape = c.IntegerArray();
      } else if (key == "data_offsets") {
        const std::vector<uint64_t> o = c.IntegerArray();
        if (o.size() != 2) throw Error(OV_ERR_IO, "safetensors header: data_offsets of " + name);
        info.begin = o[0];
        info.end = o[1];
      } else {
        c.Value();
      }
    } while (c.Eat(','));
    c.Expect('}');
    tensors_[name] = info;
  } while (c.Eat(','));
  c.Expect('}');
}

const float* SafetensorsFile::ExpectF32(const std::string& name,
                                        const std::vector<uint64_t>& shape) const {
  const auto it = tensors_.find(name);
  if (it == tensors_.end()) throw Error(OV_ERR_IO, "missing tensor " + name);
  const TensorInfo& t = it->second;
  if (t.dtype != "F32") throw Error(OV_ERR_IO, "tensor " + name + " is " + t.dtype + ", not F32");
  if (t.shape != shape) throw Error(OV_ERR_IO, "tensor " + name + " has an unexpected shape");
  uint64_t elements = 1;
  for (uint64_t d : shape) elements *= d;
  if (t.end - t.begin != elements * 4) throw Error(OV_ERR_IO, "tensor " + name + " size mismatch");
  return reinterpret_cast<const float*>(data_ + t.begin);
}

}  // namespace ovb
