// Move-only owner of a device allocation with the reference's grow-only
// Reserve semantics (device.hpp:33-77: Reserve reallocates when the count
// exceeds the capacity and discards the contents).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <string>
#include <utility>

#include "internal.hpp"

namespace ovb {

template <typename T>
class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  explicit DeviceBuffer(size_t count) { Resize(count); }
  ~DeviceBuffer() { Release(); }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  DeviceBuffer(DeviceBuffer&& other) noexcept
      : data_(std::exchange(other.data_, nullptr)), count_(std::exchange(other.count_, 0)) {}
  DeviceBuffer& operator=(DeviceBuffer&& other) noexcept {
    Release();
    data_ = std::exchange(other.data_, nullptr);
    count_ = std::exchange(other.count_, 0);
    return *this;
  }

  // Returns true when it reallocated (pointers taken earlier are invalid).
  bool Reserve(size_t count) {
    if (count <= count_ && data_ != nullptr) return false;
    Resize(count);
    return true;
  }

  T* get() const { return data_; }
  size_t size() const { return count_; }

 private:
  void Resize(size_t count) {
    Release();
    void* p = nullptr;
    const size_t bytes = (count == 0 ? 1 : count) * sizeof(T);
    const cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      throw Error(e == cudaErrorMemoryAllocation ? OV_ERR_OOM : OV_ERR_CUDA,
                  "cudaMalloc of " + std::to_string(bytes) + " bytes: " + cudaGetErrorString(e));
    }
    data_ = static_cast<T*>(p);
    count_ = count;
  }
  void Release() noexcept {
    if (data_ != nullptr) (void)cudaFree(data_);
    data_ = nullptr;
    count_ = 0;
  }

  T* data_ = nullptr;
  size_t count_ = 0;
};

}  // namespace ovb
