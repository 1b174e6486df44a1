// Host-side internals shared by the translation units of the library:
// thread-local error state behind ov_last_error, CUDA status checks, the
// per-device error word kernels report bounded-wait timeouts into, and
// TMA tensor-map encoding through the driver entry point.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "ov_runtime.h"

namespace ovb {

// Bits of the device error word kernels set (see ov_take_device_errors).
constexpr uint32_t kErrWaitTimeout = OV_DEVICE_WAIT_TIMEOUT;
constexpr uint32_t kErrBadArgument = OV_DEVICE_BAD_ARGUMENT;

// Records `message` as the calling thread's last error and returns status.
int Fail(int status, const std::string& message);
int CudaFail(cudaError_t error, const char* what);
void ClearError();

// Error thrown inside the C++ layers; converted to a status at the C-ABI
// (the reference's GpuError, device.hpp:16-19).
class Error : public std::runtime_error {
 public:
  Error(int status, const std::string& message)
      : std::runtime_error(message), status_(status) {}
  int status() const { return status_; }

 private:
  int status_;
};

inline void Check(cudaError_t error, const char* what) {
  if (error != cudaSuccess)
    throw Error(OV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(error));
}

inline void CheckStatus(int status) {
  if (status != OV_OK) throw Error(status, "status " + std::to_string(status));
}

// The device error word of the current device (allocated on first use).
uint32_t* DeviceErrorWord();

// The status word of ov_gemm_f16_noalloc on the current device (a static
// device array), or nullptr while that entry point has not run there.
uint32_t* NoAllocStatusWord();

// Streaming multiprocessors of the current device.
int SmCount();

// cuTensorMapEncodeTiled for a 2-D row-major tensor of `rows` x `inner`
// elements with `row_bytes` between rows; box is box_rows x box_inner.
void EncodeTensorMap2D(CUtensorMap* map, const void* base, CUtensorMapDataType type,
                       uint64_t inner, uint64_t rows, uint64_t row_bytes, uint32_t box_inner,
                       uint32_t box_rows, CUtensorMapSwizzle swizzle);

inline cudaStream_t AsStream(ov_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Runs `body` and converts exceptions to a status + thread-local message.
template <typename Body>
int Guard(const char* prefix, Body&& body) {
  try {
    ClearError();
    body();
    return OV_OK;
  } catch (const Error& e) {
    return Fail(e.status(), std::string(prefix) + e.what());
  } catch (const std::bad_alloc&) {
    return Fail(OV_ERR_OOM, std::string(prefix) + "host allocation failed");
  } catch (const std::exception& e) {
    return Fail(OV_ERR_INVALID, std::string(prefix) + e.what());
  }
}

#define OV_REQUIRE(cond, msg) \
  do {                        \
    if (!(cond)) throw ::ovb::Error(OV_ERR_INVALID, msg); \
  } while (0)

}  // namespace ovb
