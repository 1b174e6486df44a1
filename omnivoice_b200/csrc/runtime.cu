// The device runtime C-ABI (ov_runtime.h): the replacement of the
// reference's HIP helper layer (device.hpp:16-77) on the CUDA runtime.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "internal.hpp"
#include "ov_runtime.h"

namespace ovb {
namespace {

thread_local int t_status = OV_OK;
thread_local std::string t_message;

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
uint32_t* g_error_words[kMaxDevices] = {};
int g_sm_counts[kMaxDevices] = {};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn GetEncodeTiled() {
  static EncodeTiledFn fn = [] {
    void* symbol = nullptr;
    cudaDriverEntryPointQueryResult query{};
    const cudaError_t e =
        cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &symbol, cudaEnableDefault, &query);
    if (e != cudaSuccess || query != cudaDriverEntryPointSuccess) return EncodeTiledFn{nullptr};
    return reinterpret_cast<EncodeTiledFn>(symbol);
  }();
  return fn;
}

int CurrentDevice() {
  int device = 0;
  Check(cudaGetDevice(&device), "cudaGetDevice");
  if (device < 0 || device >= kMaxDevices) throw Error(OV_ERR_INVALID, "device index");
  return device;
}

}  // namespace

int Fail(int status, const std::string& message) {
  t_status = status;
  t_message = message;
  return status;
}

int CudaFail(cudaError_t error, const char* what) {
  return Fail(OV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(error));
}

void ClearError() {
  t_status = OV_OK;
  t_message.clear();
}

uint32_t* DeviceErrorWord() {
  const int device = CurrentDevice();
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_error_words[device] == nullptr) {
    void* p = nullptr;
    Check(cudaMalloc(&p, 256), "allocate device error word");
    Check(cudaMemset(p, 0, 256), "clear device error word");
    g_error_words[device] = static_cast<uint32_t*>(p);
  }
  return g_error_words[device];
}

int SmCount() {
  const int device = CurrentDevice();
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_sm_counts[device] == 0) {
    int count = 0;
    Check(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device),
          "query SM count");
    g_sm_counts[device] = count;
  }
  return g_sm_counts[device];
}

void EncodeTensorMap2D(CUtensorMap* map, const void* base, CUtensorMapDataType type,
                       uint64_t inner, uint64_t rows, uint64_t row_bytes, uint32_t box_inner,
                       uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn encode = GetEncodeTiled();
  if (encode == nullptr) throw Error(OV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    throw Error(OV_ERR_INVALID, "TMA base address must be 16-byte aligned");
  if (row_bytes % 16 != 0) throw Error(OV_ERR_INVALID, "TMA row stride must be 16-byte aligned");
  const cuuint64_t dims[2] = {inner, rows == 0 ? 1 : rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t elem_strides[2] = {1, 1};
  const CUresult r = encode(map, type, 2, const_cast<void*>(base), dims, strides, box,
                            elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw Error(OV_ERR_CUDA, "cuTensorMapEncodeTiled failed with " + std::to_string(r));
}

}  // namespace ovb

using ovb::AsStream;
using ovb::CudaFail;

extern "C" {

int ov_last_error(char* buffer, size_t capacity) {
  if (buffer != nullptr && capacity > 0) {
    const size_t n = std::min(capacity - 1, ovb::t_message.size());
    std::memcpy(buffer, ovb::t_message.data(), n);
    buffer[n] = '\0';
  }
  return ovb::t_status;
}

int ov_device_count(int* count) {
  const cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    return CudaFail(e, "cudaGetDeviceCount");
  }
  return OV_OK;
}

int ov_set_device(int device) {
  const cudaError_t e = cudaSetDevice(device);
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaSetDevice");
}

int ov_get_device(int* device) {
  const cudaError_t e = cudaGetDevice(device);
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaGetDevice");
}

int ov_device_info(int device, int* sm_count, int* major, int* minor) {
  cudaError_t e = cudaDeviceGetAttribute(sm_count, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(major, cudaDevAttrComputeCapabilityMajor, device);
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(minor, cudaDevAttrComputeCapabilityMinor, device);
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaDeviceGetAttribute");
}

int ov_malloc(void** pointer, size_t bytes) {
  const cudaError_t e = cudaMalloc(pointer, bytes == 0 ? 1 : bytes);
  if (e == cudaErrorMemoryAllocation) {
    (void)cudaGetLastError();
    return ovb::Fail(OV_ERR_OOM, "cudaMalloc of " + std::to_string(bytes) + " bytes");
  }
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaMalloc");
}

int ov_free(void* pointer) {
  if (pointer == nullptr) return OV_OK;
  const cudaError_t e = cudaFree(pointer);
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaFree");
}

int ov_malloc_host(void** pointer, size_t bytes) {
  const cudaError_t e = cudaMallocHost(pointer, bytes == 0 ? 1 : bytes);
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaMallocHost");
}

int ov_free_host(void* pointer) {
  if (pointer == nullptr) return OV_OK;
  const cudaError_t e = cudaFreeHost(pointer);
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaFreeHost");
}

int ov_memcpy_h2d_async(void* dst, const void* src, size_t bytes, ov_stream_t stream) {
  const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, AsStream(stream));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "host to device copy");
}

int ov_memcpy_d2h_async(void* dst, const void* src, size_t bytes, ov_stream_t stream) {
  const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, AsStream(stream));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "device to host copy");
}

int ov_memcpy_d2d_async(void* dst, const void* src, size_t bytes, ov_stream_t stream) {
  const cudaError_t e =
      cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, AsStream(stream));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "device to device copy");
}

int ov_memset_async(void* dst, int value, size_t bytes, ov_stream_t stream) {
  const cudaError_t e = cudaMemsetAsync(dst, value, bytes, AsStream(stream));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaMemsetAsync");
}

int ov_stream_create(ov_stream_t* stream) {
  cudaStream_t s = nullptr;
  const cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  *stream = s;
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaStreamCreate");
}

int ov_stream_destroy(ov_stream_t stream) {
  if (stream == nullptr) return OV_OK;
  const cudaError_t e = cudaStreamDestroy(AsStream(stream));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaStreamDestroy");
}

int ov_stream_sync(ov_stream_t stream) {
  const cudaError_t e = cudaStreamSynchronize(AsStream(stream));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaStreamSynchronize");
}

int ov_event_create(ov_event_t* event) {
  cudaEvent_t ev = nullptr;
  const cudaError_t e = cudaEventCreate(&ev);
  *event = ev;
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaEventCreate");
}

int ov_event_destroy(ov_event_t event) {
  if (event == nullptr) return OV_OK;
  const cudaError_t e = cudaEventDestroy(reinterpret_cast<cudaEvent_t>(event));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaEventDestroy");
}

int ov_event_record(ov_event_t event, ov_stream_t stream) {
  const cudaError_t e = cudaEventRecord(reinterpret_cast<cudaEvent_t>(event), AsStream(stream));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaEventRecord");
}

int ov_event_sync(ov_event_t event) {
  const cudaError_t e = cudaEventSynchronize(reinterpret_cast<cudaEvent_t>(event));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaEventSynchronize");
}

int ov_event_elapsed_ms(ov_event_t begin, ov_event_t end, float* milliseconds) {
  const cudaError_t e = cudaEventElapsedTime(milliseconds, reinterpret_cast<cudaEvent_t>(begin),
                                             reinterpret_cast<cudaEvent_t>(end));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaEventElapsedTime");
}

int ov_graph_capture_begin(ov_stream_t stream) {
  if (stream == nullptr) return ovb::Guard("ov_graph_capture_begin: ", [] {
      throw ovb::Error(OV_ERR_INVALID, "the legacy stream cannot be captured");
    });
  const cudaError_t e =
      cudaStreamBeginCapture(AsStream(stream), cudaStreamCaptureModeThreadLocal);
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaStreamBeginCapture");
}

int ov_graph_capture_end(ov_stream_t stream, ov_graph_t* graph) {
  *graph = nullptr;
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(AsStream(stream), &g);
  if (e != cudaSuccess) return CudaFail(e, "cudaStreamEndCapture");
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, g, 0);
  (void)cudaGraphDestroy(g);
  if (e != cudaSuccess) return CudaFail(e, "cudaGraphInstantiate");
  *graph = exec;
  return OV_OK;
}

int ov_graph_launch(ov_graph_t graph, ov_stream_t stream) {
  const cudaError_t e = cudaGraphLaunch(reinterpret_cast<cudaGraphExec_t>(graph), AsStream(stream));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaGraphLaunch");
}

int ov_graph_destroy(ov_graph_t graph) {
  if (graph == nullptr) return OV_OK;
  const cudaError_t e = cudaGraphExecDestroy(reinterpret_cast<cudaGraphExec_t>(graph));
  return e == cudaSuccess ? OV_OK : CudaFail(e, "cudaGraphExecDestroy");
}

int ov_take_device_errors(uint32_t* flags, ov_stream_t stream) {
  return ovb::Guard("", [&] {
    uint32_t* word = ovb::DeviceErrorWord();
    ovb::Check(cudaMemcpyAsync(flags, word, sizeof(uint32_t), cudaMemcpyDeviceToHost,
                               AsStream(stream)),
               "read device error word");
    ovb::Check(cudaMemsetAsync(word, 0, sizeof(uint32_t), AsStream(stream)),
               "clear device error word");
    // The allocation-free GEMM reports into its own static word.
    uint32_t noalloc = 0;
    uint32_t* status = ovb::NoAllocStatusWord();
    if (status != nullptr) {
      ovb::Check(cudaMemcpyAsync(&noalloc, status, sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                 AsStream(stream)),
                 "read allocation-free GEMM status word");
      ovb::Check(cudaMemsetAsync(status, 0, sizeof(uint32_t), AsStream(stream)),
                 "clear allocation-free GEMM status word");
    }
    ovb::Check(cudaStreamSynchronize(AsStream(stream)), "device error word");
    *flags |= noalloc;
  });
}

}  // extern "C"
