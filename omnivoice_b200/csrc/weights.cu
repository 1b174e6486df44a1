// Weight preparation on the device: float32 -> float16 conversion of the
// linear weights with the gate/up interleave the fused SwiGLU epilogue
// reads, and the synthetic checkpoint fill.  The reference converts and
// stacks on the host (generator.cpp:31-49, 324-352); doing it here keeps
// loading a 0.9 GB replica to tens of milliseconds.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include "internal.hpp"
#include "launch.hpp"
#include "synthetic.hpp"

namespace ovb {
namespace {

__global__ void to_half_rows_kernel(const float* __restrict__ src, __half* __restrict__ out,
                                    int64_t rows, int64_t cols, int group, int offset) {
  const int64_t total = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t j = i / cols;
    const int64_t k = i % cols;
    const int64_t dst = group > 0 ? (j / group) * 2 * group + offset + j % group : j;
    out[dst * cols + k] = __float2half_rn(src[i]);
  }
}

__global__ void synthetic_fill_kernel(float* __restrict__ out, int64_t count, uint64_t base,
                                      float scale) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = SyntheticValue(base, static_cast<uint64_t>(i), scale);
}

__global__ void fill_kernel(float* __restrict__ out, int64_t count, float value) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = value;
}

__global__ void fill_int_kernel(int32_t* __restrict__ out, int64_t count, int32_t value) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = value;
}

int GridFor(int64_t count) {
  return static_cast<int>(std::min<int64_t>((count + 255) / 256, 148 * 64));
}

std::mutex g_smem_mutex;
std::set<std::pair<const void*, int>> g_smem_done;

}  // namespace

void LaunchToHalfRows(const float* src, uint16_t* out, int64_t rows, int64_t cols, int group,
                      int offset, cudaStream_t stream) {
  if (rows * cols == 0) return;
  to_half_rows_kernel<<<GridFor(rows * cols), 256, 0, stream>>>(
      src, reinterpret_cast<__half*>(out), rows, cols, group, offset);
  Check(cudaGetLastError(), "weight conversion launch");
}

void LaunchSyntheticFill(float* out, size_t count, uint64_t seed, uint64_t tensor, float std,
                         cudaStream_t stream) {
  if (count == 0) return;
  synthetic_fill_kernel<<<GridFor(static_cast<int64_t>(count)), 256, 0, stream>>>(
      out, static_cast<int64_t>(count), SyntheticBase(seed, tensor), SyntheticScale(std));
  Check(cudaGetLastError(), "synthetic fill launch");
}

void LaunchFill(float* out, size_t count, float value, cudaStream_t stream) {
  if (count == 0) return;
  fill_kernel<<<GridFor(static_cast<int64_t>(count)), 256, 0, stream>>>(
      out, static_cast<int64_t>(count), value);
  Check(cudaGetLastError(), "fill launch");
}

void LaunchFillInt(int32_t* out, size_t count, int32_t value, cudaStream_t stream) {
  if (count == 0) return;
  fill_int_kernel<<<GridFor(static_cast<int64_t>(count)), 256, 0, stream>>>(
      out, static_cast<int64_t>(count), value);
  Check(cudaGetLastError(), "fill launch");
}

namespace {
thread_local bool t_pdl = false;
}  // namespace

bool PdlEnabled() { return t_pdl; }
PdlScope::PdlScope(bool on) : previous_(t_pdl) { t_pdl = on; }
PdlScope::~PdlScope() { t_pdl = previous_; }

void SetMaxDynamicSmem(const void* func, int bytes) {
  int device = 0;
  Check(cudaGetDevice(&device), "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_smem_mutex);
  if (g_smem_done.count({func, device}) != 0) return;
  Check(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
        "cudaFuncSetAttribute(max dynamic shared memory)");
  g_smem_done.insert({func, device});
}

}  // namespace ovb
