// gufo::models::omnivoice::HalfGemm on the B200 C-ABI (reference:
// gemm.hpp:41-62, gemm.cpp:80-288).  Linear takes the tcgen05 GEMM when
// its layout rules hold (K a multiple of 64, 16-byte aligned rows) and
// ov_matmul_f16 otherwise; both accumulate in float32.
#include "gemm.hpp"

#include <cstdint>
#include <stdexcept>
#include <string>

#include "ov_kernels.h"

namespace gufo::models::omnivoice {
namespace {

void Throw(const char* what) {
  char buffer[2048];
  ov_last_error(buffer, sizeof(buffer));
  throw std::runtime_error(std::string(what) + buffer);
}

bool Aligned(const void* p, std::size_t bytes) {
  return reinterpret_cast<std::uintptr_t>(p) % bytes == 0;
}

}  // namespace

struct HalfGemm::State {
  ov_stream_t stream = nullptr;
  void* workspace = nullptr;  // split-K counters or partials, grow-only, zeroed
  std::size_t workspace_bytes = 0;
  ~State() {
    if (workspace != nullptr) ov_free(workspace);
  }
};

HalfGemm::HalfGemm(void* /*fallback*/, ov_stream_t stream) : state_(std::make_unique<State>()) {
  state_->stream = stream;
}

HalfGemm::~HalfGemm() = default;

void HalfGemm::Linear(const void* x, const void* w, float* y, std::size_t rows, std::size_t in,
                      std::size_t out, bool accumulate) {
  if (rows == 0 || out == 0) return;
  const int epilogue = accumulate ? OV_EPI_ACCUM_F32 : OV_EPI_STORE_F32;
  const bool tiled = in > 0 && in % 64 == 0 && out % 4 == 0 && Aligned(x, 16) && Aligned(w, 16) &&
                     Aligned(y, 16);
  if (tiled) {
    const std::size_t need = ov_gemm_workspace_bytes(rows, in, out, epilogue);
    if (need > state_->workspace_bytes) {
      if (state_->workspace != nullptr) ov_free(state_->workspace);
      state_->workspace = nullptr;
      state_->workspace_bytes = 0;
      if (ov_malloc(&state_->workspace, need) != OV_OK) Throw("HalfGemm: ");
      if (ov_memset_async(state_->workspace, 0, need, state_->stream) != OV_OK)
        Throw("HalfGemm: ");
      state_->workspace_bytes = need;
    }
    if (ov_gemm_f16(static_cast<const std::uint16_t*>(x), in, static_cast<const std::uint16_t*>(w),
                    y, out, rows, in, out, epilogue, nullptr, state_->workspace,
                    state_->workspace_bytes, state_->stream) != OV_OK)
      Throw("HalfGemm::Linear: ");
    return;
  }
  // Column-major view: C[out][rows] = W^T-stored A (k x m, transposed) * X.
  MatmulShape s;
  s.transpose_a = true;
  s.m = out;
  s.n = rows;
  s.k = in;
  s.lda = in;
  s.ldb = in;
  s.ldc = out;
  s.accumulate = accumulate;
  Matmul(s, s, w, x, y);
}

void HalfGemm::Matmul(const MatmulShape& shape, const MatmulShape& /*representative*/,
                      const void* a, const void* b, float* c) {
  ov_matmul_shape s;
  s.transpose_a = shape.transpose_a ? 1 : 0;
  s.transpose_b = shape.transpose_b ? 1 : 0;
  s.m = shape.m;
  s.n = shape.n;
  s.k = shape.k;
  s.lda = shape.lda;
  s.ldb = shape.ldb;
  s.ldc = shape.ldc;
  s.stride_a = shape.stride_a;
  s.stride_b = shape.stride_b;
  s.stride_c = shape.stride_c;
  s.batch = shape.batch;
  s.accumulate = shape.accumulate ? 1 : 0;
  if (ov_matmul_f16(&s, static_cast<const std::uint16_t*>(a), static_cast<const std::uint16_t*>(b),
                    c, state_->stream) != OV_OK)
    Throw("HalfGemm::Matmul: ");
}

}  // namespace gufo::models::omnivoice
