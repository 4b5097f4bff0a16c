// LayerNorm and residual+LayerNorm entry points (layernorm.cuh:5-68,
// fused_residual_layernorm.cuh:5-62) plus the variant that also stores h.
#include "rowwise.cuh"

namespace {

int layernorm_f32(const float* x, const float* w, const float* b, float* y, std::uint64_t rows,
                  std::uint64_t cols, float eps, void* stream) {
  if (rows == 0) return 0;
  if (x == nullptr || w == nullptr || b == nullptr || y == nullptr ||
      !col::row_dims_ok(rows, cols)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (!(eps > 0.0f)) return static_cast<int>(cudaErrorInvalidValue);
  col::RowArgs a{x, nullptr, w, b, y, nullptr, rows, static_cast<std::uint32_t>(cols), eps};
  return col::launch_rows<col::RowOp::kLayerNorm, float, false>(a, col::as_stream(stream));
}

int residual_layernorm_f32(const float* x, const float* r, const float* w, const float* b,
                           float* h, float* y, std::uint64_t rows, std::uint64_t cols, float eps,
                           void* stream, bool store_h) {
  if (rows == 0) return 0;
  if (x == nullptr || r == nullptr || w == nullptr || b == nullptr || y == nullptr ||
      (store_h && h == nullptr) || !col::row_dims_ok(rows, cols)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (!(eps > 0.0f)) return static_cast<int>(cudaErrorInvalidValue);
  col::RowArgs a{x, r, w, b, y, h, rows, static_cast<std::uint32_t>(cols), eps};
  if (store_h) {
    return col::launch_rows<col::RowOp::kResidualLayerNorm, float, true>(a, col::as_stream(stream));
  }
  return col::launch_rows<col::RowOp::kResidualLayerNorm, float, false>(a, col::as_stream(stream));
}

}  // namespace

#define COL_LAYERNORM(V)                                                                         \
  COL_API int cuda_operator_layernorm_##V(const float* input, const float* weight,               \
                                          const float* bias, float* output, uint64_t rows,       \
                                          uint64_t cols, float eps, void* stream) {              \
    return layernorm_f32(input, weight, bias, output, rows, cols, eps, stream);                  \
  }
COL_LAYERNORM(v0)
COL_LAYERNORM(v1)
COL_LAYERNORM(v2)
COL_LAYERNORM(v3)
COL_LAYERNORM(v4)
COL_LAYERNORM(v5)
#undef COL_LAYERNORM

#define COL_RESIDUAL_LAYERNORM(V)                                                                \
  COL_API int cuda_operator_fused_residual_layernorm_##V(                                        \
      const float* input, const float* residual, const float* weight, const float* bias,         \
      float* output, uint64_t rows, uint64_t cols, float eps, void* stream) {                    \
    return residual_layernorm_f32(input, residual, weight, bias, nullptr, output, rows, cols,    \
                                  eps, stream, false);                                           \
  }
COL_RESIDUAL_LAYERNORM(v0)
COL_RESIDUAL_LAYERNORM(v1)
COL_RESIDUAL_LAYERNORM(v2)
COL_RESIDUAL_LAYERNORM(v3)
COL_RESIDUAL_LAYERNORM(v4)
#undef COL_RESIDUAL_LAYERNORM

COL_API int cuda_operator_fused_residual_layernorm_h(const float* input, const float* residual,
                                                     const float* weight, const float* bias,
                                                     float* h_output, float* output,
                                                     uint64_t rows, uint64_t cols, float eps,
                                                     void* stream) {
  return residual_layernorm_f32(input, residual, weight, bias, h_output, output, rows, cols, eps,
                                stream, true);
}
