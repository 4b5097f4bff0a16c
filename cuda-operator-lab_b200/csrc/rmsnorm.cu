// RMSNorm entry points: the reference's fp32 v0..v4 (rmsnorm.cuh:5-47) and
// the bf16 variant of the Llama MLP workload.
#include "rowwise.cuh"

namespace {

int rmsnorm_f32(const float* x, const float* w, float* y, std::uint64_t rows,
                std::uint64_t cols, float eps, void* stream) {
  if (rows == 0) return 0;
  if (x == nullptr || w == nullptr || y == nullptr || !col::row_dims_ok(rows, cols)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (!(eps > 0.0f)) return static_cast<int>(cudaErrorInvalidValue);
  col::RowArgs a{x, nullptr, w, nullptr, y, nullptr, rows, static_cast<std::uint32_t>(cols), eps};
  return col::launch_rows<col::RowOp::kRms, float, false>(a, col::as_stream(stream));
}

}  // namespace

COL_API int cuda_operator_rmsnorm_v0(const float* input, const float* weight, float* output,
                                     uint64_t rows, uint64_t cols, float eps, void* stream) {
  return rmsnorm_f32(input, weight, output, rows, cols, eps, stream);
}
COL_API int cuda_operator_rmsnorm_v1(const float* input, const float* weight, float* output,
                                     uint64_t rows, uint64_t cols, float eps, void* stream) {
  return rmsnorm_f32(input, weight, output, rows, cols, eps, stream);
}
COL_API int cuda_operator_rmsnorm_v2(const float* input, const float* weight, float* output,
                                     uint64_t rows, uint64_t cols, float eps, void* stream) {
  return rmsnorm_f32(input, weight, output, rows, cols, eps, stream);
}
COL_API int cuda_operator_rmsnorm_v3(const float* input, const float* weight, float* output,
                                     uint64_t rows, uint64_t cols, float eps, void* stream) {
  return rmsnorm_f32(input, weight, output, rows, cols, eps, stream);
}
COL_API int cuda_operator_rmsnorm_v4(const float* input, const float* weight, float* output,
                                     uint64_t rows, uint64_t cols, float eps, void* stream) {
  return rmsnorm_f32(input, weight, output, rows, cols, eps, stream);
}

COL_API int cuda_operator_rmsnorm_bf16(const void* input_bf16, const void* weight_bf16,
                                       void* output_bf16, uint64_t rows, uint64_t cols, float eps,
                                       void* stream) {
  if (rows == 0) return 0;
  if (input_bf16 == nullptr || weight_bf16 == nullptr || output_bf16 == nullptr ||
      !col::row_dims_ok(rows, cols)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (!(eps > 0.0f)) return static_cast<int>(cudaErrorInvalidValue);
  col::RowArgs a{input_bf16, nullptr, weight_bf16, nullptr, output_bf16, nullptr, rows,
                 static_cast<std::uint32_t>(cols), eps};
  return col::launch_rows<col::RowOp::kRms, __nv_bfloat16, false>(a, col::as_stream(stream));
}

// Residual add + RMSNorm in one pass (no reference counterpart; the decode /
// prefill norm that feeds the MLP GEMM): h = input + residual is stored and
// y = rmsnorm(h) * weight, each input read once.  bf16: h is rounded to bf16
// before the statistics, exactly as a separate add kernel would leave it.
// Same argument rules as the RMSNorm entries (rows == 0 succeeds first).
namespace {

template <typename T>
int residual_rmsnorm(const void* x, const void* r, const void* w, void* h, void* y,
                     std::uint64_t rows, std::uint64_t cols, float eps, void* stream) {
  if (rows == 0) return 0;
  if (x == nullptr || r == nullptr || w == nullptr || h == nullptr || y == nullptr ||
      !col::row_dims_ok(rows, cols)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (!(eps > 0.0f)) return static_cast<int>(cudaErrorInvalidValue);
  col::RowArgs a{x, r, w, nullptr, y, h, rows, static_cast<std::uint32_t>(cols), eps};
  return col::launch_rows<col::RowOp::kResidualRms, T, true>(a, col::as_stream(stream));
}

}  // namespace

COL_API int cuda_operator_fused_residual_rmsnorm_bf16(const void* input_bf16,
                                                      const void* residual_bf16,
                                                      const void* weight_bf16, void* h_out_bf16,
                                                      void* output_bf16, uint64_t rows,
                                                      uint64_t cols, float eps, void* stream) {
  return residual_rmsnorm<__nv_bfloat16>(input_bf16, residual_bf16, weight_bf16, h_out_bf16,
                                         output_bf16, rows, cols, eps, stream);
}

COL_API int cuda_operator_fused_residual_rmsnorm_h(const float* input, const float* residual,
                                                   const float* weight, float* h_out,
                                                   float* output, uint64_t rows, uint64_t cols,
                                                   float eps, void* stream) {
  return residual_rmsnorm<float>(input, residual, weight, h_out, output, rows, cols, eps, stream);
}

// Per-row inverse RMS of a bf16 matrix, rstd[row] = rsqrt(mean(x[row]^2) + eps)
// in fp32 (no reference counterpart): the statistics half of RMSNorm, for
// cuda_operator_gemm_swiglu_rowscale_bf16, which applies it in the GEMM's
// epilogue.  Reads x once, writes 4 bytes per row.
COL_API int cuda_operator_rmsnorm_rstd_bf16(const void* input_bf16, float* rstd, uint64_t rows,
                                            uint64_t cols, float eps, void* stream) {
  if (rows == 0) return 0;
  if (input_bf16 == nullptr || rstd == nullptr || !col::row_dims_ok(rows, cols)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (!(eps > 0.0f)) return static_cast<int>(cudaErrorInvalidValue);
  col::RowArgs a{input_bf16, nullptr, nullptr, nullptr, rstd, nullptr, rows,
                 static_cast<std::uint32_t>(cols), eps};
  return col::launch_rows<col::RowOp::kRmsRstd, __nv_bfloat16, false>(a, col::as_stream(stream));
}
