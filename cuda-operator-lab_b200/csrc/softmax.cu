// Row softmax entry points (softmax.cuh:5-47).
#include "rowwise.cuh"

namespace {

int softmax_f32(const float* x, float* y, std::uint64_t rows, std::uint64_t cols, void* stream) {
  if (rows == 0) return 0;
  if (x == nullptr || y == nullptr || !col::row_dims_ok(rows, cols)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  col::RowArgs a{x, nullptr, nullptr, nullptr, y, nullptr, rows, static_cast<std::uint32_t>(cols),
                 0.0f};
  return col::launch_rows<col::RowOp::kSoftmax, float, false>(a, col::as_stream(stream));
}

}  // namespace

#define COL_SOFTMAX(V)                                                                           \
  COL_API int cuda_operator_softmax_##V(const float* input, float* output, uint64_t rows,        \
                                        uint64_t cols, void* stream) {                           \
    return softmax_f32(input, output, rows, cols, stream);                                       \
  }
COL_SOFTMAX(v0)
COL_SOFTMAX(v1)
COL_SOFTMAX(v2)
COL_SOFTMAX(v3)
COL_SOFTMAX(v4)
COL_SOFTMAX(v5)
#undef COL_SOFTMAX
