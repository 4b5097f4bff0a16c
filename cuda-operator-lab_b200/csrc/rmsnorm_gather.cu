// Row-sharded bf16 RMSNorm whose output rows are stored into several buffers
// at once: this GPU's and, through CUDA IPC mappings over NVLink, the other
// ranks'.  It is the exchange step of the N-sharded Llama MLP block, where
// every rank's GEMM (an N slice) reads all M normalised rows: rank r
// normalises its M/g rows and its threads store each finished 16-byte vector
// into all g buffers, so the NVLink transfer is spread over the whole kernel
// and needs no second pass over the rows.  Each thread fences at system scope
// after its stores; a cuda_operator_lab_peer_barrier after the kernel on the
// same stream then tells every rank that the rows have landed.
//
// The arithmetic is that of cuda_operator_rmsnorm_bf16 for the same width:
// the same thread group per row (the width table of dispatch_row_width), the
// same per-thread sums in the same order and the same group reduction, so
// every destination receives bit for bit what cuda_operator_rmsnorm_bf16
// would write.  Vector path only: cols a multiple of 8 and at most 8192, all
// pointers 16-byte aligned.

#include <cstring>

#include "rowwise.cuh"

namespace {

constexpr int kMaxDests = 8;

struct NormDests {
  void* d[kMaxDests];
  int n;
};

struct GatherArgs {
  const void* x;
  const void* weight;
  NormDests dst;
  std::uint64_t rows;
  std::uint32_t cols;
  float eps;
};

template <int TPR, int NV>
__global__ void __launch_bounds__(TPR * col::rows_per_cta<TPR>())
rmsnorm_gather_kernel(const GatherArgs a) {
  constexpr int kVec = 8;
  constexpr int kRpc = col::rows_per_cta<TPR>();
  col::grid_dependency_wait();
  __shared__ float sh[kRpc * TPR / 32];

  const int t = threadIdx.x % TPR;
  const std::uint64_t row = static_cast<std::uint64_t>(blockIdx.x) * kRpc + threadIdx.x / TPR;
  const bool row_ok = row < a.rows;
  const std::uint32_t cols = a.cols;
  const std::uint64_t base = row * cols;
  const __nv_bfloat16* __restrict__ x = static_cast<const __nv_bfloat16*>(a.x) + base;
  const __nv_bfloat16* __restrict__ w = static_cast<const __nv_bfloat16*>(a.weight);

  float v[NV][kVec];
  bool ok[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const std::uint32_t idx = (static_cast<std::uint32_t>(j) * TPR + t) * kVec;
    ok[j] = row_ok && idx < cols;
    if (ok[j]) {
      col::load_vec<__nv_bfloat16, kVec>(x + idx, v[j]);
    } else {
#pragma unroll
      for (int e = 0; e < kVec; ++e) v[j][e] = 0.0f;
    }
  }
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int e = 0; e < kVec; ++e) s = fmaf(v[j][e], v[j][e], s);
  s = col::group_sum<TPR>(s, sh);
  const float rstd = rsqrtf(s * (1.0f / static_cast<float>(cols)) + a.eps);

  uint4 q[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if (ok[j]) {
      float wl[kVec], o[kVec];
      col::load_param<__nv_bfloat16, kVec>(w + (static_cast<std::uint32_t>(j) * TPR + t) * kVec,
                                           wl);
#pragma unroll
      for (int e = 0; e < kVec; ++e) o[e] = (v[j][e] * rstd) * wl[e];
      q[j] = col::pack_bf16x8(o);
    }
  }
  // One destination after the other: a warp's 16-byte stores to one buffer
  // are contiguous 512-byte runs.  The loop is unrolled over the maximum so
  // that every destination address is read from the parameter bank directly.
#pragma unroll
  for (int d = 0; d < kMaxDests; ++d) {
    if (d < a.dst.n) {
      __nv_bfloat16* __restrict__ y = static_cast<__nv_bfloat16*>(a.dst.d[d]) + base;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        if (ok[j]) {
          *reinterpret_cast<uint4*>(y + (static_cast<std::uint32_t>(j) * TPR + t) * kVec) = q[j];
        }
      }
    }
  }
  __threadfence_system();  // the peer barrier after this kernel publishes the rows
}

template <int TPR, int NV>
int launch_gather(const GatherArgs& a, cudaStream_t s) {
  constexpr int kRpc = col::rows_per_cta<TPR>();
  const std::uint64_t blocks = (a.rows + kRpc - 1) / kRpc;
  return col::launch_serialised(rmsnorm_gather_kernel<TPR, NV>,
                                dim3(static_cast<unsigned>(blocks)), dim3(TPR * kRpc), 0, s, a);
}

// The thread group per row of dispatch_row_width (rowwise.cuh), vector units
// of 8 bf16, so that the sums match cuda_operator_rmsnorm_bf16 exactly.
int dispatch_gather(std::uint32_t units, const GatherArgs& a, cudaStream_t s) {
  if (units <= 32) return launch_gather<32, 1>(a, s);
  if (units <= 64) return launch_gather<32, 2>(a, s);
  if (units <= 128) return launch_gather<32, 4>(a, s);
  if (units <= 256) return launch_gather<64, 4>(a, s);
  if (units <= 512) return launch_gather<128, 4>(a, s);
  return launch_gather<256, 4>(a, s);  // units <= 1024 (cols <= 8192)
}

}  // namespace

COL_API int cuda_operator_rmsnorm_allgather_bf16(const void* input_bf16, const void* weight_bf16,
                                                 void* const* dests, int num_dests, uint64_t rows,
                                                 uint64_t cols, float eps, void* stream) {
  if (rows == 0) return 0;
  if (input_bf16 == nullptr || weight_bf16 == nullptr || dests == nullptr || num_dests < 1 ||
      num_dests > kMaxDests || !col::row_dims_ok(rows, cols) || cols % 8 != 0 || cols > 8192 ||
      !(eps > 0.0f) || !col::aligned16(input_bf16) || !col::aligned16(weight_bf16)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  GatherArgs a;
  std::memset(&a, 0, sizeof(a));
  a.x = input_bf16;
  a.weight = weight_bf16;
  a.rows = rows;
  a.cols = static_cast<std::uint32_t>(cols);
  a.eps = eps;
  a.dst.n = num_dests;
  for (int i = 0; i < num_dests; ++i) {
    if (dests[i] == nullptr || !col::aligned16(dests[i])) {
      return static_cast<int>(cudaErrorInvalidValue);
    }
    a.dst.d[i] = dests[i];
  }
  return dispatch_gather(a.cols / 8, a, col::as_stream(stream));
}
