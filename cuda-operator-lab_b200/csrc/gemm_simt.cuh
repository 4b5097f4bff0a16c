// CUDA-core GEMM with the same fused epilogues as the tensor-core kernel.
//
// Serves the fp32-input entry points (gemm_swiglu v0..v3, gemm_bias_gelu
// v0..v6), whose reference arithmetic is full fp32 (cuBLAS SGEMM,
// gemm_swiglu.cu:165-190, gemm_bias_gelu.cu:889-903): products and sums stay
// in fp32 FMA.  It also serves bf16 shapes the TMA path cannot address (row
// strides that are not a multiple of 16 bytes, unaligned bases).
//
// 64x64 output tile per 256-thread CTA, 16-deep k slices staged through
// shared memory (transposed so each k step is two broadcast-free vector
// reads), 4x4 outputs per thread for each of the gate and up accumulators.
#pragma once

#include <cstdint>
#include <type_traits>

#include "common.cuh"
#include "gemm_sm100.cuh"  // Epilogue enum

namespace col {
namespace simt {

constexpr int kBM = 64;
constexpr int kBN = 64;
constexpr int kBK = 16;
constexpr int kThreads = 256;

struct SimtParams {
  const void* a;    // [M, K]
  const void* b0;   // gate / W rows [N, K]
  const void* b1;   // up rows [N, K] (SwiGLU only)
  const float* bias;
  const void* residual;  // kEpiResidual: bf16 [M, N]
  const float* row_scale;  // kEpiSwiGLURowScale: fp32 [M]
  void* out;        // [M, N]
  int m;
  int n;
  int k;
};

template <typename T>
__device__ __forceinline__ float load_elem(const T* p, std::size_t i) {
  if constexpr (std::is_same<T, float>::value) {
    return __ldg(p + i);
  } else {
    return __bfloat162float(p[i]);
  }
}

template <typename TIn, int EPI, typename TOut>
__global__ void __launch_bounds__(kThreads) simt_gemm_kernel(const SimtParams p) {
  grid_dependency_wait();
  constexpr bool kSwiGLU = (EPI == sm100::kEpiSwiGLU || EPI == sm100::kEpiSwiGLURoundBf16 ||
                           EPI == sm100::kEpiSwiGLURowScale);
  __shared__ float As[kBK][kBM + 4];
  __shared__ float Bs0[kBK][kBN + 4];
  __shared__ float Bs1[kSwiGLU ? kBK : 1][kSwiGLU ? kBN + 4 : 1];

  const TIn* __restrict__ A = static_cast<const TIn*>(p.a);
  const TIn* __restrict__ B0 = static_cast<const TIn*>(p.b0);
  const TIn* __restrict__ B1 = static_cast<const TIn*>(p.b1);
  const int m0 = blockIdx.y * kBM;
  const int n0 = blockIdx.x * kBN;
  const int tx = threadIdx.x % 16;
  const int ty = threadIdx.x / 16;

  float accg[4][4] = {};
  float accu[4][4] = {};

  for (int k0 = 0; k0 < p.k; k0 += kBK) {
    // Stage A[m0:m0+64, k0:k0+16] and B rows [n0:n0+64] transposed (k-major).
#pragma unroll
    for (int i = 0; i < (kBM * kBK) / kThreads; ++i) {
      const int e = threadIdx.x + i * kThreads;
      const int r = e / kBK;
      const int kk = e % kBK;
      const int gk = k0 + kk;
      const int gm = m0 + r;
      const int gn = n0 + r;
      As[kk][r] = (gm < p.m && gk < p.k) ? load_elem(A, static_cast<std::size_t>(gm) * p.k + gk) : 0.0f;
      Bs0[kk][r] = (gn < p.n && gk < p.k) ? load_elem(B0, static_cast<std::size_t>(gn) * p.k + gk) : 0.0f;
      if constexpr (kSwiGLU) {
        Bs1[kk][r] = (gn < p.n && gk < p.k) ? load_elem(B1, static_cast<std::size_t>(gn) * p.k + gk) : 0.0f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      float a[4], b[4], c[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs0[kk][tx * 4 + j];
      if constexpr (kSwiGLU) {
#pragma unroll
        for (int j = 0; j < 4; ++j) c[j] = Bs1[kk][tx * 4 + j];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          accg[i][j] = fmaf(a[i], b[j], accg[i][j]);
          if constexpr (kSwiGLU) accu[i][j] = fmaf(a[i], c[j], accu[i][j]);
        }
      }
    }
    __syncthreads();
  }

  TOut* __restrict__ out = static_cast<TOut*>(p.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= p.m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= p.n) continue;
      float o;
      if constexpr (EPI == sm100::kEpiSwiGLU) {
        o = silu_f(accg[i][j]) * accu[i][j];
      } else if constexpr (EPI == sm100::kEpiSwiGLURowScale) {
        const float rs = __ldg(p.row_scale + gm);
        o = silu_f(accg[i][j] * rs) * (accu[i][j] * rs);
      } else if constexpr (EPI == sm100::kEpiSwiGLURoundBf16) {
        o = silu_f(bf16_round(accg[i][j])) * bf16_round(accu[i][j]);
      } else if constexpr (EPI == sm100::kEpiResidual) {
        o = accg[i][j] + __bfloat162float(static_cast<const __nv_bfloat16*>(
                             p.residual)[static_cast<std::size_t>(gm) * p.n + gn]);
      } else if constexpr (EPI == sm100::kEpiBiasGeluErf) {
        o = gelu_erf_f(accg[i][j] + __ldg(p.bias + gn));
      } else {
        o = gelu_tanh_f(accg[i][j] + __ldg(p.bias + gn));
      }
      if constexpr (std::is_same<TOut, float>::value) {
        out[static_cast<std::size_t>(gm) * p.n + gn] = o;
      } else {
        out[static_cast<std::size_t>(gm) * p.n + gn] = __float2bfloat16_rn(o);
      }
    }
  }
}

template <typename TIn, int EPI, typename TOut>
inline int launch_simt(const SimtParams& p, cudaStream_t s) {
  const dim3 grid((p.n + kBN - 1) / kBN, (p.m + kBM - 1) / kBM);
  if (grid.y > 65535u) return static_cast<int>(cudaErrorInvalidValue);
  return launch_serialised(simt_gemm_kernel<TIn, EPI, TOut>, grid, dim3(kThreads), 0, s, p);
}

}  // namespace simt
}  // namespace col
