// Row engine shared by RMSNorm, LayerNorm, residual+LayerNorm, residual+RMSNorm
// and softmax.
//
// One group of TPR threads owns one row.  Each thread loads NV vectors of VEC
// elements (16-byte vectors when the row width and all pointers allow it,
// scalars otherwise) into registers with one HBM read, the group reduces its
// statistics with warp shuffles (plus a shared-memory step when the group
// spans several warps), and the thread writes its outputs from the same
// registers: every input byte is read once and every output byte written
// once.  Rows wider than TPR*NV*VEC use a streaming kernel that re-reads the
// row (from L2) once per statistic.
#pragma once

#include <cmath>
#include <cstdint>
#include <type_traits>

#include "common.cuh"

namespace col {

enum class RowOp : int {
  kRms = 0,
  kLayerNorm = 1,
  kResidualLayerNorm = 2,
  kSoftmax = 3,
  kResidualRms = 4,
  kRmsRstd = 5,  // only rsqrt(mean(x^2) + eps) per row, as fp32 into y[row]
};

// Ops that normalise h = x + residual (and may store h).
constexpr bool has_residual(RowOp op) {
  return op == RowOp::kResidualLayerNorm || op == RowOp::kResidualRms;
}

struct RowArgs {
  const void* x;
  const void* residual;  // residual ops only
  const void* weight;    // RMSNorm weight / LayerNorm gamma
  const void* bias;      // LayerNorm beta
  void* y;
  void* h;  // x + residual, stored when the kernel is instantiated with STORE_H
  std::uint64_t rows;
  std::uint32_t cols;
  float eps;
};

// ------------------------------------------------------------ vector access
//
// Row data use plain (L2-allocating) loads and stores: a norm's input usually
// comes from the kernel before it and its output feeds the next one, so both
// are worth keeping in the 126 MB L2 (streaming hints would evict them).

template <typename T, int VEC>
__device__ __forceinline__ void load_vec(const T* p, float (&v)[VEC]) {
  if constexpr (std::is_same<T, float>::value && VEC == 4) {
    const float4 q = *reinterpret_cast<const float4*>(p);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value && VEC == 8) {
    unpack_bf16x8(*reinterpret_cast<const uint4*>(p), v);
  } else if constexpr (std::is_same<T, float>::value && VEC == 1) {
    v[0] = *p;
  } else {
    static_assert(std::is_same<T, __nv_bfloat16>::value && VEC == 1, "unsupported vector");
    v[0] = __bfloat162float(p[0]);
  }
}

// Parameters (weights, biases) are re-read by every row: keep them cached.
template <typename T, int VEC>
__device__ __forceinline__ void load_param(const T* p, float (&v)[VEC]) {
  if constexpr (std::is_same<T, float>::value && VEC == 4) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value && VEC == 8) {
    unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(p)), v);
  } else if constexpr (std::is_same<T, float>::value && VEC == 1) {
    v[0] = __ldg(p);
  } else {
    v[0] = __bfloat162float(p[0]);
  }
}

template <typename T>
__device__ __forceinline__ float load_param1(const T* p) {
  if constexpr (std::is_same<T, float>::value) return __ldg(p);
  else return __bfloat162float(p[0]);
}

template <typename T, int VEC>
__device__ __forceinline__ void store_vec(T* p, const float (&v)[VEC]) {
  if constexpr (std::is_same<T, float>::value && VEC == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value && VEC == 8) {
    *reinterpret_cast<uint4*>(p) = pack_bf16x8(v);
  } else if constexpr (std::is_same<T, float>::value && VEC == 1) {
    p[0] = v[0];
  } else {
    p[0] = __float2bfloat16_rn(v[0]);
  }
}

// ------------------------------------------------------------ group reductions

// Sum/max over the TPR threads that own one row.  Every thread of the CTA
// must call these the same number of times (they contain __syncthreads when
// a row spans several warps).  The cross-warp step adds the per-warp values
// in a fixed order, so results do not depend on scheduling.
template <int TPR>
__device__ __forceinline__ float group_sum(float v, float* sh) {
  v = warp_sum(v);
  if constexpr (TPR == 32) {
    return v;
  } else {
    constexpr int kWarpsPerRow = TPR / 32;
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) sh[warp] = v;
    __syncthreads();
    const int first = (warp / kWarpsPerRow) * kWarpsPerRow;
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kWarpsPerRow; ++i) s += sh[first + i];
    __syncthreads();
    return s;
  }
}

template <int TPR>
__device__ __forceinline__ float group_max(float v, float* sh) {
  v = warp_max(v);
  if constexpr (TPR == 32) {
    return v;
  } else {
    constexpr int kWarpsPerRow = TPR / 32;
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) sh[warp] = v;
    __syncthreads();
    const int first = (warp / kWarpsPerRow) * kWarpsPerRow;
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kWarpsPerRow; ++i) m = fmaxf(m, sh[first + i]);
    __syncthreads();
    return m;
  }
}

template <int TPR>
__host__ __device__ constexpr int rows_per_cta() { return TPR >= 128 ? 1 : 128 / TPR; }

// ------------------------------------------------------------ register kernel

template <RowOp OP, typename T, int VEC, int TPR, int NV, bool STORE_H>
__global__ void __launch_bounds__(TPR * rows_per_cta<TPR>())
row_kernel(const RowArgs a) {
  constexpr int kRpc = rows_per_cta<TPR>();
  grid_dependency_wait();
  __shared__ float sh[kRpc * TPR / 32];

  const int t = threadIdx.x % TPR;
  const std::uint64_t row = static_cast<std::uint64_t>(blockIdx.x) * kRpc + threadIdx.x / TPR;
  const bool row_ok = row < a.rows;
  const std::uint32_t cols = a.cols;
  const std::uint64_t base = row * cols;

  const T* __restrict__ x = static_cast<const T*>(a.x) + base;
  float v[NV][VEC];
  bool ok[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const std::uint32_t idx = (static_cast<std::uint32_t>(j) * TPR + t) * VEC;
    ok[j] = row_ok && idx < cols;
    if (ok[j]) {
      load_vec<T, VEC>(x + idx, v[j]);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) v[j][e] = 0.0f;
    }
  }
  if constexpr (has_residual(OP)) {
    // h = x + residual in T: for bf16, h is rounded to bf16 before the
    // statistics, as a separate add kernel writing h would leave it.
    const T* __restrict__ r = static_cast<const T*>(a.residual) + base;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (ok[j]) {
        float rv[VEC];
        load_vec<T, VEC>(r + (static_cast<std::uint32_t>(j) * TPR + t) * VEC, rv);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          v[j][e] += rv[e];
          if constexpr (!std::is_same<T, float>::value) v[j][e] = bf16_round(v[j][e]);
        }
      }
    }
    if constexpr (STORE_H) {
      T* __restrict__ h = static_cast<T*>(a.h) + base;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        if (ok[j]) store_vec<T, VEC>(h + (static_cast<std::uint32_t>(j) * TPR + t) * VEC, v[j]);
      }
    }
  }

  T* __restrict__ y = static_cast<T*>(a.y) + base;
  const float inv_cols = 1.0f / static_cast<float>(cols);

  if constexpr (OP == RowOp::kRmsRstd) {
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int e = 0; e < VEC; ++e) s = fmaf(v[j][e], v[j][e], s);
    s = group_sum<TPR>(s, sh);
    if (row_ok && t == 0) static_cast<float*>(a.y)[row] = rsqrtf(s * inv_cols + a.eps);
  } else if constexpr (OP == RowOp::kRms || OP == RowOp::kResidualRms) {
    // Weights are loaded before the reduction so their latency overlaps it
    // (when the registers allow: up to 16 elements per thread).
    constexpr bool kEarly = NV * VEC <= 16;
    const T* __restrict__ w = static_cast<const T*>(a.weight);
    float wv[kEarly ? NV : 1][VEC];
    if constexpr (kEarly) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        if (ok[j]) load_param<T, VEC>(w + (static_cast<std::uint32_t>(j) * TPR + t) * VEC, wv[j]);
      }
    }
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int e = 0; e < VEC; ++e) s = fmaf(v[j][e], v[j][e], s);
    s = group_sum<TPR>(s, sh);
    const float rstd = rsqrtf(s * inv_cols + a.eps);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (ok[j]) {
        const std::uint32_t idx = (static_cast<std::uint32_t>(j) * TPR + t) * VEC;
        float o[VEC];
        if constexpr (kEarly) {
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[e] = (v[j][e] * rstd) * wv[j][e];
        } else {
          float wl[VEC];
          load_param<T, VEC>(w + idx, wl);
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[e] = (v[j][e] * rstd) * wl[e];
        }
        store_vec<T, VEC>(y + idx, o);
      }
    }
  } else if constexpr (OP == RowOp::kLayerNorm || OP == RowOp::kResidualLayerNorm) {
    // gamma/beta are loaded before the reductions so their latency overlaps
    // them (when the registers allow: up to 16 elements per thread).
    constexpr bool kEarly = NV * VEC <= 16;
    const T* __restrict__ g = static_cast<const T*>(a.weight);
    const T* __restrict__ b = static_cast<const T*>(a.bias);
    float gv[kEarly ? NV : 1][VEC], bv[kEarly ? NV : 1][VEC];
    if constexpr (kEarly) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        if (ok[j]) {
          const std::uint32_t idx = (static_cast<std::uint32_t>(j) * TPR + t) * VEC;
          load_param<T, VEC>(g + idx, gv[j]);
          load_param<T, VEC>(b + idx, bv[j]);
        }
      }
    }
    // Shifted sum: subtracting the row's first element (the same value in
    // every thread of the row) keeps the partial sums small when the row
    // carries a large common offset, so the mean keeps its low-order bits.
    float shift = 0.0f;
    if (row_ok) {
      shift = load_param1(static_cast<const T*>(a.x) + base);
      if constexpr (OP == RowOp::kResidualLayerNorm) {
        shift += load_param1(static_cast<const T*>(a.residual) + base);
      }
    }
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (ok[j]) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) s += v[j][e] - shift;
      }
    }
    const float mean = shift + group_sum<TPR>(s, sh) * inv_cols;
    float q = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (ok[j]) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float d = v[j][e] - mean;
          q = fmaf(d, d, q);
        }
      }
    }
    const float var = group_sum<TPR>(q, sh) * inv_cols;
    const float rstd = rsqrtf(var + a.eps);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (ok[j]) {
        const std::uint32_t idx = (static_cast<std::uint32_t>(j) * TPR + t) * VEC;
        float o[VEC];
        if constexpr (kEarly) {
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[e] = fmaf((v[j][e] - mean) * rstd, gv[j][e], bv[j][e]);
        } else {
          float gl[VEC], bl[VEC];
          load_param<T, VEC>(g + idx, gl);
          load_param<T, VEC>(b + idx, bl);
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[e] = fmaf((v[j][e] - mean) * rstd, gl[e], bl[e]);
        }
        store_vec<T, VEC>(y + idx, o);
      }
    }
  } else {  // softmax
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (ok[j]) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) m = fmaxf(m, v[j][e]);
      }
    }
    m = group_max<TPR>(m, sh);
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        v[j][e] = ok[j] ? expf(v[j][e] - m) : 0.0f;
        s += v[j][e];
      }
    }
    s = group_sum<TPR>(s, sh);
    const float inv = 1.0f / s;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (ok[j]) {
        float o[VEC];
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[e] = v[j][e] * inv;
        store_vec<T, VEC>(y + (static_cast<std::uint32_t>(j) * TPR + t) * VEC, o);
      }
    }
  }
}

// ------------------------------------------------------------ streaming kernel

constexpr int kLongThreads = 1024;

__device__ __forceinline__ float block_sum_long(float v, float* sh) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < kLongThreads / 32; ++i) s += sh[i];
  __syncthreads();
  return s;
}

__device__ __forceinline__ float block_max_long(float v, float* sh) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kLongThreads / 32; ++i) m = fmaxf(m, sh[i]);
  __syncthreads();
  return m;
}

template <typename T>
__device__ __forceinline__ float ld1(const T* p) {
  if constexpr (std::is_same<T, float>::value) return p[0];
  else return __bfloat162float(p[0]);
}
template <typename T>
__device__ __forceinline__ void st1(T* p, float v) {
  if constexpr (std::is_same<T, float>::value) p[0] = v;
  else p[0] = __float2bfloat16_rn(v);
}

// One CTA per row, rows of any width; the row is re-read once per pass.
template <RowOp OP, typename T, bool STORE_H>
__global__ void __launch_bounds__(kLongThreads) row_kernel_long(const RowArgs a) {
  grid_dependency_wait();
  __shared__ float sh[kLongThreads / 32];
  const std::uint64_t row = blockIdx.x;
  const std::uint32_t cols = a.cols;
  const std::uint64_t base = row * cols;
  const T* __restrict__ x = static_cast<const T*>(a.x) + base;
  const T* __restrict__ r = static_cast<const T*>(a.residual) + base;
  T* __restrict__ y = static_cast<T*>(a.y) + base;
  const T* __restrict__ w = static_cast<const T*>(a.weight);
  const T* __restrict__ b = static_cast<const T*>(a.bias);
  const float inv_cols = 1.0f / static_cast<float>(cols);

  auto in = [&](std::uint32_t i) -> float {
    if constexpr (has_residual(OP)) {
      const float hv = ld1(x + i) + ld1(r + i);
      if constexpr (std::is_same<T, float>::value) return hv;
      else return bf16_round(hv);
    } else {
      return ld1(x + i);
    }
  };

  if constexpr (OP == RowOp::kRmsRstd) {
    float s = 0.0f;
    for (std::uint32_t i = threadIdx.x; i < cols; i += kLongThreads) {
      const float v = in(i);
      s = fmaf(v, v, s);
    }
    const float rstd = rsqrtf(block_sum_long(s, sh) * inv_cols + a.eps);
    if (threadIdx.x == 0) static_cast<float*>(a.y)[row] = rstd;
  } else if constexpr (OP == RowOp::kRms || OP == RowOp::kResidualRms) {
    float s = 0.0f;
    for (std::uint32_t i = threadIdx.x; i < cols; i += kLongThreads) {
      const float v = in(i);
      s = fmaf(v, v, s);
    }
    const float rstd = rsqrtf(block_sum_long(s, sh) * inv_cols + a.eps);
    for (std::uint32_t i = threadIdx.x; i < cols; i += kLongThreads) {
      const float hv = in(i);
      if constexpr (STORE_H && OP == RowOp::kResidualRms) st1(static_cast<T*>(a.h) + base + i, hv);
      st1(y + i, (hv * rstd) * ld1(w + i));
    }
  } else if constexpr (OP == RowOp::kLayerNorm || OP == RowOp::kResidualLayerNorm) {
    const float shift = in(0);  // shifted sum, as in row_kernel
    float s = 0.0f;
    for (std::uint32_t i = threadIdx.x; i < cols; i += kLongThreads) s += in(i) - shift;
    const float mean = shift + block_sum_long(s, sh) * inv_cols;
    float q = 0.0f;
    for (std::uint32_t i = threadIdx.x; i < cols; i += kLongThreads) {
      const float d = in(i) - mean;
      q = fmaf(d, d, q);
    }
    const float rstd = rsqrtf(block_sum_long(q, sh) * inv_cols + a.eps);
    for (std::uint32_t i = threadIdx.x; i < cols; i += kLongThreads) {
      const float hv = in(i);
      if constexpr (STORE_H) st1(static_cast<T*>(a.h) + base + i, hv);
      st1(y + i, fmaf((hv - mean) * rstd, ld1(w + i), ld1(b + i)));
    }
  } else {
    float m = -INFINITY;
    for (std::uint32_t i = threadIdx.x; i < cols; i += kLongThreads) m = fmaxf(m, in(i));
    m = block_max_long(m, sh);
    float s = 0.0f;
    for (std::uint32_t i = threadIdx.x; i < cols; i += kLongThreads) s += expf(in(i) - m);
    const float inv = 1.0f / block_sum_long(s, sh);
    for (std::uint32_t i = threadIdx.x; i < cols; i += kLongThreads) st1(y + i, expf(in(i) - m) * inv);
  }
}

// ------------------------------------------------------------ host dispatch

template <RowOp OP, typename T, int VEC, int TPR, int NV, bool STORE_H>
inline int launch_row_cfg(const RowArgs& a, cudaStream_t s) {
  constexpr int kRpc = rows_per_cta<TPR>();
  const std::uint64_t blocks = (a.rows + kRpc - 1) / kRpc;
  return launch_serialised(row_kernel<OP, T, VEC, TPR, NV, STORE_H>,
                           dim3(static_cast<unsigned>(blocks)), dim3(TPR * kRpc), 0, s, a);
}

// units = row width in VEC-element vectors.  Chooses the smallest thread
// group whose registers hold the whole row (at most 8 vectors per thread).
template <RowOp OP, typename T, int VEC, bool STORE_H>
inline int dispatch_row_width(std::uint32_t units, const RowArgs& a, cudaStream_t s) {
  if (units <= 32) return launch_row_cfg<OP, T, VEC, 32, 1, STORE_H>(a, s);
  if (units <= 64) return launch_row_cfg<OP, T, VEC, 32, 2, STORE_H>(a, s);
  if (units <= 128) return launch_row_cfg<OP, T, VEC, 32, 4, STORE_H>(a, s);
  if (units <= 256) return launch_row_cfg<OP, T, VEC, 64, 4, STORE_H>(a, s);
  if (units <= 512) return launch_row_cfg<OP, T, VEC, 128, 4, STORE_H>(a, s);
  if (units <= 1024) return launch_row_cfg<OP, T, VEC, 256, 4, STORE_H>(a, s);
  if (units <= 2048) return launch_row_cfg<OP, T, VEC, 512, 4, STORE_H>(a, s);
  if (units <= 4096) return launch_row_cfg<OP, T, VEC, 1024, 4, STORE_H>(a, s);
  if (units <= 8192) return launch_row_cfg<OP, T, VEC, 1024, 8, STORE_H>(a, s);
  return launch_serialised(row_kernel_long<OP, T, STORE_H>, dim3(static_cast<unsigned>(a.rows)),
                           dim3(kLongThreads), 0, s, a);
}

template <RowOp OP, typename T, bool STORE_H>
inline int launch_rows(const RowArgs& a, cudaStream_t s) {
  constexpr int kVec = std::is_same<T, float>::value ? 4 : 8;
  bool vec = (a.cols % kVec) == 0 && aligned16(a.x) && aligned16(a.y) && aligned16(a.weight);
  if (OP == RowOp::kLayerNorm || OP == RowOp::kResidualLayerNorm) vec = vec && aligned16(a.bias);
  if (has_residual(OP)) vec = vec && aligned16(a.residual);
  if (STORE_H) vec = vec && aligned16(a.h);
  if (OP == RowOp::kSoftmax) vec = (a.cols % kVec) == 0 && aligned16(a.x) && aligned16(a.y);
  if (OP == RowOp::kRmsRstd) vec = (a.cols % kVec) == 0 && aligned16(a.x);
  if (vec) return dispatch_row_width<OP, T, kVec, STORE_H>(a.cols / kVec, a, s);
  return dispatch_row_width<OP, T, 1, STORE_H>(a.cols, a, s);
}

// Reference argument rules (rmsnorm.cu:208-225, layernorm.cu:411-430,
// softmax.cu:336-348): rows == 0 succeeds before any other check; NULL
// pointers, cols == 0 and eps <= 0 are cudaErrorInvalidValue.
inline bool row_dims_ok(std::uint64_t rows, std::uint64_t cols) {
  return cols != 0 && cols <= 0x7fffffffull && rows <= 0x7fffffffull;
}

}  // namespace col
