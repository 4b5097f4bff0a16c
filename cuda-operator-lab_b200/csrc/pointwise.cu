// Pointwise fused ops: bias + exact GELU (fused_bias_gelu.cuh:5-29) and
// SwiGLU (swiglu.cuh:5-27).  Both are pure HBM streams: 16-byte loads and
// stores, several independent vectors in flight per thread, and a grid of
// exactly one resident wave (SM count x CTAs per SM from the occupancy API)
// with equal work per CTA, so no SM idles in a partial second wave.  Plain
// (L2-allocating) loads and stores: the output usually feeds the next kernel.
#include <mutex>

#include "common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;  // independent 16-byte vectors in flight per thread

// CTAs of `kKernel` resident on the whole device (queried once per device
// and kernel; 8 per SM if the query fails).
template <auto kKernel>
std::uint64_t wave_ctas() {
  constexpr int kMaxDevices = 64;
  static int cached[kMaxDevices] = {};
  static std::once_flag flags[kMaxDevices];
  int dev = 0;
  const col::DeviceInfo& info = col::device_info(&dev);
  std::call_once(flags[dev & 63], [dev]() {
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kKernel, kThreads, 0) != cudaSuccess ||
        blocks <= 0) {
      cudaGetLastError();
      blocks = 8;
    }
    cached[dev & 63] = blocks;
  });
  return static_cast<std::uint64_t>(info.sm_count) * cached[dev & 63];
}

unsigned grid_for(std::uint64_t work_items, std::uint64_t wave) {
  std::uint64_t blocks = (work_items + kThreads - 1) / kThreads;
  if (blocks > wave) blocks = wave;
  if (blocks == 0) blocks = 1;
  return static_cast<unsigned>(blocks);
}

// ---------------------------------------------------------------- SwiGLU

__global__ void __launch_bounds__(kThreads)
swiglu_vec_kernel(const float4* __restrict__ g, const float4* __restrict__ u,
                  float4* __restrict__ o, std::uint64_t nvec) {
  col::grid_dependency_wait();
  const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
  // Groups of kUnroll strided vectors, the last group predicated, so the
  // ragged end costs one memory round trip like every other group.
  for (std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x; i < nvec;
       i += kUnroll * stride) {
    float4 gv[kUnroll], uv[kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      const std::uint64_t idx = i + j * stride;
      if (idx < nvec) {
        gv[j] = g[idx];
        uv[j] = u[idx];
      }
    }
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      const std::uint64_t idx = i + j * stride;
      if (idx < nvec) {
        float4 r;
        r.x = col::silu_f(gv[j].x) * uv[j].x;
        r.y = col::silu_f(gv[j].y) * uv[j].y;
        r.z = col::silu_f(gv[j].z) * uv[j].z;
        r.w = col::silu_f(gv[j].w) * uv[j].w;
        o[idx] = r;
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads)
swiglu_scalar_kernel(const float* __restrict__ g, const float* __restrict__ u,
                     float* __restrict__ o, std::uint64_t begin, std::uint64_t n) {
  col::grid_dependency_wait();
  const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
  for (std::uint64_t i = begin + static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
       i < n; i += stride) {
    o[i] = col::silu_f(g[i]) * u[i];
  }
}

int swiglu_launch(const float* g, const float* u, float* o, std::uint64_t n, cudaStream_t s) {
  std::uint64_t done = 0;
  if (col::aligned16(g) && col::aligned16(u) && col::aligned16(o)) {
    const std::uint64_t nvec = n / 4;
    if (nvec) {
      const int rc = col::launch_serialised(
          swiglu_vec_kernel, dim3(grid_for(nvec, wave_ctas<swiglu_vec_kernel>())), dim3(kThreads),
          0, s, reinterpret_cast<const float4*>(g), reinterpret_cast<const float4*>(u),
          reinterpret_cast<float4*>(o), nvec);
      if (rc != 0) return rc;
      done = nvec * 4;
    }
  }
  if (done < n) {
    return col::launch_serialised(
        swiglu_scalar_kernel, dim3(grid_for(n - done, wave_ctas<swiglu_scalar_kernel>())),
        dim3(kThreads), 0, s, g, u, o, done, n);
  }
  return 0;
}

// ---------------------------------------------------------------- bias + GELU

// 2-D decomposition: blockIdx.x picks 256 float4 columns, blockIdx.y strides
// over rows.  Each thread loads its bias vector once and reuses it for every
// row it visits (no per-element modulo, no repeated bias loads), with kUnroll
// rows in flight.
__global__ void __launch_bounds__(kThreads)
bias_gelu_vec_kernel(const float4* __restrict__ x, const float4* __restrict__ b,
                     float4* __restrict__ o, std::uint32_t rows, std::uint32_t vcols) {
  col::grid_dependency_wait();
  const std::uint32_t c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= vcols) return;
  const float4 bv = __ldg(b + c);
  const std::uint32_t rstride = gridDim.y;
  for (std::uint32_t r = blockIdx.y; r < rows; r += kUnroll * rstride) {
    float4 xv[kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      const std::uint32_t rr = r + j * rstride;
      if (rr < rows) xv[j] = x[static_cast<std::uint64_t>(rr) * vcols + c];
    }
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      const std::uint32_t rr = r + j * rstride;
      if (rr < rows) {
        float4 v;
        v.x = col::gelu_erf_f(xv[j].x + bv.x);
        v.y = col::gelu_erf_f(xv[j].y + bv.y);
        v.z = col::gelu_erf_f(xv[j].z + bv.z);
        v.w = col::gelu_erf_f(xv[j].w + bv.w);
        o[static_cast<std::uint64_t>(rr) * vcols + c] = v;
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads)
bias_gelu_scalar_kernel(const float* __restrict__ x, const float* __restrict__ b,
                        float* __restrict__ o, std::uint64_t rows, std::uint32_t cols) {
  col::grid_dependency_wait();
  const std::uint64_t total = rows * cols;
  const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
  for (std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
       i < total; i += stride) {
    o[i] = col::gelu_erf_f(x[i] + __ldg(b + static_cast<std::uint32_t>(i % cols)));
  }
}

int bias_gelu(const float* x, const float* b, float* o, std::uint64_t rows, std::uint64_t cols,
              void* stream) {
  // fused_bias_gelu.cu:54-66: rows == 0 succeeds first; NULL or cols == 0 fail.
  if (rows == 0) return 0;
  if (x == nullptr || b == nullptr || o == nullptr || cols == 0 || cols > 0xffffffffull) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const cudaStream_t s = col::as_stream(stream);
  const std::uint32_t c = static_cast<std::uint32_t>(cols);
  if ((c % 4) == 0 && col::aligned16(x) && col::aligned16(b) && col::aligned16(o) &&
      rows <= 0xffffffffull) {
    const std::uint32_t vcols = c / 4;
    const unsigned gx = (vcols + kThreads - 1) / kThreads;
    // Row slots per column block: as many as one wave holds, then trimmed so
    // every slot visits the same number of rows (rows_per = ceil(rows / gy)).
    const std::uint64_t wave = wave_ctas<bias_gelu_vec_kernel>();
    std::uint64_t gy = wave / gx;
    if (gy == 0) gy = 1;
    if (gy > 65535) gy = 65535;
    const std::uint64_t rows_per = (rows + gy - 1) / gy;
    gy = (rows + rows_per - 1) / rows_per;
    return col::launch_serialised(
        bias_gelu_vec_kernel, dim3(gx, static_cast<unsigned>(gy)), dim3(kThreads), 0, s,
        reinterpret_cast<const float4*>(x), reinterpret_cast<const float4*>(b),
        reinterpret_cast<float4*>(o), static_cast<std::uint32_t>(rows), vcols);
  }
  return col::launch_serialised(
      bias_gelu_scalar_kernel, dim3(grid_for(rows * c, wave_ctas<bias_gelu_scalar_kernel>())),
      dim3(kThreads), 0, s, x, b, o, rows, c);
}

}  // namespace

COL_API int cuda_operator_fused_bias_gelu_v0(const float* input, const float* bias, float* output,
                                             uint64_t rows, uint64_t cols, void* stream) {
  return bias_gelu(input, bias, output, rows, cols, stream);
}
COL_API int cuda_operator_fused_bias_gelu_v1(const float* input, const float* bias, float* output,
                                             uint64_t rows, uint64_t cols, void* stream) {
  return bias_gelu(input, bias, output, rows, cols, stream);
}
COL_API int cuda_operator_fused_bias_gelu_v2(const float* input, const float* bias, float* output,
                                             uint64_t rows, uint64_t cols, void* stream) {
  return bias_gelu(input, bias, output, rows, cols, stream);
}

// swiglu.cu:50-61 (v0/v1): elements == 0 succeeds first; NULL fails.
COL_API int cuda_operator_swiglu_v0(const float* gate, const float* up, float* output,
                                    uint64_t elements, void* stream) {
  if (elements == 0) return 0;
  if (gate == nullptr || up == nullptr || output == nullptr) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  return swiglu_launch(gate, up, output, elements, col::as_stream(stream));
}
COL_API int cuda_operator_swiglu_v1(const float* gate, const float* up, float* output,
                                    uint64_t elements, void* stream) {
  return cuda_operator_swiglu_v0(gate, up, output, elements, stream);
}
// swiglu.cu:115-128 (v2): rows*cols == 0 succeeds first; NULL or cols == 0 fail.
COL_API int cuda_operator_swiglu_v2(const float* gate, const float* up, float* output,
                                    uint64_t rows, uint64_t cols, void* stream) {
  const std::uint64_t elements = rows * cols;
  if (elements == 0) return 0;
  if (gate == nullptr || up == nullptr || output == nullptr || cols == 0) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  return swiglu_launch(gate, up, output, elements, col::as_stream(stream));
}
