// Shared host/device helpers for the sm_100a operator library.
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/cuda_operator_lab.h"

#define COL_API extern "C" __attribute__((visibility("default")))

namespace col {

// Library-specific return codes (cudaError_t values stay below 10000).
constexpr int kErrNoTensorMapEncoder = 10001;   // driver lacks cuTensorMapEncodeTiled
constexpr int kErrTensorMapEncode = 10002;      // cuTensorMapEncodeTiled rejected a map
constexpr int kErrDeviceNotSupported = 10003;   // device is not sm_100
constexpr int kErrNoAllocCapacity = 10004;      // input larger than the allocation-free sum's scratch
constexpr int kErrGatherLayout = 10005;         // peer-gather GEMM operands the tensor path cannot take

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Programmatic dependent launch.  The library's kernels are launched with
// programmatic stream serialisation (launch_serialised): a launch may start
// while the previous kernel on its stream is still running.  Before touching
// global memory every kernel waits until the previous grid has completed and
// its memory is visible (grid_dependency_wait; at once when there is none).
// What overlaps is launch latency and set-up, never memory traffic.  Only the
// tensor-core GEMMs (one CTA per SM, which nothing else fits beside) let the
// next launch start early (grid_dependents_launch); the other kernels trigger
// it by exiting, because an early trigger packs the next grid's CTAs beside
// running ones and unbalances it (measured: LayerNorm [128, 8192] 3.1 -> 3.7
// us with it, 2.7 us without).
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KernelArgs, typename... Args>
inline int launch_serialised(void (*kernel)(KernelArgs...), dim3 grid, dim3 block,
                             std::size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, args...));
}

inline bool aligned16(const void* p) {
  return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0u;
}

// Per-device properties read once (thread safe); the library never queries
// device attributes on the launch path after the first call on a device.
struct DeviceInfo {
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  int max_smem_optin = 0;
  int l2_bytes = 0;
};

// Library-owned stream-ordered memory pool of the current device (freed
// blocks stay mapped), shared by the operators that need scratch.
cudaError_t library_pool(cudaMemPool_t* pool);

// Stream-ordered scratch on stream s: from library_pool normally; while s is
// being captured into a CUDA graph, from cudaMallocAsync (a graph memory
// node), since creating the pool is not a capturable operation.  Release
// with cudaFreeAsync on the same stream.
cudaError_t scratch_alloc(void** ptr, std::size_t bytes, cudaStream_t s);

inline const DeviceInfo& device_info(int* device_out = nullptr) {
  constexpr int kMaxDevices = 64;
  static DeviceInfo infos[kMaxDevices];
  static std::once_flag flags[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) dev = 0;
  std::call_once(flags[dev], [dev]() {
    DeviceInfo info;
    cudaDeviceGetAttribute(&info.sm_count, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&info.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&info.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&info.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&info.l2_bytes, cudaDevAttrL2CacheSize, dev);
    if (info.sm_count <= 0) info.sm_count = 148;
    infos[dev] = info;
  });
  if (device_out) *device_out = dev;
  return infos[dev];
}

// ---------------------------------------------------------------- device math

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// silu(x) = x / (1 + exp(-x)), the form of swiglu.cu:11-13.
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// Exact-form GELU, 0.5 x (1 + erf(x / sqrt 2)) (fused_bias_gelu.cu:12-14),
// with erf from Abramowitz & Stegun, Handbook of Mathematical Functions,
// formula 7.1.26: for a >= 0, erfc(a) = t (a1 + t (a2 + t (a3 + t (a4 + t a5))))
// e^(-a^2) + e(a), t = 1 / (1 + p a), |e(a)| <= 1.5e-7.  1 + erf(z) is then
// 2 - erfc(z) for z >= 0 and erfc(-z) for z < 0, so negative z keeps full
// relative accuracy (no 1 + erf cancellation).  Two special-function-unit
// ops (one reciprocal, one exponential) per element instead of the library
// erff, which made the fp32 bias+GELU kernel compute-bound.  Error against the
// float64 function over [-12, 12], emulated in fp32: 4.2e-7 absolute, at most
// 0.21 of the 1e-6 + 1e-5 |y| bar.
__device__ __forceinline__ float gelu_erf_f(float x) {
  const float z = x * 0.70710678118654752440f;
  const float a = fabsf(z);
  const float t = __fdividef(1.0f, fmaf(0.3275911f, a, 1.0f));
  float poly = fmaf(1.061405429f, t, -1.453152027f);
  poly = fmaf(poly, t, 1.421413741f);
  poly = fmaf(poly, t, -0.284496736f);
  poly = fmaf(poly, t, 0.254829592f);
  const float erfc_a = poly * t * __expf(-a * a);
  const float one_plus_erf = z >= 0.0f ? 2.0f - erfc_a : erfc_a;
  return 0.5f * x * one_plus_erf;
}

// SiLU for the GEMM epilogues from two special-function-unit ops (__expf,
// and the approximate division __fdividef = x * rcp.approx(y)): a few ulp of
// fp32 (~1e-6 relative), far inside the GEMM tolerances, at a fraction of
// the instructions of expf + IEEE division -- the epilogue of a single-wave
// GEMM is on its critical path.  Saturates correctly: for x -> -inf the
// divisor overflows to +inf and the result is -0; for x -> +inf it is x.
__device__ __forceinline__ float silu_fast(float x) {
  return __fdividef(x, 1.0f + __expf(-x));
}

// tanh-approximate GELU, 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))),
// the form torch.nn.functional.gelu(approximate="tanh") and the reference's
// GELU_BIAS GEMM versions (v2..v6) produce.
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float inner = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanhf(inner));
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Streaming (evict-first) 16-byte load for read-once inputs whose data is not
// needed again (the global reduction).
__device__ __forceinline__ float4 ld_stream_f4(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ float4 ld_cached_f4(const float4* p) { return __ldg(p); }

__device__ __forceinline__ void unpack_bf16x8(uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&f)[8]) {
  uint4 v;
  v.x = pack_bf16x2(f[0], f[1]);
  v.y = pack_bf16x2(f[2], f[3]);
  v.z = pack_bf16x2(f[4], f[5]);
  v.w = pack_bf16x2(f[6], f[7]);
  return v;
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

}  // namespace col
