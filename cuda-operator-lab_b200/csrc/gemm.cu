// GEMM entry points: gemm_swiglu v0..v11 (gemm_swiglu.cuh:5-136),
// gemm_bias_gelu v0..v6 (gemm_bias_gelu.cuh:5-79) and the bf16-output
// variants.  bf16 operands go to the tcgen05 kernel (gemm_sm100.cuh) whenever
// TMA can address them; fp32 operands and unaddressable bf16 layouts go to the
// CUDA-core kernel (gemm_simt.cuh).
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>
#include <mutex>

#include "gemm_simt.cuh"
#include "gemm_sm100.cuh"
#include "gemm_sm100_2sm.cuh"

namespace {

using col::sm100::GemmParams;
using col::sm100::TileCfg;

// Device-side status word of the bounded waits (one per device context).
__device__ unsigned g_gemm_status;

constexpr int kMaxDevices = 64;

unsigned* status_ptr(int dev) {
  static unsigned* ptrs[kMaxDevices] = {};
  static std::once_flag flags[kMaxDevices];
  std::call_once(flags[dev], [dev]() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemm_status) == cudaSuccess) ptrs[dev] = static_cast<unsigned*>(p);
  });
  return ptrs[dev];
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  });
  return fn;
}

// 2-D bf16 map over a row-major [rows, cols] matrix; box = 64 columns (128 B,
// the 128-byte swizzle span) x box_rows rows.  Out-of-range boxes read zeros.
int encode_bf16_rows(CUtensorMap* map, const void* base, std::uint64_t rows, std::uint64_t cols,
                     std::uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return col::kErrNoTensorMapEncoder;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(col::sm100::kBlockK), box_rows};
  const cuuint32_t estrides[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                         strides, box, estrides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : col::kErrTensorMapEncode;
}

template <int BNH, int EPI, typename TOut>
int launch_tc(GemmParams& p, cudaStream_t s, int dev, int sm_count) {
  using Cfg = TileCfg<BNH>;
  auto kernel = col::sm100::gemm_bf16_tc_kernel<BNH, EPI, TOut>;
  static std::atomic<std::uint64_t> attr_set{0};
  const std::uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set.load(std::memory_order_acquire) & bit)) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(Cfg::kSmemBytes));
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set.fetch_or(bit, std::memory_order_release);
  }
  const int tiles = p.num_m_blocks * p.num_n_blocks;
  const int grid = tiles < sm_count ? tiles : sm_count;
  kernel<<<grid, col::sm100::kCtaThreads, Cfg::kSmemBytes, s>>>(p);
  return static_cast<int>(cudaGetLastError());
}

// CTA pairs (2-SM kernel) that can be resident at once on the current device
// (cudaOccupancyMaxActiveClusters for one instantiation; every BNH variant
// uses over half of the shared memory, so all fit one CTA per SM and share
// the answer).  Queried once per device; 0 if clusters are unavailable.
template <int EPI, typename TOut>
int max_pair_clusters(int dev) {
  using Cfg = col::sm100::TileCfg2<128>;
  static int cached[64] = {};
  static std::once_flag flags[64];
  std::call_once(flags[dev & 63], [dev]() {
    auto kernel = col::sm100::gemm_bf16_tc2_kernel<128, EPI, TOut>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(col::sm100::kCtaThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters <= 0) {
      cudaGetLastError();  // clear the error; fall back to the 1-CTA kernel
      clusters = 0;
    }
    cached[dev & 63] = clusters;
  });
  return cached[dev & 63];
}

template <int BNH, int EPI, typename TOut>
int launch_tc2(GemmParams& p, cudaStream_t s, int dev, int clusters) {
  using Cfg = col::sm100::TileCfg2<BNH>;
  auto kernel = col::sm100::gemm_bf16_tc2_kernel<BNH, EPI, TOut>;
  const int tiles = p.num_m_blocks * p.num_n_blocks;
  const int grid = 2 * (tiles < clusters ? tiles : clusters);
  kernel<<<grid, col::sm100::kCtaThreads, Cfg::kSmemBytes, s>>>(p);
  (void)dev;
  return static_cast<int>(cudaGetLastError());
}

template <int BNH, int EPI, typename TOut>
int set_smem_attr_2sm(int dev) {
  using Cfg = col::sm100::TileCfg2<BNH>;
  static std::atomic<std::uint64_t> attr_set{0};
  const std::uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set.load(std::memory_order_acquire) & bit)) {
    const cudaError_t e = cudaFuncSetAttribute(col::sm100::gemm_bf16_tc2_kernel<BNH, EPI, TOut>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(Cfg::kSmemBytes));
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set.fetch_or(bit, std::memory_order_release);
  }
  return 0;
}

enum class BMode { kSwiGLU, kGelu };

// Tile width: the B box height BNH (MMA N = 2*BNH; output columns per tile =
// BNH for SwiGLU, 2*BNH for GELU).  The persistent grid processes tiles in
// waves of sm_count; a tile's main loop costs ~2*BNH MMA columns per k-block,
// so the cost of a choice is waves * 2*BNH.  Ties go to the wider tile (fewer
// epilogues, better MMA efficiency).  Example: M=512, N=4096 SwiGLU gives 128
// tiles at BNH=128 (one 86 %-full wave) but exactly 148 at BNH=112.
int choose_bnh(int mblocks, std::uint64_t n, bool swiglu, int sm_count) {
  constexpr int kCandidates[] = {128, 112, 96, 64};
  int best = 128;
  std::uint64_t best_cost = ~0ull;
  for (int bnh : kCandidates) {
    const std::uint64_t cols = swiglu ? bnh : 2 * bnh;
    const std::uint64_t tiles = static_cast<std::uint64_t>(mblocks) * ((n + cols - 1) / cols);
    const std::uint64_t waves = (tiles + sm_count - 1) / sm_count;
    const std::uint64_t cost = waves * 2 * bnh;
    if (cost < best_cost) {
      best_cost = cost;
      best = bnh;
    }
  }
  return best;
}

// bf16 tensor-core path.  For kSwiGLU, w0/w1 are the gate/up matrices [n, k];
// for kGelu, w0 is W [n, k] (w1 ignored).  Returns -1 when TMA cannot address
// the operands (caller falls back to the CUDA-core kernel).
template <int EPI, typename TOut>
int gemm_bf16_tc(const void* x, const void* w0, const void* w1, BMode mode, const float* bias,
                 void* out, std::uint64_t m, std::uint64_t n, std::uint64_t k, cudaStream_t s) {
  if ((k % 8) != 0 || !col::aligned16(x) || !col::aligned16(w0) ||
      (mode == BMode::kSwiGLU && !col::aligned16(w1))) {
    return -1;
  }
  int dev = 0;
  const col::DeviceInfo& info = col::device_info(&dev);
  if (info.cc_major != 10) return col::kErrDeviceNotSupported;
  unsigned* status = status_ptr(dev);
  if (!status) return static_cast<int>(cudaErrorInvalidDevice);

  const int mblocks = static_cast<int>((m + 127) / 128);
  // CTA-pair kernel when there are at least two 128-row blocks: half of each
  // weight tile per SM.  Its BNH choice uses pair blocks and pair slots.
  const bool pair = mblocks >= 2;
  int pair_slots = 0;
  if (pair) {
    if (int rc = set_smem_attr_2sm<128, EPI, TOut>(dev)) return rc;
    pair_slots = max_pair_clusters<EPI, TOut>(dev);
  }
  const bool use_pair = pair && pair_slots > 0;
  const int mblocks_sched = use_pair ? (mblocks + 1) / 2 : mblocks;
  const int bnh = choose_bnh(mblocks_sched, n, mode == BMode::kSwiGLU,
                             use_pair ? pair_slots : info.sm_count);

  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  int rc = encode_bf16_rows(&p.map_a, x, m, k, 128);
  if (rc == 0) rc = encode_bf16_rows(&p.map_b0, w0, n, k, bnh);
  if (rc == 0) rc = encode_bf16_rows(&p.map_b1, mode == BMode::kSwiGLU ? w1 : w0, n, k, bnh);
  if (rc == col::kErrTensorMapEncode) return -1;  // layout TMA cannot express: CUDA cores
  if (rc != 0) return rc;
  p.bias = bias;
  p.out = out;
  p.status = status;
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.num_m_blocks = mblocks_sched;
  p.num_k_blocks = static_cast<int>((k + col::sm100::kBlockK - 1) / col::sm100::kBlockK);
  if (mode == BMode::kSwiGLU) {
    p.num_n_blocks = static_cast<int>((n + bnh - 1) / bnh);
    p.b_row_stride = bnh;
    p.b1_row_offset = 0;
  } else {
    p.num_n_blocks = static_cast<int>((n + 2 * bnh - 1) / (2 * bnh));
    p.b_row_stride = 2 * bnh;
    p.b1_row_offset = bnh;
  }
  // Few M-blocks per weight tile: the weights stream from DRAM with little L2
  // reuse, so warm L2 ahead of the ring.  Many M-blocks: the raster already
  // keeps each weight tile L2-resident across its M-group.
  p.prefetch_b = mblocks <= 8 ? 1 : 0;
  p.out_ld = static_cast<int>(n);
  p.out_vec_ok = col::aligned16(out) && ((n * sizeof(TOut)) % 16 == 0);
  if (use_pair) {
    int rc = 0;
    switch (bnh) {
      case 128: return launch_tc2<128, EPI, TOut>(p, s, dev, pair_slots);
      case 112:
        if ((rc = set_smem_attr_2sm<112, EPI, TOut>(dev))) return rc;
        return launch_tc2<112, EPI, TOut>(p, s, dev, pair_slots);
      case 96:
        if ((rc = set_smem_attr_2sm<96, EPI, TOut>(dev))) return rc;
        return launch_tc2<96, EPI, TOut>(p, s, dev, pair_slots);
      default:
        if ((rc = set_smem_attr_2sm<64, EPI, TOut>(dev))) return rc;
        return launch_tc2<64, EPI, TOut>(p, s, dev, pair_slots);
    }
  }
  switch (bnh) {
    case 128: return launch_tc<128, EPI, TOut>(p, s, dev, info.sm_count);
    case 112: return launch_tc<112, EPI, TOut>(p, s, dev, info.sm_count);
    case 96: return launch_tc<96, EPI, TOut>(p, s, dev, info.sm_count);
    default: return launch_tc<64, EPI, TOut>(p, s, dev, info.sm_count);
  }
}

template <typename TIn, int EPI, typename TOut>
int gemm_simt(const void* x, const void* w0, const void* w1, const float* bias, void* out,
              std::uint64_t m, std::uint64_t n, std::uint64_t k, cudaStream_t s) {
  col::simt::SimtParams p{x, w0, w1, bias, out, static_cast<int>(m), static_cast<int>(n),
                          static_cast<int>(k)};
  return col::simt::launch_simt<TIn, EPI, TOut>(p, s);
}

// bf16 SwiGLU: tensor cores when addressable, CUDA cores otherwise.
template <int EPI, typename TOut>
int swiglu_bf16(const void* x, const void* wg, const void* wu, void* out, std::uint64_t m,
                std::uint64_t n, std::uint64_t k, cudaStream_t s) {
  const int rc = gemm_bf16_tc<EPI, TOut>(x, wg, wu, BMode::kSwiGLU, nullptr, out, m, n, k, s);
  if (rc != -1) return rc;
  return gemm_simt<__nv_bfloat16, EPI, TOut>(x, wg, wu, nullptr, out, m, n, k, s);
}

inline bool dims_ok(std::uint64_t m, std::uint64_t n, std::uint64_t k, std::uint64_t n_limit) {
  return m <= 0x7fffffffull && n <= n_limit && k <= 0x7fffffffull && k != 0;
}

const void* up_half(const void* packed, std::uint64_t n, std::uint64_t k, std::size_t elem) {
  return static_cast<const char*>(packed) + n * k * elem;
}

// ---------------------------------------------------------------- fp32 GEMMs

// gemm_swiglu.cu:143-163: m == 0 or n == 0 succeeds first; NULL, k == 0 and
// sizes above INT32_MAX are invalid.
int swiglu_f32_dual(const float* x, const float* wg, const float* wu, const float* ws, float* out,
                    std::uint64_t m, std::uint64_t k, std::uint64_t n, void* stream) {
  if (m == 0 || n == 0) return 0;
  if (!x || !wg || !wu || !ws || !out || !dims_ok(m, n, k, 0x7fffffffull)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  return gemm_simt<float, col::sm100::kEpiSwiGLU, float>(x, wg, wu, nullptr, out, m, n, k,
                                                        col::as_stream(stream));
}

// gemm_swiglu.cu:335-351: packed [2N, K]; n above INT32_MAX / 2 is invalid.
int swiglu_f32_packed(const float* x, const float* w, const float* ws, float* out, std::uint64_t m,
                      std::uint64_t k, std::uint64_t n, void* stream) {
  if (m == 0 || n == 0) return 0;
  if (!x || !w || !ws || !out || !dims_ok(m, n, k, 0x7fffffffull / 2)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  return gemm_simt<float, col::sm100::kEpiSwiGLU, float>(
      x, w, up_half(w, n, k, sizeof(float)), nullptr, out, m, n, k, col::as_stream(stream));
}

template <int EPI>
int bias_gelu_f32(const float* x, const float* w, const float* b, float* out, std::uint64_t m,
                  std::uint64_t k, std::uint64_t n, void* stream) {
  // gemm_bias_gelu.cu:830-849.
  if (m == 0 || n == 0) return 0;
  if (!x || !w || !b || !out || !dims_ok(m, n, k, 0x7fffffffull)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  return gemm_simt<float, EPI, float>(x, w, nullptr, b, out, m, n, k, col::as_stream(stream));
}

// ---------------------------------------------------------------- bf16 GEMMs

int swiglu_bf16_packed_f32out(const void* x, const void* w, const void* ws, float* out,
                              std::uint64_t m, std::uint64_t k, std::uint64_t n, void* stream,
                              bool round_bf16) {
  // gemm_swiglu.cu:991-1012.
  if (m == 0 || n == 0) return 0;
  if (!x || !w || !ws || !out || !dims_ok(m, n, k, 0x7fffffffull / 2)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const void* wu = up_half(w, n, k, 2);
  if (round_bf16) {
    return swiglu_bf16<col::sm100::kEpiSwiGLURoundBf16, float>(x, w, wu, out, m, n, k,
                                                              col::as_stream(stream));
  }
  return swiglu_bf16<col::sm100::kEpiSwiGLU, float>(x, w, wu, out, m, n, k, col::as_stream(stream));
}

int swiglu_bf16_dual_f32out(const void* x, const void* wg, const void* wu, float* out,
                            std::uint64_t m, std::uint64_t k, std::uint64_t n, void* stream,
                            std::uint64_t m_mult, std::uint64_t k_mult, std::uint64_t n_mult) {
  // gemm_swiglu.cu:1108-1132 (and the V7/V8/V9 guards at :1169, :1213, :1257).
  if (m == 0 || n == 0) return 0;
  if (!x || !wg || !wu || !out || k == 0) return static_cast<int>(cudaErrorInvalidValue);
  if ((m % m_mult) != 0 || (k % k_mult) != 0 || (n % n_mult) != 0) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (!dims_ok(m, n, k, 0x7fffffffull)) return static_cast<int>(cudaErrorInvalidValue);
  return swiglu_bf16<col::sm100::kEpiSwiGLU, float>(x, wg, wu, out, m, n, k, col::as_stream(stream));
}

}  // namespace

// ---------------------------------------------------------------- exports

COL_API int cuda_operator_gemm_swiglu_v0(const float* input, const float* gate_weight,
                                         const float* up_weight, float* workspace, float* output,
                                         uint64_t m, uint64_t k, uint64_t n, void* stream) {
  return swiglu_f32_dual(input, gate_weight, up_weight, workspace, output, m, k, n, stream);
}
COL_API int cuda_operator_gemm_swiglu_v1(const float* input, const float* gate_weight,
                                         const float* up_weight, float* workspace, float* output,
                                         uint64_t m, uint64_t k, uint64_t n, void* stream) {
  return swiglu_f32_dual(input, gate_weight, up_weight, workspace, output, m, k, n, stream);
}
COL_API int cuda_operator_gemm_swiglu_v2(const float* input, const float* packed_weight,
                                         float* workspace, float* output, uint64_t m, uint64_t k,
                                         uint64_t n, void* stream) {
  return swiglu_f32_packed(input, packed_weight, workspace, output, m, k, n, stream);
}
COL_API int cuda_operator_gemm_swiglu_v3(const float* input, const float* packed_weight,
                                         float* workspace, float* output, uint64_t m, uint64_t k,
                                         uint64_t n, void* stream) {
  return swiglu_f32_packed(input, packed_weight, workspace, output, m, k, n, stream);
}
COL_API int cuda_operator_gemm_swiglu_v4(const void* input_bf16, const void* packed_weight_bf16,
                                         float* workspace, float* output, uint64_t m, uint64_t k,
                                         uint64_t n, void* stream) {
  return swiglu_bf16_packed_f32out(input_bf16, packed_weight_bf16, workspace, output, m, k, n,
                                   stream, false);
}
COL_API int cuda_operator_gemm_swiglu_v5(const void* input_bf16, const void* packed_weight_bf16,
                                         void* workspace_bf16, float* output, uint64_t m,
                                         uint64_t k, uint64_t n, void* stream) {
  return swiglu_bf16_packed_f32out(input_bf16, packed_weight_bf16, workspace_bf16, output, m, k, n,
                                   stream, true);
}
COL_API int cuda_operator_gemm_swiglu_v6(const void* input_bf16, const void* gate_weight_bf16,
                                         const void* up_weight_bf16, float* output, uint64_t m,
                                         uint64_t k, uint64_t n, void* stream) {
  return swiglu_bf16_dual_f32out(input_bf16, gate_weight_bf16, up_weight_bf16, output, m, k, n,
                                 stream, 16, 16, 16);
}
COL_API int cuda_operator_gemm_swiglu_v7(const void* input_bf16, const void* gate_weight_bf16,
                                         const void* up_weight_bf16, float* output, uint64_t m,
                                         uint64_t k, uint64_t n, void* stream) {
  return swiglu_bf16_dual_f32out(input_bf16, gate_weight_bf16, up_weight_bf16, output, m, k, n,
                                 stream, 16, 16, 64);
}
COL_API int cuda_operator_gemm_swiglu_v8(const void* input_bf16, const void* gate_weight_bf16,
                                         const void* up_weight_bf16, float* output, uint64_t m,
                                         uint64_t k, uint64_t n, void* stream) {
  return swiglu_bf16_dual_f32out(input_bf16, gate_weight_bf16, up_weight_bf16, output, m, k, n,
                                 stream, 32, 16, 64);
}
COL_API int cuda_operator_gemm_swiglu_v9(const void* input_bf16, const void* gate_weight_bf16,
                                         const void* up_weight_bf16, float* output, uint64_t m,
                                         uint64_t k, uint64_t n, void* stream) {
  return swiglu_bf16_dual_f32out(input_bf16, gate_weight_bf16, up_weight_bf16, output, m, k, n,
                                 stream, 16, 16, 128);
}
COL_API int cuda_operator_gemm_swiglu_v10(const void* input_bf16, const void* packed_weight_bf16,
                                          float* workspace, float* output, uint64_t m, uint64_t k,
                                          uint64_t n, void* stream) {
  return swiglu_bf16_packed_f32out(input_bf16, packed_weight_bf16, workspace, output, m, k, n,
                                   stream, false);
}
COL_API int cuda_operator_gemm_swiglu_v11(const void* input_bf16, const void* packed_weight_bf16,
                                          float* workspace, float* output, uint64_t m, uint64_t k,
                                          uint64_t n, void* stream) {
  return swiglu_bf16_packed_f32out(input_bf16, packed_weight_bf16, workspace, output, m, k, n,
                                   stream, false);
}

#define COL_GEMM_BIAS_GELU(V, EPI)                                                               \
  COL_API int cuda_operator_gemm_bias_gelu_##V(const float* input, const float* weight,          \
                                               const float* bias, float* output, uint64_t m,     \
                                               uint64_t k, uint64_t n, void* stream) {           \
    return bias_gelu_f32<EPI>(input, weight, bias, output, m, k, n, stream);                     \
  }
COL_GEMM_BIAS_GELU(v0, col::sm100::kEpiBiasGeluErf)
COL_GEMM_BIAS_GELU(v1, col::sm100::kEpiBiasGeluErf)
COL_GEMM_BIAS_GELU(v2, col::sm100::kEpiBiasGeluTanh)
COL_GEMM_BIAS_GELU(v3, col::sm100::kEpiBiasGeluTanh)
COL_GEMM_BIAS_GELU(v4, col::sm100::kEpiBiasGeluTanh)
COL_GEMM_BIAS_GELU(v5, col::sm100::kEpiBiasGeluTanh)
COL_GEMM_BIAS_GELU(v6, col::sm100::kEpiBiasGeluTanh)
#undef COL_GEMM_BIAS_GELU

COL_API int cuda_operator_gemm_swiglu_bf16(const void* input_bf16, const void* packed_weight_bf16,
                                           void* output_bf16, uint64_t m, uint64_t k, uint64_t n,
                                           void* stream) {
  if (m == 0 || n == 0) return 0;
  if (!input_bf16 || !packed_weight_bf16 || !output_bf16 || !dims_ok(m, n, k, 0x7fffffffull / 2)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  return swiglu_bf16<col::sm100::kEpiSwiGLU, __nv_bfloat16>(
      input_bf16, packed_weight_bf16, up_half(packed_weight_bf16, n, k, 2), output_bf16, m, n, k,
      col::as_stream(stream));
}

COL_API int cuda_operator_gemm_bias_gelu_bf16(const void* input_bf16, const void* weight_bf16,
                                              const float* bias, void* output_bf16, uint64_t m,
                                              uint64_t k, uint64_t n, void* stream) {
  if (m == 0 || n == 0) return 0;
  if (!input_bf16 || !weight_bf16 || !bias || !output_bf16 || !dims_ok(m, n, k, 0x7fffffffull)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const cudaStream_t s = col::as_stream(stream);
  const int rc = gemm_bf16_tc<col::sm100::kEpiBiasGeluErf, __nv_bfloat16>(
      input_bf16, weight_bf16, nullptr, BMode::kGelu, bias, output_bf16, m, n, k, s);
  if (rc != -1) return rc;
  return gemm_simt<__nv_bfloat16, col::sm100::kEpiBiasGeluErf, __nv_bfloat16>(
      input_bf16, weight_bf16, nullptr, bias, output_bf16, m, n, k, s);
}

COL_API int cuda_operator_lab_gemm_status(unsigned int* status, int clear) {
  if (status == nullptr) return static_cast<int>(cudaErrorInvalidValue);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemcpyFromSymbol(status, g_gemm_status, sizeof(unsigned));
  if (e != cudaSuccess) return static_cast<int>(e);
  if (clear) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(unsigned));
  }
  return static_cast<int>(e);
}
