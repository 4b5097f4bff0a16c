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
#include "gemm_sm100_sk.cuh"

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

// Recently encoded tensor maps of the calling thread.  A map is a pure
// function of (base, rows, cols, box_rows) -- the element type, swizzle, L2
// promotion and fill are fixed -- so a call on the same operands (the common
// case: weights, and activations in reused buffers) copies 128 bytes instead
// of encoding again, which keeps a small GEMM's host path short.
struct TensorMapCacheEntry {
  CUtensorMap map;
  const void* base;
  std::uint64_t rows;
  std::uint64_t cols;
  std::uint32_t box_rows;
  bool valid;
};
constexpr int kTensorMapCacheSize = 16;

// 2-D bf16 map over a row-major [rows, cols] matrix; box = 64 columns (128 B,
// the 128-byte swizzle span) x box_rows rows.  Out-of-range boxes read zeros.
int encode_bf16_rows(CUtensorMap* map, const void* base, std::uint64_t rows, std::uint64_t cols,
                     std::uint32_t box_rows) {
  thread_local TensorMapCacheEntry cache[kTensorMapCacheSize] = {};
  const std::uintptr_t h = (reinterpret_cast<std::uintptr_t>(base) >> 7) ^ rows ^ (cols * 31u) ^
                           (static_cast<std::uintptr_t>(box_rows) * 131u);
  TensorMapCacheEntry& e = cache[(h ^ (h >> 4) ^ (h >> 9)) % kTensorMapCacheSize];
  if (e.valid && e.base == base && e.rows == rows && e.cols == cols && e.box_rows == box_rows) {
    std::memcpy(map, &e.map, sizeof(CUtensorMap));
    return 0;
  }
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
  if (r != CUDA_SUCCESS) return col::kErrTensorMapEncode;
  std::memcpy(&e.map, map, sizeof(CUtensorMap));
  e.base = base;
  e.rows = rows;
  e.cols = cols;
  e.box_rows = box_rows;
  e.valid = true;
  return 0;
}

template <int BNH, int EPI, typename TOut, bool FLUSH>
int launch_tc(GemmParams& p, cudaStream_t s, int dev, int sm_count) {
  using Cfg = TileCfg<BNH, FLUSH ? 1 : 2, col::sm100::epi_smem_reserve(EPI)>;
  auto kernel = col::sm100::gemm_bf16_tc_kernel<BNH, EPI, TOut, FLUSH>;
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
  return col::launch_serialised(kernel, dim3(grid), dim3(col::sm100::kCtaThreads),
                                 Cfg::kSmemBytes, s, p);
}

// CTA pairs (2-SM kernel) that can be resident at once on the current device
// (cudaOccupancyMaxActiveClusters for one instantiation; every BNH variant
// uses over half of the shared memory, so all fit one CTA per SM and share
// the answer).  Queried once per device; 0 if clusters are unavailable.
template <int EPI, typename TOut>
int max_pair_clusters(int dev) {
  using Cfg = col::sm100::TileCfg2<128, col::sm100::pair_kps(128, EPI, false),
                                    col::sm100::epi_smem_reserve(EPI)>;
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

template <int BNH, int EPI, typename TOut, bool FLUSH>
int launch_tc2(GemmParams& p, cudaStream_t s, int dev, int clusters) {
  using Cfg = col::sm100::TileCfg2<BNH, col::sm100::pair_kps(BNH, EPI, FLUSH),
                                    col::sm100::epi_smem_reserve(EPI)>;
  auto kernel = col::sm100::gemm_bf16_tc2_kernel<BNH, EPI, TOut, FLUSH>;
  const int tiles = p.num_m_blocks * p.num_n_blocks;
  const int grid = 2 * (tiles < clusters ? tiles : clusters);
  (void)dev;
  return col::launch_serialised(kernel, dim3(grid), dim3(col::sm100::kCtaThreads),
                                 Cfg::kSmemBytes, s, p);
}

template <int BNH, int EPI, typename TOut, bool FLUSH>
int set_smem_attr_2sm(int dev) {
  using Cfg = col::sm100::TileCfg2<BNH, col::sm100::pair_kps(BNH, EPI, FLUSH),
                                    col::sm100::epi_smem_reserve(EPI)>;
  static std::atomic<std::uint64_t> attr_set{0};
  const std::uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set.load(std::memory_order_acquire) & bit)) {
    const cudaError_t e = cudaFuncSetAttribute(col::sm100::gemm_bf16_tc2_kernel<BNH, EPI, TOut, FLUSH>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(Cfg::kSmemBytes));
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set.fetch_or(bit, std::memory_order_release);
  }
  return 0;
}

// Split-K cluster kernel (gemm_sm100_sk.cuh): shared-memory attribute and the
// number of co-resident 4-CTA clusters, both once per device.
template <int EPI, typename TOut>
int sk_clusters(int dev) {
  static int cached[64] = {};
  static std::once_flag flags[64];
  std::call_once(flags[dev & 63], [dev]() {
    auto kernel = col::sm100::gemm_bf16_sk_kernel<EPI, TOut>;
    int clusters = 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(col::sm100::kSkSmemBytes)) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(4, 1, 1);
      cfg.blockDim = dim3(col::sm100::kCtaThreads, 1, 1);
      cfg.dynamicSmemBytes = col::sm100::kSkSmemBytes;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 4;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) clusters = 0;
    }
    cudaGetLastError();  // a failed query means: no split-K path
    cached[dev & 63] = clusters > 0 ? clusters : 0;
  });
  return cached[dev & 63];
}

enum class BMode { kSwiGLU, kGelu };

// Tile width: the B box height BNH (MMA N = 2*BNH; output columns per tile =
// BNH for SwiGLU, 2*BNH for GELU).  The persistent grid processes tiles in
// waves of the resident CTAs (or pairs).  A k-block of the main loop costs a
// nearly width-independent floor -- measured 0.35 us at MMA N = 128 and 0.38 us
// at N = 256 per CTA pair, the producer/MMA handshake of the pipeline, not
// the MMA itself -- so a choice costs waves * (kKBlockFloor + 2*BNH), the
// floor expressed in MMA columns (fitted to those two points).  Fewer waves
// win; among equal waves the narrower tile wins slightly.  Examples: the
// N-sharded headline (M=16384, N=7168 per GPU) runs BNH=128 (49 waves) rather
// than BNH=96 (65 waves, which a pure MMA-column model would pick); M=512,
// N=4096 SwiGLU runs BNH=112 (74 tiles, one wave).
constexpr std::uint64_t kKBlockFloor = 1365;
constexpr int kNarrowMaxKBlocks = 16;

int choose_bnh(int mblocks, std::uint64_t n, bool swiglu, int sm_count, int max_bnh,
               bool with112, bool with32, std::uint64_t* cost_out = nullptr) {
  constexpr int kCandidates[] = {128, 112, 96, 64, 32};
  int best = 64;
  std::uint64_t best_cost = ~0ull;
  for (int bnh : kCandidates) {
    if (bnh > max_bnh || (bnh == 112 && !with112) || (bnh == 32 && !with32)) continue;
    const std::uint64_t cols = swiglu ? bnh : 2 * bnh;
    const std::uint64_t tiles = static_cast<std::uint64_t>(mblocks) * ((n + cols - 1) / cols);
    const std::uint64_t waves = (tiles + sm_count - 1) / sm_count;
    const std::uint64_t cost = waves * (kKBlockFloor + 2 * bnh);
    if (cost < best_cost) {
      best_cost = cost;
      best = bnh;
    }
  }
  if (cost_out) *cost_out = best_cost;
  return best;
}

// Split-K cluster path (gemm_sm100_sk.cuh) for GELU-form GEMMs (bias+GELU,
// residual): one 256x256 tile per cluster of two CTA pairs, each pair half of
// K.  Chosen when every tile has a cluster (one wave) and the cost model --
// per-k-block floor as in choose_bnh, half the k-blocks at MMA N = 256, plus
// the partial-accumulator exchange counted as kSkExchangeKBlocks k-blocks --
// beats the best one-pair-per-tile choice.  Needs K long enough to split.
constexpr int kSkMinKBlocks = 16;
constexpr std::uint64_t kSkExchangeKBlocks = 3;

// fp32 emulation (below): k-blocks per flushed accumulation chunk of the a0*b0 segment (512 k): on
// unit-scale data the max error against a float64 GEMM is ~5e-8 of
// sum_k |x||w| at k = 4096, against ~7e-6 with one accumulation per tile.
constexpr int kFlushKBlocks = 8;

// Operands of one tensor-core launch: A [m, a_cols] bf16 (row stride a_cols)
// and the two B maps [b_rows, b_cols] bf16 (SwiGLU: gate and up; GELU: W
// twice).  k_blocks = number of 64-wide k-blocks; seg_* describe a segmented
// K (fp32 emulation, below) or are 0.
struct TcOperands {
  const void* a;
  std::uint64_t a_cols;
  const void* b0;
  const void* b1;
  std::uint64_t b_rows;
  std::uint64_t b_cols;
  int k_blocks;
  int seg_k_blocks;
  std::uint32_t seg_pairs;
};

// Launch the tcgen05 kernel (CTA-pair when there are two or more 128-row
// blocks).  Returns -1 when TMA cannot express the operands.
// FLUSH (fp32 emulation) keeps a tile row's sums in registers, BNH floats a
// thread.  Up to BNH = 96 they fit the 168 registers every thread gets; the
// BNH = 128 kernels move registers from the control warpgroup to the
// epilogue (setmaxnreg), which needs the kernel to have been compiled with
// the full 168 a thread: checked once per kernel here, else BNH stops at 96.
template <typename Kernel>
bool launch_regs_cover_split(Kernel kernel) {
  cudaFuncAttributes attr;
  if (cudaFuncGetAttributes(&attr, kernel) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return attr.numRegs >= col::sm100::kRegsLaunchNeeded;
}

template <int EPI, typename TOut>
bool flush_wide_ok(bool pair) {
  static const bool one = launch_regs_cover_split(col::sm100::gemm_bf16_tc_kernel<128, EPI, TOut, true>);
  static const bool two = launch_regs_cover_split(col::sm100::gemm_bf16_tc2_kernel<128, EPI, TOut, true>);
  return pair ? two : one;
}

// Output placement of the gathering epilogue: row stride `ld` (elements) and
// the peer copies of the output block.
struct GatherOut {
  std::uint64_t ld;
  int num_peers;
  void* peers[col::sm100::kMaxPeers];
};

template <int EPI, typename TOut, bool FLUSH = false>
int launch_tensor_gemm(const TcOperands& ops, BMode mode, const float* bias, void* out,
                       std::uint64_t m, std::uint64_t n, cudaStream_t s,
                       const void* residual = nullptr, const float* row_scale = nullptr,
                       const GatherOut* gather = nullptr) {
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
    if (int rc = set_smem_attr_2sm<128, EPI, TOut, false>(dev)) return rc;
    pair_slots = max_pair_clusters<EPI, TOut>(dev);
  }
  const bool use_pair = pair && pair_slots > 0;
  const int mblocks_sched = use_pair ? (mblocks + 1) / 2 : mblocks;
  int max_bnh = 128;
  if constexpr (FLUSH) max_bnh = flush_wide_ok<EPI, TOut>(use_pair) ? 128 : 96;
  // BNH = 32 (twice the tiles of 64, each with half the B box and half the
  // epilogue) only where a tile's fixed cost outweighs its main loop.
  const bool with32 = !FLUSH && ops.k_blocks <= kNarrowMaxKBlocks;
  std::uint64_t tile_cost = 0;
  const int bnh = choose_bnh(mblocks_sched, n, mode == BMode::kSwiGLU,
                             use_pair ? pair_slots : info.sm_count, max_bnh, !FLUSH, with32,
                             &tile_cost);
  if constexpr (!FLUSH && (EPI == col::sm100::kEpiBiasGeluErf ||
                           EPI == col::sm100::kEpiBiasGeluTanh || EPI == col::sm100::kEpiResidual)) {
    if (use_pair && gather == nullptr && ops.seg_k_blocks == 0 && mode == BMode::kGelu &&
        ops.k_blocks >= kSkMinKBlocks) {
      const std::uint64_t sk_nblocks = (n + 255) / 256;
      const std::uint64_t sk_tiles = static_cast<std::uint64_t>(mblocks_sched) * sk_nblocks;
      const int clusters = sk_clusters<EPI, TOut>(dev);
      const std::uint64_t kb = static_cast<std::uint64_t>(ops.k_blocks);
      const std::uint64_t sk_cost = ((kb + 1) / 2 + kSkExchangeKBlocks) * (kKBlockFloor + 256);
      if (clusters > 0 && sk_tiles <= static_cast<std::uint64_t>(clusters) &&
          sk_cost < tile_cost * kb) {
        GemmParams p;
        std::memset(&p, 0, sizeof(p));
        int rc = encode_bf16_rows(&p.map_a, ops.a, m, ops.a_cols, 128);
        if (rc == 0) rc = encode_bf16_rows(&p.map_b0, ops.b0, ops.b_rows, ops.b_cols, 128);
        if (rc == col::kErrTensorMapEncode) return -1;
        if (rc != 0) return rc;
        p.map_b1 = p.map_b0;
        p.bias = bias;
        p.residual = residual;
        p.out = out;
        p.status = status;
        p.m = static_cast<int>(m);
        p.n = static_cast<int>(n);
        p.k = static_cast<int>(ops.a_cols);
        p.num_m_blocks = mblocks_sched;
        p.num_n_blocks = static_cast<int>(sk_nblocks);
        p.num_k_blocks = ops.k_blocks;
        p.b_row_stride = 256;
        p.b1_row_offset = 128;
        p.out_ld = static_cast<int>(n);
        p.out_vec_ok = col::aligned16(out) && ((n * sizeof(TOut)) % 16 == 0);
        return col::launch_serialised(col::sm100::gemm_bf16_sk_kernel<EPI, TOut>,
                                      dim3(static_cast<unsigned>(4 * sk_tiles)),
                                      dim3(col::sm100::kCtaThreads),
                                      col::sm100::kSkSmemBytes, s, p);
      }
    }
  }

  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  int rc = encode_bf16_rows(&p.map_a, ops.a, m, ops.a_cols, 128);
  if (rc == 0) rc = encode_bf16_rows(&p.map_b0, ops.b0, ops.b_rows, ops.b_cols, bnh);
  if (rc == 0) rc = encode_bf16_rows(&p.map_b1, ops.b1, ops.b_rows, ops.b_cols, bnh);
  if (rc == col::kErrTensorMapEncode) return -1;  // layout TMA cannot express: CUDA cores
  if (rc != 0) return rc;
  p.bias = bias;
  p.residual = residual;
  p.row_scale = row_scale;
  p.out = out;
  p.status = status;
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(ops.a_cols);
  p.num_m_blocks = mblocks_sched;
  p.num_k_blocks = ops.k_blocks;
  p.seg_k_blocks = ops.seg_k_blocks;
  p.seg_pairs = ops.seg_pairs;
  if (mode == BMode::kSwiGLU) {
    p.num_n_blocks = static_cast<int>((n + bnh - 1) / bnh);
    p.b_row_stride = bnh;
    p.b1_row_offset = 0;
  } else {
    p.num_n_blocks = static_cast<int>((n + 2 * bnh - 1) / (2 * bnh));
    p.b_row_stride = 2 * bnh;
    p.b1_row_offset = bnh;
  }
  p.out_ld = static_cast<int>(n);
  p.out_vec_ok = col::aligned16(out) && ((n * sizeof(TOut)) % 16 == 0);
  if (gather != nullptr) {
    p.out_ld = static_cast<int>(gather->ld);
    p.out_vec_ok = col::aligned16(out) && ((gather->ld * sizeof(TOut)) % 16 == 0);
    p.num_peers = gather->num_peers;
    for (int i = 0; i < gather->num_peers; ++i) {
      p.peer_out[i] = gather->peers[i];
      p.out_vec_ok = p.out_vec_ok && col::aligned16(gather->peers[i]);
    }
  }
  p.flush_k_blocks = FLUSH ? kFlushKBlocks : 0;
  if constexpr (FLUSH) {
    if (use_pair) {
      switch (bnh) {
        case 128:
          if ((rc = set_smem_attr_2sm<128, EPI, TOut, true>(dev))) return rc;
          return launch_tc2<128, EPI, TOut, true>(p, s, dev, pair_slots);
        case 96:
          if ((rc = set_smem_attr_2sm<96, EPI, TOut, true>(dev))) return rc;
          return launch_tc2<96, EPI, TOut, true>(p, s, dev, pair_slots);
        default:
          if ((rc = set_smem_attr_2sm<64, EPI, TOut, true>(dev))) return rc;
          return launch_tc2<64, EPI, TOut, true>(p, s, dev, pair_slots);
      }
    }
    switch (bnh) {  // choose_bnh offers 128, 96 and 64 only here
      case 128: return launch_tc<128, EPI, TOut, true>(p, s, dev, info.sm_count);
      case 96: return launch_tc<96, EPI, TOut, true>(p, s, dev, info.sm_count);
      default: return launch_tc<64, EPI, TOut, true>(p, s, dev, info.sm_count);
    }
  } else {
    if (use_pair) {
      switch (bnh) {
        case 128: return launch_tc2<128, EPI, TOut, false>(p, s, dev, pair_slots);
        case 112:
          if ((rc = set_smem_attr_2sm<112, EPI, TOut, false>(dev))) return rc;
          return launch_tc2<112, EPI, TOut, false>(p, s, dev, pair_slots);
        case 96:
          if ((rc = set_smem_attr_2sm<96, EPI, TOut, false>(dev))) return rc;
          return launch_tc2<96, EPI, TOut, false>(p, s, dev, pair_slots);
        case 32:
          if ((rc = set_smem_attr_2sm<32, EPI, TOut, false>(dev))) return rc;
          return launch_tc2<32, EPI, TOut, false>(p, s, dev, pair_slots);
        default:
          if ((rc = set_smem_attr_2sm<64, EPI, TOut, false>(dev))) return rc;
          return launch_tc2<64, EPI, TOut, false>(p, s, dev, pair_slots);
      }
    }
    switch (bnh) {
      case 128: return launch_tc<128, EPI, TOut, false>(p, s, dev, info.sm_count);
      case 112: return launch_tc<112, EPI, TOut, false>(p, s, dev, info.sm_count);
      case 96: return launch_tc<96, EPI, TOut, false>(p, s, dev, info.sm_count);
      case 32: return launch_tc<32, EPI, TOut, false>(p, s, dev, info.sm_count);
      default: return launch_tc<64, EPI, TOut, false>(p, s, dev, info.sm_count);
    }
  }
}

// bf16 operands straight from the caller: x [m, k], w0/w1 [n, k] (kGelu: w0 only).
template <int EPI, typename TOut>
int gemm_bf16_tc(const void* x, const void* w0, const void* w1, BMode mode, const float* bias,
                 void* out, std::uint64_t m, std::uint64_t n, std::uint64_t k, cudaStream_t s,
                 const void* residual = nullptr, const float* row_scale = nullptr,
                 const GatherOut* gather = nullptr) {
  if ((k % 8) != 0 || !col::aligned16(x) || !col::aligned16(w0) ||
      (mode == BMode::kSwiGLU && !col::aligned16(w1))) {
    return -1;
  }
  TcOperands ops{x, k, w0, mode == BMode::kSwiGLU ? w1 : w0, n, k,
                 static_cast<int>((k + col::sm100::kBlockK - 1) / col::sm100::kBlockK), 0, 0u};
  return launch_tensor_gemm<EPI, TOut>(ops, mode, bias, out, m, n, s, residual, row_scale, gather);
}

// ---------------------------------------------------------------- fp32 on tensor cores
//
// An fp32 value a is split into three bf16 parts a = a0 + a1 + a2 + e with
// a0 = bf16(a), a1 = bf16(a - a0), a2 = bf16(a - a0 - a1): 3 x 8 significand
// bits, |e| <= 2^-24 |a|.  A product a.b is then the sum of the six part
// products of total order <= 2 (a0b0, a0b1, a1b0, a1b1, a0b2, a2b0); the
// three dropped ones are ~2^-23 |a||b|, the size of fp32 rounding.  bf16 x
// bf16 products are exact in the tensor core's fp32 accumulator, so the GEMM
// keeps fp32 accuracy while running on tcgen05: the parts are laid out side
// by side along K ([a0 | a1 | a2], each part padded to a multiple of 64) and
// one launch walks the six (A part, B part) segments.
constexpr int kSplitSegments = 6;
constexpr std::uint32_t kSplitPairs =
    (0u << 0) | (0u << 2) |    // a0 b0
    (0u << 4) | (1u << 6) |    // a0 b1
    (1u << 8) | (0u << 10) |   // a1 b0
    (1u << 12) | (1u << 14) |  // a1 b1
    (0u << 16) | (2u << 18) |  // a0 b2
    (2u << 20) | (0u << 22);   // a2 b0

__global__ void __launch_bounds__(256)
split_fp32_bf16x3_kernel(const float* __restrict__ src, std::uint64_t rows, std::uint32_t k,
                         std::uint32_t kp, __nv_bfloat16* __restrict__ dst) {
  col::grid_dependency_wait();
  // One thread per 8 consecutive k of one row: three 16-byte stores.
  const std::uint64_t groups_per_row = kp / 8;
  const std::uint64_t total = rows * groups_per_row;
  for (std::uint64_t gi = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       gi < total; gi += static_cast<std::uint64_t>(gridDim.x) * blockDim.x) {
    const std::uint64_t r = gi / groups_per_row;
    const std::uint32_t k0 = static_cast<std::uint32_t>(gi - r * groups_per_row) * 8;
    const float* row = src + r * k;
    float p0[8], p1[8], p2[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = (k0 + j < k) ? __ldg(row + k0 + j) : 0.0f;
      const float h = col::bf16_round(v);
      const float r1 = v - h;
      const float m = col::bf16_round(r1);
      p0[j] = h;
      p1[j] = m;
      p2[j] = r1 - m;
    }
    uint4* out = reinterpret_cast<uint4*>(dst + r * (3ull * kp) + k0);
    out[0] = col::pack_bf16x8(p0);
    out[kp / 8] = col::pack_bf16x8(p1);
    out[2 * (kp / 8)] = col::pack_bf16x8(p2);
  }
}

int split_fp32(const float* src, std::uint64_t rows, std::uint64_t k, std::uint64_t kp,
               __nv_bfloat16* dst, cudaStream_t s) {
  const std::uint64_t work = rows * (kp / 8);
  std::uint64_t blocks = (work + 255) / 256;
  const std::uint64_t cap = static_cast<std::uint64_t>(col::device_info().sm_count) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks == 0) blocks = 1;
  return col::launch_serialised(split_fp32_bf16x3_kernel, dim3(static_cast<unsigned>(blocks)),
                                dim3(256), 0, s, src, rows, static_cast<std::uint32_t>(k),
                                static_cast<std::uint32_t>(kp), dst);
}

// fp32 GEMM with fused epilogue on tensor cores.  kSwiGLU: w0/w1 are the gate
// and up matrices [n, k] (for a packed weight, its two halves); kGelu: w0 is
// W [n, k].  Scratch (the bf16 parts, 6 bytes per input element) comes from
// the library's stream-ordered pool.  Returns -1 to request the CUDA-core path.
template <int EPI>
int gemm_fp32_tc(const float* x, const float* w0, const float* w1, BMode mode, const float* bias,
                 float* out, std::uint64_t m, std::uint64_t n, std::uint64_t k, cudaStream_t s) {
  if (col::device_info().cc_major != 10) return -1;
  // Tiny problems: the split passes and the launch overheads would dominate.
  if (static_cast<double>(m) * static_cast<double>(n) * static_cast<double>(k) < 4.0e6) return -1;
  const std::uint64_t kp = (k + col::sm100::kBlockK - 1) / col::sm100::kBlockK * col::sm100::kBlockK;
  const std::uint64_t b_rows = mode == BMode::kSwiGLU ? 2 * n : n;
  const std::size_t a_bytes = static_cast<std::size_t>(m) * 3 * kp * 2;
  const std::size_t b_bytes = static_cast<std::size_t>(b_rows) * 3 * kp * 2;
  void* scratch = nullptr;
  if (col::scratch_alloc(&scratch, a_bytes + b_bytes, s) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  __nv_bfloat16* a3 = static_cast<__nv_bfloat16*>(scratch);
  __nv_bfloat16* b3 = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(scratch) + a_bytes);
  int rc = split_fp32(x, m, k, kp, a3, s);
  if (rc == 0) rc = split_fp32(w0, n, k, kp, b3, s);
  if (rc == 0 && mode == BMode::kSwiGLU) rc = split_fp32(w1, n, k, kp, b3 + n * 3 * kp, s);
  if (rc == 0) {
    const int seg_kb = static_cast<int>(kp / col::sm100::kBlockK);
    TcOperands ops{a3, 3 * kp, b3, mode == BMode::kSwiGLU ? b3 + n * 3 * kp : b3, n, 3 * kp,
                   kSplitSegments * seg_kb, seg_kb, kSplitPairs};
    rc = launch_tensor_gemm<EPI, float, true>(ops, mode, bias, out, m, n, s);
  }
  const cudaError_t fe = cudaFreeAsync(scratch, s);
  if (rc == 0 && fe != cudaSuccess) rc = static_cast<int>(fe);
  return rc;
}

template <typename TIn, int EPI, typename TOut>
int gemm_simt(const void* x, const void* w0, const void* w1, const float* bias, void* out,
              std::uint64_t m, std::uint64_t n, std::uint64_t k, cudaStream_t s,
              const void* residual = nullptr, const float* row_scale = nullptr) {
  col::simt::SimtParams p{x,        w0,  w1,
                          bias,     residual, row_scale,
                          out,      static_cast<int>(m), static_cast<int>(n),
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
  const cudaStream_t s = col::as_stream(stream);
  const int rc = gemm_fp32_tc<col::sm100::kEpiSwiGLU>(x, wg, wu, BMode::kSwiGLU, nullptr, out, m,
                                                      n, k, s);
  if (rc != -1) return rc;
  return gemm_simt<float, col::sm100::kEpiSwiGLU, float>(x, wg, wu, nullptr, out, m, n, k, s);
}

// gemm_swiglu.cu:335-351: packed [2N, K]; n above INT32_MAX / 2 is invalid.
int swiglu_f32_packed(const float* x, const float* w, const float* ws, float* out, std::uint64_t m,
                      std::uint64_t k, std::uint64_t n, void* stream) {
  if (m == 0 || n == 0) return 0;
  if (!x || !w || !ws || !out || !dims_ok(m, n, k, 0x7fffffffull / 2)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const cudaStream_t s = col::as_stream(stream);
  const float* wu = static_cast<const float*>(up_half(w, n, k, sizeof(float)));
  const int rc = gemm_fp32_tc<col::sm100::kEpiSwiGLU>(x, w, wu, BMode::kSwiGLU, nullptr, out, m,
                                                      n, k, s);
  if (rc != -1) return rc;
  return gemm_simt<float, col::sm100::kEpiSwiGLU, float>(x, w, wu, nullptr, out, m, n, k, s);
}

template <int EPI>
int bias_gelu_f32(const float* x, const float* w, const float* b, float* out, std::uint64_t m,
                  std::uint64_t k, std::uint64_t n, void* stream) {
  // gemm_bias_gelu.cu:830-849.
  if (m == 0 || n == 0) return 0;
  if (!x || !w || !b || !out || !dims_ok(m, n, k, 0x7fffffffull)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const cudaStream_t s = col::as_stream(stream);
  const int rc = gemm_fp32_tc<EPI>(x, w, nullptr, BMode::kGelu, b, out, m, n, k, s);
  if (rc != -1) return rc;
  return gemm_simt<float, EPI, float>(x, w, nullptr, b, out, m, n, k, s);
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

// Down projection with the residual add fused (no reference counterpart):
// out[m, n] = bf16(x[m, :] . w[n, :] + residual[m, n]), fp32 accumulation,
// bf16 x [M, K], W [N, K], residual and out [M, N].  out may be the residual
// buffer itself (each element is read before it is written, by the same
// thread).  m == 0 or n == 0 succeeds first; NULL, k == 0 or sizes above
// INT32_MAX are invalid.
COL_API int cuda_operator_gemm_residual_bf16(const void* input_bf16, const void* weight_bf16,
                                             const void* residual_bf16, void* output_bf16,
                                             uint64_t m, uint64_t k, uint64_t n, void* stream) {
  if (m == 0 || n == 0) return 0;
  if (!input_bf16 || !weight_bf16 || !residual_bf16 || !output_bf16 ||
      !dims_ok(m, n, k, 0x7fffffffull)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const cudaStream_t s = col::as_stream(stream);
  // The vector residual loads share the output's alignment test.
  const bool same_alignment =
      (reinterpret_cast<std::uintptr_t>(residual_bf16) & 15u) ==
      (reinterpret_cast<std::uintptr_t>(output_bf16) & 15u);
  int rc = -1;
  if (same_alignment) {
    rc = gemm_bf16_tc<col::sm100::kEpiResidual, __nv_bfloat16>(
        input_bf16, weight_bf16, nullptr, BMode::kGelu, nullptr, output_bf16, m, n, k, s,
        residual_bf16);
  }
  if (rc != -1) return rc;
  return gemm_simt<__nv_bfloat16, col::sm100::kEpiResidual, __nv_bfloat16>(
      input_bf16, weight_bf16, nullptr, nullptr, output_bf16, m, n, k, s, residual_bf16);
}

// Packed GEMM + SwiGLU with the RMSNorm of x folded in (no reference
// counterpart): out[m, j] = bf16(silu(rs[m] * g) * (rs[m] * u)) where g and u
// are the fp32-accumulated products of the raw bf16 x with the packed weight,
// whose columns the caller has already multiplied by the RMSNorm weight, and
// rs[m] = rsqrt(mean(x[m]^2) + eps) (cuda_operator_rmsnorm_rstd_bf16).  Since
// (x * rs * w) . W^T = rs * (x . (W * w)^T), this is the RMSNorm -> GEMM+SwiGLU
// block without writing or re-reading the normalised activations.
COL_API int cuda_operator_gemm_swiglu_rowscale_bf16(const void* input_bf16, const float* row_scale,
                                                    const void* packed_weight_bf16,
                                                    void* output_bf16, uint64_t m, uint64_t k,
                                                    uint64_t n, void* stream) {
  if (m == 0 || n == 0) return 0;
  if (!input_bf16 || !row_scale || !packed_weight_bf16 || !output_bf16 ||
      !dims_ok(m, n, k, 0x7fffffffull / 2)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const cudaStream_t s = col::as_stream(stream);
  const void* wu = up_half(packed_weight_bf16, n, k, 2);
  const int rc = gemm_bf16_tc<col::sm100::kEpiSwiGLURowScale, __nv_bfloat16>(
      input_bf16, packed_weight_bf16, wu, BMode::kSwiGLU, nullptr, output_bf16, m, n, k, s, nullptr,
      row_scale);
  if (rc != -1) return rc;
  return gemm_simt<__nv_bfloat16, col::sm100::kEpiSwiGLURowScale, __nv_bfloat16>(
      input_bf16, packed_weight_bf16, wu, nullptr, output_bf16, m, n, k, s, nullptr, row_scale);
}

// N-sharded packed GEMM + SwiGLU whose epilogue also all-gathers the output
// over NVLink (no reference counterpart).  Rank r of g computes its [m, n]
// column block (packed_weight_bf16 = its [2n, K] shard, row_scale as in
// cuda_operator_gemm_swiglu_rowscale_bf16, or null for plain SwiGLU) and
// stores it into each of the `num_dests` destinations: dests[0] is the
// block's place in this GPU's [m, ld] output, dests[1..] the same place in the
// other ranks' outputs, mapped into this process (cuda_operator_lab_peer_open).
// The tensor-core path only: operands TMA cannot take (k not a multiple of 8,
// unaligned x or weight) return 10005.
COL_API int cuda_operator_gemm_swiglu_allgather_bf16(const void* input_bf16, const float* row_scale,
                                                     const void* packed_weight_bf16,
                                                     void* const* dests, int num_dests,
                                                     uint64_t m, uint64_t k, uint64_t n,
                                                     uint64_t ld, void* stream) {
  if (m == 0 || n == 0) return 0;
  if (!input_bf16 || !packed_weight_bf16 || !dests || num_dests < 1 ||
      num_dests > col::sm100::kMaxPeers + 1 || ld < n || !dims_ok(m, n, k, 0x7fffffffull / 2) ||
      ld > 0x7fffffffull) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  GatherOut g;
  std::memset(&g, 0, sizeof(g));
  g.ld = ld;
  g.num_peers = num_dests - 1;
  for (int i = 0; i < num_dests; ++i) {
    if (dests[i] == nullptr) return static_cast<int>(cudaErrorInvalidValue);
    if (i > 0) g.peers[i - 1] = dests[i];
  }
  const cudaStream_t s = col::as_stream(stream);
  const void* wu = up_half(packed_weight_bf16, n, k, 2);
  const int rc = gemm_bf16_tc<col::sm100::kEpiSwiGLUGather, __nv_bfloat16>(
      input_bf16, packed_weight_bf16, wu, BMode::kSwiGLU, nullptr, dests[0], m, n, k, s, nullptr,
      row_scale, &g);
  return rc == -1 ? col::kErrGatherLayout : rc;
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
