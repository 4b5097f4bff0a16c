// Blackwell (sm_100a) tensor-core GEMM with fused SwiGLU / bias+GELU
// epilogues: D[M, N'] = X[M, K] . B[N', K]^T, bf16 operands, fp32 accumulate.
//
// Persistent, warp-specialised CTA (384 threads, one CTA per SM):
//   warp 0      TMA producer: one thread streams 128x64 X tiles and two
//               BNHx64 B boxes per k-block into a STAGES-deep smem ring
//               (128-byte swizzle, completion counted on an mbarrier);
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=2*BNH,
//               K=16) from the smem descriptors into a TMEM accumulator and
//               releases ring slots with tcgen05.commit;
//   warp 2      allocates/frees the TMEM columns;
//   warps 4..11 epilogue: tcgen05.ld the accumulator (one row per thread,
//               two warps per TMEM lane quarter splitting the columns),
//               apply silu(g)*u or gelu(acc+bias) in registers, store once.
// Two TMEM accumulators alternate between tiles, so the epilogue of tile i
// overlaps the main loop of tile i+1.
//
// SwiGLU pairing: the B stage holds the gate box (rows n0..n0+BNH of Wg) and
// the up box (the same rows of Wu) back to back, so one MMA of N = 2*BNH puts
// gate columns in accumulator columns [0, BNH) and up columns in [BNH, 2*BNH).
// For bias+GELU both boxes come from W (rows n0.. and n0+BNH..), giving 2*BNH
// output columns per tile.
//
// Every mbarrier wait is bounded (kWaitLimitNs); on timeout the waiting
// thread ORs a code into the device status word, raises a CTA-wide abort
// flag that the other roles poll, and all roles drain in-flight copies and
// MMAs (again with bounded waits) before TMEM is freed and the CTA exits.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "common.cuh"

namespace col {
namespace sm100 {

enum Epilogue : int {
  kEpiSwiGLU = 0,           // out = silu(g) * u
  kEpiSwiGLURoundBf16 = 1,  // g, u rounded to bf16 first (bf16 GEMM workspace semantics)
  kEpiBiasGeluErf = 2,      // out = gelu_erf(acc + bias[n])
  kEpiBiasGeluTanh = 3,     // out = gelu_tanh(acc + bias[n])
  kEpiResidual = 4,         // out = acc + residual[m, n] (bf16 residual, down projection)
  kEpiSwiGLURowScale = 5,   // g, u scaled by row_scale[m] first (RMSNorm folded into the GEMM)
  kEpiSwiGLUGather = 6,     // as kEpiSwiGLURowScale (no scale when row_scale is null); every
                            // output row run is also stored to each peer_out (column all-gather)
};

// Peer destinations of the gathering epilogue (an 8-GPU NVLink domain).
constexpr int kMaxPeers = 7;

constexpr int kBlockM = 128;
constexpr int kBlockK = 64;  // bf16 elements per k-block: one 128-byte swizzle row
constexpr int kGroupM = 16;  // m-blocks per rasterisation group (L2 reuse of B)
constexpr int kEpiWarps = 8;       // warps 4..11: two per TMEM lane quarter
constexpr int kEpiGroups = kEpiWarps / 4;
constexpr int kCtaThreads = 128 + 32 * kEpiWarps;  // producer, MMA, TMEM, idle + epilogue
// The gathering epilogue stages each warp's 32 rows x up to 64 output columns
// (bf16, 128 bytes a row) in shared memory so that its stores to other GPUs
// go out as whole 128-byte row runs.
constexpr uint32_t kGatherRowBytes = 128;
constexpr uint32_t kGatherWarpBytes = 32 * kGatherRowBytes;
constexpr uint32_t epi_smem_reserve(int epi) {
  return epi == kEpiSwiGLUGather ? kEpiWarps * kGatherWarpBytes : 0u;
}
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// Status bits written on a bounded-wait timeout.
constexpr unsigned kStatusProducer = 1u;
constexpr unsigned kStatusMma = 2u;
constexpr unsigned kStatusEpilogue = 4u;
constexpr unsigned kStatusDrain = 8u;

struct __align__(64) GemmParams {
  CUtensorMap map_a;   // X [M, K]
  CUtensorMap map_b0;  // gate rows (SwiGLU) or W rows (GELU)
  CUtensorMap map_b1;  // up rows (SwiGLU) or W rows (GELU)
  const float* bias;
  const void* residual;  // kEpiResidual: bf16 [m, n], row stride out_ld (may equal out)
  const float* row_scale;  // kEpiSwiGLURowScale: fp32 [m]
  void* out;
  unsigned* status;
  int m;
  int n;  // output columns
  int k;
  int num_m_blocks;
  int num_n_blocks;
  int num_k_blocks;
  int b_row_stride;   // B rows advanced per n-block (box 0)
  int b1_row_offset;  // box-1 row relative to box 0
  int out_ld;         // output row stride in elements
  int out_vec_ok;     // 16-byte vector stores allowed
  // Segmented K (fp32 operands split into bf16 parts, see gemm.cu): when
  // seg_k_blocks > 0 the k-loop runs over num_k_blocks = segments *
  // seg_k_blocks blocks; segment s reads A from part (seg_pairs >> 4s) & 3
  // and B from part (seg_pairs >> (4s + 2)) & 3, each part seg_k_blocks wide.
  int seg_k_blocks;
  uint32_t seg_pairs;
  int flush_k_blocks;  // fp32 emulation: k-blocks per flushed chunk of segment 0
  // kEpiSwiGLUGather: the same [m, n] block (row stride out_ld) in the output
  // buffers of other GPUs, mapped into this process (peer stores over NVLink).
  int num_peers;
  void* peer_out[kMaxPeers];
};

// Column (x) coordinates of k-block kb in A and in B.
__device__ __forceinline__ void k_block_coords(const GemmParams& p, int kb, int& ax, int& bx) {
  if (p.seg_k_blocks == 0) {
    ax = bx = kb * kBlockK;
    return;
  }
  const int seg = kb / p.seg_k_blocks;
  const int local = kb - seg * p.seg_k_blocks;
  const int a_part = static_cast<int>((p.seg_pairs >> (4 * seg)) & 3u);
  const int b_part = static_cast<int>((p.seg_pairs >> (4 * seg + 2)) & 3u);
  ax = (a_part * p.seg_k_blocks + local) * kBlockK;
  bx = (b_part * p.seg_k_blocks + local) * kBlockK;
}

// Accumulation chunks of one tile.  The tensor core's fp32 accumulator adds
// each K=16 step's products with truncation, so over thousands of k its
// error grows to ~1e-5 of sum|a||b| -- harmless for bf16 outputs, too much for
// the fp32 GEMMs.  With FLUSH the K loop is cut into chunks: segment 0 (the
// a0*b0 products, the large ones) in chunks of flush_k_blocks k-blocks, then
// one chunk for the remaining (2^-8 smaller) segments.  Each chunk restarts
// the TMEM accumulator and the epilogue adds the chunk sums in registers with
// round-to-nearest fp32 adds, which brings the error under fp32 rounding size.
template <bool FLUSH>
__device__ __forceinline__ int tile_chunks(const GemmParams& p) {
  if constexpr (!FLUSH) {
    return 1;
  } else {
    const int head = (p.seg_k_blocks + p.flush_k_blocks - 1) / p.flush_k_blocks;
    return head + (p.num_k_blocks > p.seg_k_blocks ? 1 : 0);
  }
}

template <bool FLUSH>
__device__ __forceinline__ void chunk_range(const GemmParams& p, int c, int& kb0, int& kb1) {
  if constexpr (!FLUSH) {
    kb0 = 0;
    kb1 = p.num_k_blocks;
  } else {
    const int head = (p.seg_k_blocks + p.flush_k_blocks - 1) / p.flush_k_blocks;
    if (c < head) {
      kb0 = c * p.flush_k_blocks;
      kb1 = min(kb0 + p.flush_k_blocks, p.seg_k_blocks);
    } else {
      kb0 = p.seg_k_blocks;
      kb1 = p.num_k_blocks;
    }
  }
}

constexpr uint32_t kSmemLimit = 232448;  // max dynamic shared memory per CTA on sm_100

__host__ __device__ constexpr uint32_t pow2_at_least(uint32_t v) {
  uint32_t p = 32;
  while (p < v) p <<= 1;
  return p;
}

// BNH = rows of each B box (gate/up half, or half of the GELU tile); the MMA
// is M=128 x N=2*BNH.  BNH must keep the box a whole number of 1024-byte
// swizzle atoms (BNH % 8 == 0) and 2*BNH a multiple of 16 in [16, 256].
// KPS = k-blocks per pipeline stage: the producer/MMA handshake of a stage
// (barrier wait, commit) costs ~0.13 us that does not overlap the MMAs
// (measured), so stages of two k-blocks halve it per k-block; the FLUSH
// kernels keep one k-block per stage (their chunk boundaries).
// RESERVE = shared memory the epilogue keeps for itself (the gathering
// epilogue's staging tiles), taken from the ring.
template <int BNH, int KPS = 1, uint32_t RESERVE = 0>
struct TileCfg {
  static_assert(BNH % 16 == 0 && BNH >= 32 && BNH <= 128, "unsupported B box height");
  static_assert(KPS == 1 || KPS == 2, "one or two k-blocks per stage");
  static constexpr int kMmaN = 2 * BNH;
  static constexpr uint32_t kABytes = kBlockM * kBlockK * 2;
  static constexpr uint32_t kBBytes = kMmaN * kBlockK * 2;
  static constexpr uint32_t kKBlockBytes = kABytes + kBBytes;  // [A | B] of one k-block
  static constexpr uint32_t kStageBytes = KPS * kKBlockBytes;
  static constexpr uint32_t kBarrierBytes = 256;
  static constexpr int kStagesFit =
      static_cast<int>((kSmemLimit - 1024 - kBarrierBytes - RESERVE) / kStageBytes);
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr uint32_t kAccStride = pow2_at_least(kMmaN);  // TMEM columns per accumulator
  static constexpr uint32_t kTmemCols = 2 * kAccStride;
  static constexpr uint32_t kEpiSmemOffset = kStages * kStageBytes + kBarrierBytes;
  static constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024 + kBarrierBytes + RESERVE;
  static_assert(kTmemCols <= 512, "two accumulators must fit in TMEM");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
};

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait: true when the phase of `parity` completed; false after the
// time limit or when another role raised the abort flag.
// The clock is first read only after 64 failed polls, so short waits (the
// common case) never pay for a %globaltimer read.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  uint64_t t0 = 0;
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u) {
      if (*abort_flag) return false;
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        return false;
      }
    }
  }
}

// Epilogue-side wait on an accumulator barrier.  Lane 0 alone polls,
// sleeping kEpiPollSleepNs between polls, then the warp agrees: the epilogue
// waits on whole tiles, so waking ~0.1 us late costs nothing, while 256
// threads polling would take shared-memory and issue slots from the TMA and
// MMA threads that share their SM sub-partitions.  __syncwarp orders the
// other lanes after lane 0's acquire.  Same time limit as mbar_wait.
constexpr unsigned kEpiPollSleepNs = 64;

__device__ __forceinline__ bool epi_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                         int lane) {
  int got = 0;
  if (lane == 0) {
    uint64_t t0 = 0;
    for (uint32_t i = 1;; ++i) {
      if (mbar_try_wait(bar, parity)) {
        got = 1;
        break;
      }
      if (kEpiPollSleepNs) __nanosleep(kEpiPollSleepNs);
      if ((i & 15u) == 0u) {
        if (*abort_flag) break;
        const uint64_t now = globaltimer_ns();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > kWaitLimitNs) {
          break;
        }
      }
    }
  }
  __syncwarp();
  return __shfl_sync(0xffffffffu, got, 0) != 0;
}

// Bounded wait that ignores the abort flag (used while draining).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 63u && globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Register split between warpgroups (setmaxnreg, whole warpgroup, aligned):
// used by the FLUSH kernels with BNH = 128, whose epilogue holds 128 running
// sums per thread.  Warpgroup 0 (producer, MMA, TMEM, idle warps) gives up
// registers, the two epilogue warpgroups take them.  The shares must fit the
// registers the CTA was launched with: 128 x kRegsControl + 256 x kRegsEpilogue
// = 62464 <= 384 x 168 (the host checks the compiled count before launching).
constexpr int kRegsControl = 56;
constexpr int kRegsEpilogue = 216;
constexpr int kRegsLaunchNeeded = (128 * kRegsControl + 32 * kEpiWarps * kRegsEpilogue + kCtaThreads - 1) / kCtaThreads;

template <int N>
__device__ __forceinline__ void regs_release() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_acquire() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// Named CTA barriers (barrier 0 is __syncthreads): arrive without waiting,
// and arrive-and-wait, for `count` threads (a multiple of 32).
constexpr int kStartBarrier = 1;

__device__ __forceinline__ void named_barrier_arrive(int id, int count) {
  asm volatile("barrier.cta.arrive.aligned %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_barrier_sync(int id, int count) {
  asm volatile("barrier.cta.sync.aligned %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t holder, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the
// 128-byte swizzle: 8-row core groups 1024 bytes apart (SBO), leading offset
// unused for swizzled K-major tiles (encoded as 16 bytes), version 1, layout
// SWIZZLE_128B (2).  Tile bases are 1024-byte aligned.
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor, kind::f16: D fp32, A and B bf16, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane; the
// wait is in the same asm block so no use of r[] can be scheduled before the
// asynchronous load has landed.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Two 16-column loads (e.g. the gate and the up columns of one output chunk)
// completed by one wait.
__device__ __forceinline__ void tmem_ld16x2(uint32_t ta, uint32_t tb, uint32_t (&a)[16],
                                            uint32_t (&b)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]),
        "=r"(a[7]), "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]),
        "=r"(a[14]), "=r"(a[15]), "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]),
        "=r"(b[5]), "=r"(b[6]), "=r"(b[7]), "=r"(b[8]), "=r"(b[9]), "=r"(b[10]), "=r"(b[11]),
        "=r"(b[12]), "=r"(b[13]), "=r"(b[14]), "=r"(b[15])
      : "r"(ta), "r"(tb)
      : "memory");
}

template <int W>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[W]) {
  if constexpr (W == 32) {
    tmem_ld32(taddr, r);
  } else {
    static_assert(W == 16, "chunk width");
    tmem_ld16(taddr, r);
  }
}

// ------------------------------------------------------------ tile schedule

__device__ __forceinline__ void tile_coords(int tile, const GemmParams& p, int& mb, int& nb) {
  const int group_tiles = kGroupM * p.num_n_blocks;
  const int group = tile / group_tiles;
  const int first_m = group * kGroupM;
  const int rows = min(p.num_m_blocks - first_m, kGroupM);
  const int in_group = tile - group * group_tiles;
  mb = first_m + in_group % rows;
  nb = in_group / rows;
}

// ------------------------------------------------------------ epilogue store

template <typename TOut, int W>
__device__ __forceinline__ void store_chunk(const GemmParams& p, int row, int col0,
                                            const float (&o)[W]) {
  if (row >= p.m) return;
  TOut* dst = static_cast<TOut*>(p.out) + static_cast<std::size_t>(row) * p.out_ld + col0;
  if (p.out_vec_ok && col0 + W <= p.n) {
    if constexpr (sizeof(TOut) == 4) {
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int j = 0; j < W / 4; ++j) {
        __stcs(d4 + j, make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]));
      }
    } else {
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int j = 0; j < W / 8; ++j) {
        uint4 v;
        v.x = pack_bf16x2(o[8 * j + 0], o[8 * j + 1]);
        v.y = pack_bf16x2(o[8 * j + 2], o[8 * j + 3]);
        v.z = pack_bf16x2(o[8 * j + 4], o[8 * j + 5]);
        v.w = pack_bf16x2(o[8 * j + 6], o[8 * j + 7]);
        __stcs(d4 + j, v);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < W; ++j) {
      if (col0 + j < p.n) {
        if constexpr (sizeof(TOut) == 4) {
          dst[j] = o[j];
        } else {
          dst[j] = __float2bfloat16_rn(o[j]);
        }
      }
    }
  }
}

// ------------------------------------------------------------ epilogue

// 16 residual values (bf16) of row `row` from column col0, zero outside the
// matrix; two 16-byte loads when the row is fully in range and aligned (the
// same condition as the vector output store).
__device__ __forceinline__ void load_residual16(const GemmParams& p, int row, int col0,
                                                float (&r)[16]) {
  if (row >= p.m) {
#pragma unroll
    for (int j = 0; j < 16; ++j) r[j] = 0.0f;
    return;
  }
  const __nv_bfloat16* src =
      static_cast<const __nv_bfloat16*>(p.residual) + static_cast<std::size_t>(row) * p.out_ld + col0;
  if (p.out_vec_ok && col0 + 16 <= p.n) {
    float lo[8], hi[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(src), lo);
    unpack_bf16x8(*reinterpret_cast<const uint4*>(src + 8), hi);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      r[j] = lo[j];
      r[8 + j] = hi[j];
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) r[j] = col0 + j < p.n ? __bfloat162float(src[j]) : 0.0f;
  }
}

// One accumulator tile, this thread's TMEM lane (one output row): 16-column
// chunks dealt round-robin to the kEpiGroups warps that share the lane
// quarter.  SwiGLU: gate at accumulator column c, up at BNH + c, output
// column nb*BNH + c.  GELU: accumulator column c is output nb*2*BNH + c.
template <int BNH, int EPI, typename TOut>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, int row, int nb, uint32_t t_row,
                                              int group) {
  if constexpr (EPI == kEpiSwiGLU || EPI == kEpiSwiGLURoundBf16 || EPI == kEpiSwiGLURowScale) {
    const int col_base = nb * BNH;
    float rs = 1.0f;
    if constexpr (EPI == kEpiSwiGLURowScale) rs = row < p.m ? __ldg(p.row_scale + row) : 0.0f;
#pragma unroll 1
    for (int c = group * 16; c < BNH; c += 16 * kEpiGroups) {
      uint32_t g[16], u[16];
      tmem_ld16x2(t_row + c, t_row + BNH + c, g, u);
      float o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float gv = __uint_as_float(g[j]);
        float uv = __uint_as_float(u[j]);
        if constexpr (EPI == kEpiSwiGLURoundBf16) {
          gv = bf16_round(gv);
          uv = bf16_round(uv);
        } else if constexpr (EPI == kEpiSwiGLURowScale) {
          gv *= rs;
          uv *= rs;
        }
        o[j] = silu_fast(gv) * uv;
      }
      store_chunk<TOut, 16>(p, row, col_base + c, o);
    }
  } else if constexpr (EPI == kEpiResidual) {
    const int col_base = nb * 2 * BNH;
#pragma unroll 1
    for (int c = group * 16; c < 2 * BNH; c += 16 * kEpiGroups) {
      uint32_t a[16];
      tmem_ld16(t_row + c, a);
      float res[16];
      load_residual16(p, row, col_base + c, res);
      float o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = __uint_as_float(a[j]) + res[j];
      store_chunk<TOut, 16>(p, row, col_base + c, o);
    }
  } else {
    const int col_base = nb * 2 * BNH;
#pragma unroll 1
    for (int c = group * 16; c < 2 * BNH; c += 16 * kEpiGroups) {
      uint32_t a[16];
      tmem_ld16(t_row + c, a);
      float o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int colj = col_base + c + j;
        const float bv = colj < p.n ? __ldg(p.bias + colj) : 0.0f;
        const float z = __uint_as_float(a[j]) + bv;
        if constexpr (EPI == kEpiBiasGeluErf) {
          o[j] = gelu_erf_f(z);
        } else {
          o[j] = gelu_tanh_f(z);
        }
      }
      store_chunk<TOut, 16>(p, row, col_base + c, o);
    }
  }
}

// ------------------------------------------------------------ gathering epilogue
//
// kEpiSwiGLUGather: the two warps of a TMEM lane quarter split a tile's BNH
// output columns into contiguous parts (group 0 the first ceil(BNH/32)
// 16-column chunks, group 1 the rest; at most 64 columns).  A warp computes
// its part of its 32 rows, stores it to this GPU's output and into its
// staging tile (row r at r * 128 bytes, 16-byte segment s in slot s ^ (r & 7),
// so neither the row-wise writes nor the segment-wise reads conflict on
// banks), releases the accumulator, and then sends the staging tile to every
// peer output with 8 lanes per row: one store instruction moves four whole
// 128-byte row runs over NVLink instead of 32 separate 16-byte pieces.

template <int BNH>
struct GatherSplit {
  static constexpr int kChunks = BNH / 16;
  static constexpr int kChunks0 = (kChunks + 1) / 2;
  static_assert(kChunks0 * 16 * 2 <= static_cast<int>(kGatherRowBytes), "staging row too short");
  __device__ __forceinline__ static int first(int group) { return group == 0 ? 0 : kChunks0; }
  __device__ __forceinline__ static int last(int group) { return group == 0 ? kChunks0 : kChunks; }
};

template <int BNH>
__device__ __forceinline__ void epilogue_gather_local(const GemmParams& p, int row, int nb,
                                                      uint32_t t_row, int group, int lane,
                                                      uint8_t* stage) {
  using Split = GatherSplit<BNH>;
  const int c0 = Split::first(group);
  const int c1 = Split::last(group);
  const int col_base = nb * BNH;
  float rs = 1.0f;
  if (p.row_scale != nullptr) rs = row < p.m ? __ldg(p.row_scale + row) : 0.0f;
  uint8_t* my_row = stage + lane * kGatherRowBytes;
#pragma unroll 1
  for (int ci = c0; ci < c1; ++ci) {
    const int c = ci * 16;
    uint32_t g[16], u[16];
    tmem_ld16x2(t_row + c, t_row + BNH + c, g, u);
    float o[16], lo[8], hi[8];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      // rs = 1 multiplies exactly: the same bits as the unscaled epilogue
      o[j] = silu_fast(__uint_as_float(g[j]) * rs) * (__uint_as_float(u[j]) * rs);
    }
    store_chunk<__nv_bfloat16, 16>(p, row, col_base + c, o);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      lo[j] = o[j];
      hi[j] = o[8 + j];
    }
    const int seg = 2 * (ci - c0);
    *reinterpret_cast<uint4*>(my_row + ((seg ^ (lane & 7)) << 4)) = pack_bf16x8(lo);
    *reinterpret_cast<uint4*>(my_row + (((seg + 1) ^ (lane & 7)) << 4)) = pack_bf16x8(hi);
  }
}

// Sends a warp's staging tile (rows row0.., its column part of n-block nb)
// to every peer output.  Call after __syncwarp() following the local part.
template <int BNH>
__device__ __forceinline__ void epilogue_gather_peers(const GemmParams& p, int row0, int nb,
                                                      int group, int lane, const uint8_t* stage) {
  using Split = GatherSplit<BNH>;
  if (p.num_peers == 0) return;
  const int c0 = Split::first(group);
  const int segs = 2 * (Split::last(group) - c0);
  const int col0 = nb * BNH + c0 * 16;
#pragma unroll 1
  for (int idx = lane; idx < 32 * segs; idx += 32) {
    const int r = idx / segs;
    const int sg = idx - r * segs;
    const int grow = row0 + r;
    const int gcol = col0 + sg * 8;
    if (grow >= p.m || gcol >= p.n) continue;
    const uint4 v = *reinterpret_cast<const uint4*>(stage + r * kGatherRowBytes + ((sg ^ (r & 7)) << 4));
    const std::size_t off = static_cast<std::size_t>(grow) * p.out_ld + gcol;
    if (p.out_vec_ok && gcol + 8 <= p.n) {
#pragma unroll 1
      for (int i = 0; i < p.num_peers; ++i) {
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.peer_out[i]) + off) = v;
      }
    } else {
      float f[8];
      unpack_bf16x8(v, f);
#pragma unroll 1
      for (int i = 0; i < p.num_peers; ++i) {
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.peer_out[i]) + off;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (gcol + j < p.n) dst[j] = __float2bfloat16_rn(f[j]);
        }
      }
    }
  }
}

// Register sums for FLUSH: this thread's columns of one accumulator row.
// Slot i covers accumulator columns c = group*16 + i*32 (16 wide; SwiGLU adds
// the up columns BNH + c), so a thread holds BNH floats.
template <int BNH, int EPI>
struct ChunkSums {
  static constexpr bool kSwiGLU = EPI == kEpiSwiGLU || EPI == kEpiSwiGLURoundBf16;
  static constexpr int kLimit = kSwiGLU ? BNH : 2 * BNH;  // accumulator columns walked
  static constexpr int kSlots = (kLimit + 16 * kEpiGroups - 1) / (16 * kEpiGroups);
  static constexpr int kPerSlot = kSwiGLU ? 32 : 16;
  float v[kSlots * kPerSlot];
};

template <int BNH, int EPI>
__device__ __forceinline__ void accumulate_chunk(uint32_t t_row, int group, bool first,
                                                 ChunkSums<BNH, EPI>& sums) {
  using S = ChunkSums<BNH, EPI>;
#pragma unroll
  for (int i = 0; i < S::kSlots; ++i) {
    const int c = group * 16 + i * 16 * kEpiGroups;
    if (c < S::kLimit) {  // warp-uniform: group is per warp
      float* dst = sums.v + i * S::kPerSlot;
      if constexpr (S::kSwiGLU) {
        uint32_t g[16], u[16];
        tmem_ld16x2(t_row + c, t_row + BNH + c, g, u);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          dst[j] = first ? __uint_as_float(g[j]) : __fadd_rn(dst[j], __uint_as_float(g[j]));
          dst[16 + j] = first ? __uint_as_float(u[j]) : __fadd_rn(dst[16 + j], __uint_as_float(u[j]));
        }
      } else {
        uint32_t a[16];
        tmem_ld16(t_row + c, a);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          dst[j] = first ? __uint_as_float(a[j]) : __fadd_rn(dst[j], __uint_as_float(a[j]));
        }
      }
    }
  }
}

template <int BNH, int EPI, typename TOut>
__device__ __forceinline__ void epilogue_sums(const GemmParams& p, int row, int nb, int group,
                                              const ChunkSums<BNH, EPI>& sums) {
  using S = ChunkSums<BNH, EPI>;
#pragma unroll
  for (int i = 0; i < S::kSlots; ++i) {
    const int c = group * 16 + i * 16 * kEpiGroups;
    if (c < S::kLimit) {
      const float* src = sums.v + i * S::kPerSlot;
      float o[16];
      if constexpr (S::kSwiGLU) {
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] = silu_f(src[j]) * src[16 + j];
        store_chunk<TOut, 16>(p, row, nb * BNH + c, o);
      } else {
        const int col_base = nb * 2 * BNH + c;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float bv = col_base + j < p.n ? __ldg(p.bias + col_base + j) : 0.0f;
          if constexpr (EPI == kEpiBiasGeluErf) {
            o[j] = gelu_erf_f(src[j] + bv);
          } else {
            o[j] = gelu_tanh_f(src[j] + bv);
          }
        }
        store_chunk<TOut, 16>(p, row, col_base, o);
      }
    }
  }
}

// ------------------------------------------------------------ the kernel

template <int BNH, int EPI, typename TOut, bool FLUSH = false>
__global__ void __launch_bounds__(kCtaThreads, 1) gemm_bf16_tc_kernel(const __grid_constant__ GemmParams p) {
  constexpr int kKps = FLUSH ? 1 : 2;
  using Cfg = TileCfg<BNH, kKps, epi_smem_reserve(EPI)>;
  static_assert(EPI != kEpiSwiGLUGather || (sizeof(TOut) == 2 && !FLUSH), "gather: bf16 out");
  constexpr int kStages = Cfg::kStages;
  constexpr uint32_t kIdesc = idesc_bf16_f32(kBlockM, Cfg::kMmaN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~static_cast<std::uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * Cfg::kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kStages;
  uint64_t* tfull_bar = bars + 2 * kStages;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.num_m_blocks * p.num_n_blocks;

  if (threadIdx.x == 0) {
    prefetch_tmap(&p.map_a);
    prefetch_tmap(&p.map_b0);
    prefetch_tmap(&p.map_b1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(full_bar + s), 1);
      mbar_init(smem_u32(empty_bar + s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(tfull_bar + a), 1);
      mbar_init(smem_u32(tempty_bar + a), kEpiWarps);
    }
    mbar_init(smem_u32(drain_bar), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    grid_dependents_launch();
  }
  // Warp 0 (the TMA producer; thread 0 initialised the barriers) needs no
  // TMEM, so it only arrives at the start-up barrier and goes straight to its
  // first loads, whose latency then overlaps the TMEM allocation; the other
  // warps wait there for the barriers and the TMEM address.
  uint32_t tmem_base = 0;
  if (warp == 0) {
    named_barrier_arrive(kStartBarrier, kCtaThreads);
  } else {
    if (warp == 2) tmem_alloc(smem_u32(tmem_holder), Cfg::kTmemCols);
    tc_fence_before();
    named_barrier_sync(kStartBarrier, kCtaThreads);
    tc_fence_after();
    tmem_base = *tmem_holder;
  }
  auto fail = [&](unsigned code) {
    atomicOr(p.status, code);
    *abort_flag = 1;
  };

  // Warpgroup 0: producer, MMA issuer, TMEM owner; warpgroups 1-2: epilogue.
  if (warp < 4) {
    if constexpr (FLUSH && BNH > 96) regs_release<kRegsControl>();
    if (warp == 0) {
      if (lane == 0) {
        // ---------------- TMA producer
        grid_dependency_wait();
        int stage = 0;
        uint32_t phase = 0;
        uint32_t issued_mask = 0;  // stages holding a copy that may be in flight
        uint32_t issued_phase = 0;
        int filled = 0;  // loads issued so far, counted up to kStages
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
          int mb, nb;
          tile_coords(tile, p, mb, nb);
          const int a_row = mb * kBlockM;
          const int b0_row = nb * p.b_row_stride;
          const int b1_row = b0_row + p.b1_row_offset;
          for (int kb = 0; kb < p.num_k_blocks; kb += kKps) {
            // The first pass over the ring needs no wait (every slot starts
            // empty), and skipping it saves the first wait on a barrier just
            // initialised (~0.4 us measured), which a one-k-block tile feels.
            if (filled >= kStages &&
                !mbar_wait(smem_u32(empty_bar + stage), phase ^ 1u, abort_flag)) {
              fail(kStatusProducer);
              ok = false;
              break;
            }
            const int nk = min(kKps, p.num_k_blocks - kb);
            const uint32_t fb = smem_u32(full_bar + stage);
            mbar_arrive_expect_tx(fb, nk * Cfg::kKBlockBytes);
#pragma unroll
            for (int j = 0; j < kKps; ++j) {
              if (j > 0 && j >= nk) break;  // k-block 0 of a stage always exists
              const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes + j * Cfg::kKBlockBytes);
              const uint32_t sb = sa + Cfg::kABytes;
              int ax, kx;
              k_block_coords(p, kb + j, ax, kx);
              tma_load_2d(sa, &p.map_a, fb, ax, a_row);
              tma_load_2d(sb, &p.map_b0, fb, kx, b0_row);
              tma_load_2d(sb + BNH * 128, &p.map_b1, fb, kx, b1_row);
            }
            if (filled < kStages) ++filled;
            issued_mask |= 1u << stage;
            issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
        if (!ok || *abort_flag) {
          // Drain: every copy this thread issued must land before the CTA exits.
          for (int s = 0; s < kStages; ++s) {
            if (issued_mask & (1u << s)) {
              if (!mbar_wait_drain(smem_u32(full_bar + s), (issued_phase >> s) & 1u)) {
                atomicOr(p.status, kStatusDrain);
              }
            }
          }
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        // ---------------- MMA issuer
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        bool ok = true;
        bool issued_any = false;
        const int chunks = tile_chunks<FLUSH>(p);
        for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
          for (int c = 0; c < chunks; ++c, ++local) {
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!mbar_wait(smem_u32(tempty_bar + acc), acc_phase ^ 1u, abort_flag)) {
              fail(kStatusMma);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * Cfg::kAccStride;
            int kb0, kb1;
            chunk_range<FLUSH>(p, c, kb0, kb1);
            for (int kb = kb0; kb < kb1; kb += kKps) {
              if (!mbar_wait(smem_u32(full_bar + stage), phase, abort_flag)) {
                fail(kStatusMma);
                ok = false;
                break;
              }
              tc_fence_after();
              const int nk = min(kKps, kb1 - kb);
#pragma unroll
              for (int j = 0; j < kKps; ++j) {
                if (j > 0 && j >= nk) break;  // k-block 0 of a stage always exists
                const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes + j * Cfg::kKBlockBytes);
                const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll
                for (int k = 0; k < kBlockK / 16; ++k) {
                  umma_bf16(d_tmem, sdesc_kmajor_sw128(sa + k * 32), sdesc_kmajor_sw128(sb + k * 32),
                            kIdesc, (kb + j != kb0 || k != 0) ? 1u : 0u);
                }
              }
              issued_any = true;
              umma_commit(smem_u32(empty_bar + stage));
              if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
              }
            }
            if (!ok) break;
            umma_commit(smem_u32(tfull_bar + acc));
          }
        }
        // All MMAs this thread issued must finish before TMEM is released.
        if (issued_any) {
          umma_commit(smem_u32(drain_bar));
          if (!mbar_wait_drain(smem_u32(drain_bar), 0)) atomicOr(p.status, kStatusDrain);
        }
      }
    }
  } else {
    if constexpr (FLUSH && BNH > 96) regs_acquire<kRegsEpilogue>();
    grid_dependency_wait();
    // ---------------- epilogue: warp w owns TMEM lanes [32q, 32q + 32) with
    // q = w % 4; the kEpiGroups warps of a quarter split its columns.
    const int q = warp & 3;
    const int group = (warp - 4) >> 2;
    const int chunks = tile_chunks<FLUSH>(p);
    uint8_t* gather_stage = smem + Cfg::kEpiSmemOffset + (warp - 4) * kGatherWarpBytes;
    (void)gather_stage;
    int local = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const int row = mb * kBlockM + q * 32 + lane;
      ChunkSums<BNH, EPI> sums;
      for (int c = 0; c < chunks; ++c, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        // The warp agrees on the outcome, so the warp-collective tcgen05.ld
        // below always runs with the full warp.
        if (!epi_wait(smem_u32(tfull_bar + acc), acc_phase, abort_flag, lane)) {
          if (lane == 0) fail(kStatusEpilogue);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * Cfg::kAccStride;
        if constexpr (FLUSH) {
          accumulate_chunk<BNH, EPI>(t_row, group, c == 0, sums);
        } else if constexpr (EPI == kEpiSwiGLUGather) {
          epilogue_gather_local<BNH>(p, row, nb, t_row, group, lane, gather_stage);
        } else {
          epilogue_tile<BNH, EPI, TOut>(p, row, nb, t_row, group);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(tempty_bar + acc));
      }
      if constexpr (FLUSH) {
        if (ok) epilogue_sums<BNH, EPI, TOut>(p, row, nb, group, sums);
      }
      if constexpr (EPI == kEpiSwiGLUGather) {
        // the accumulator is already released: the next tile's MMAs run
        // while this tile travels to the peers
        if (ok) epilogue_gather_peers<BNH>(p, row - lane, nb, group, lane, gather_stage);
        __syncwarp();
      }
    }
    // Peer stores of this thread complete before the kernel does, so a flag
    // raised after the launch (stream order) publishes them system-wide.
    if constexpr (EPI == kEpiSwiGLUGather) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace sm100
}  // namespace col
