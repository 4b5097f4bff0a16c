// Split-K over a cluster of two CTA pairs: the tensor-core GEMM for mid-size
// problems whose wide tiles are too few to fill the GPU.
//
// A GEMM such as M=512, K=4096, N=4096 with 256x256 output tiles has only 32
// tiles: one per CTA pair leaves most SMs idle, and narrower tiles (more of
// them) pay the pipeline's per-k-block floor on half the MMA work.  Here a
// cluster of four CTAs computes ONE tile: CTAs {0,1} are a CTA pair
// (tcgen05.mma.cta_group::2, as in gemm_sm100_2sm.cuh) accumulating k-blocks
// [0, K/2), CTAs {2,3} a second pair accumulating [K/2, K).  When both main
// loops are done, the two pairs exchange halves of their fp32 accumulators
// through distributed shared memory, reduce-scatter style: CTA r and CTA r^2
// hold the same 128 rows; CTA r finishes accumulator columns [0, 128) if
// r < 2, else [128, 256), and sends the other 128 columns of its partial to
// CTA r^2.  Sending is st.async from the epilogue warps' registers (TMEM
// loads) into the receiver's operand ring, which is free once the receiver's
// last MMA has completed; each write completes bytes on an mbarrier of the
// receiving warp.  The receiver adds the partner's partial to its own
// accumulator in a fixed order (k-blocks [0, K/2) + [K/2, K)) and runs the
// epilogue (bias + GELU, or the residual add) on its 128 columns, so the
// exchange and the epilogue are split evenly over all four SMs.  The
// epilogue warps, idle during the main loop, stage the tile's bias in shared
// memory first; TMEM loads and residual loads of the next chunk are issued
// before the current chunk is computed.
//
// Handshakes (every wait bounded as in the other kernels):
//   ready      in each CTA: one arrival from CTA r^2 once its ring is free
//              (its accumulator barrier completed);
//   red[w]     in each CTA, one per epilogue warp: armed at start-up for the
//              8 KB that the matching warp of CTA r^2 sends.
// Loads never use TMA multicast; every operand is this GPU's own memory.
#pragma once

#include "gemm_sm100_2sm.cuh"

namespace col {
namespace sm100 {

constexpr int kSkBnh = 128;                 // B box height: MMA N = 256
constexpr int kSkKps = 2;                   // k-blocks per pipeline stage
constexpr int kSkAccCols = 2 * kSkBnh;      // accumulator columns of a tile
constexpr int kSkChunksPerWarp = kSkAccCols / (16 * kEpiGroups);  // 16-column chunks
constexpr int kSkHalfChunks = kSkChunksPerWarp / 2;               // finished / sent per warp
constexpr uint32_t kSkWarpBytes = 32u * 16u * 4u * kSkHalfChunks;  // 32 rows x 64 fp32
constexpr uint32_t kSkPartialBytes = kEpiWarps * kSkWarpBytes;     // 64 KB received per CTA
constexpr uint32_t kSkBiasBytes = kSkAccCols * 4;                  // the tile's bias, staged

using SkCfg = TileCfg2<kSkBnh, kSkKps, 0>;
constexpr uint32_t kSkTmemCols = kSkAccCols;  // one accumulator: one tile per cluster
// dynamic shared memory: operand ring, barriers, then the staged bias
constexpr uint32_t kSkSmemBytes = SkCfg::kSmemBytes + kSkBiasBytes;
static_assert(SkCfg::kStages * SkCfg::kStageBytes >= kSkPartialBytes,
              "the partial accumulator must fit in the operand ring");
static_assert(kSkSmemBytes <= kSmemLimit, "shared memory budget");

__device__ __forceinline__ void mbar_arrive_expect_tx_local(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// Bounded wait with cluster-scope acquire: the data it guards was written by
// another CTA of the cluster.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Lane 0 polls (sleeping between polls), the warp agrees, as epi_wait.
__device__ __forceinline__ bool epi_wait_cluster(uint32_t bar, uint32_t parity,
                                                 volatile int* abort_flag, int lane) {
  int got = 0;
  if (lane == 0) {
    uint64_t t0 = 0;
    for (uint32_t i = 1;; ++i) {
      if (mbar_try_wait_cluster(bar, parity)) {
        got = 1;
        break;
      }
      __nanosleep(kEpiPollSleepNs);
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

// 16 bytes into another CTA's shared memory (shared::cluster address), the
// bytes counted on an mbarrier of that CTA.
__device__ __forceinline__ void st_async_v4(uint32_t remote_addr, uint32_t a, uint32_t b,
                                            uint32_t c, uint32_t d, uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
          remote_addr),
      "r"(a), "r"(b), "r"(c), "r"(d), "r"(remote_bar)
      : "memory");
}

// Byte offset of (epilogue warp w, its half-chunk il, 16-byte segment j,
// lane) in the received partial: a warp's 32 lanes write and read 512
// contiguous bytes per (chunk, segment), so neither side has bank conflicts.
__device__ __forceinline__ uint32_t sk_offset(int w, int il, int j, int lane) {
  return ((static_cast<uint32_t>(w * kSkHalfChunks + il) * 4u + static_cast<uint32_t>(j)) * 32u +
          static_cast<uint32_t>(lane)) * 16u;
}

// tcgen05.ld of 16 columns without waiting; tmem_wait16 completes it.  The
// wait names the registers as operands, so no use of them is scheduled
// before it.
__device__ __forceinline__ void tmem_ld16_start(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// Accumulator column of this warp's chunk i (0..kSkChunksPerWarp-1).
__device__ __forceinline__ int sk_chunk_col(int group, int i) {
  return group * 16 + i * 16 * kEpiGroups;
}

// Receiver: this thread's row, the chunks of its own half of the columns
// (chunks [first, first + kSkHalfChunks)): own accumulator + the partner's
// partial, then bias + GELU (bias from shared memory) or + residual.
template <int EPI, typename TOut>
__device__ __forceinline__ void sk_epilogue_finish(const GemmParams& p, int row, int nb,
                                                   uint32_t t_row, int group, int w, int lane,
                                                   int first, const uint8_t* partial,
                                                   const float* bias_tile) {
  const int col_base = nb * kSkAccCols;
  uint32_t next[16];
  float next_res[16];
  tmem_ld16_start(t_row + sk_chunk_col(group, first), next);
  if constexpr (EPI == kEpiResidual) load_residual16(p, row, col_base + sk_chunk_col(group, first), next_res);
#pragma unroll 1
  for (int il = 0; il < kSkHalfChunks; ++il) {
    const int c = sk_chunk_col(group, first + il);
    tmem_wait16(next);
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = __uint_as_float(next[j]);
    float res[16];
    if constexpr (EPI == kEpiResidual) {
#pragma unroll
      for (int j = 0; j < 16; ++j) res[j] = next_res[j];
    }
    if (il + 1 < kSkHalfChunks) {
      const int cn = sk_chunk_col(group, first + il + 1);
      tmem_ld16_start(t_row + cn, next);
      if constexpr (EPI == kEpiResidual) load_residual16(p, row, col_base + cn, next_res);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(partial + sk_offset(w, il, j, lane));
      acc[4 * j + 0] += v.x;
      acc[4 * j + 1] += v.y;
      acc[4 * j + 2] += v.z;
      acc[4 * j + 3] += v.w;
    }
    float o[16];
    if constexpr (EPI == kEpiResidual) {
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = acc[j] + res[j];
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float z = acc[j] + bias_tile[c + j];
        if constexpr (EPI == kEpiBiasGeluErf) {
          o[j] = gelu_erf_f(z);
        } else {
          o[j] = gelu_tanh_f(z);
        }
      }
    }
    store_chunk<TOut, 16>(p, row, col_base + c, o);
  }
}

// Sender: this thread's row, the partner's half of the columns (chunks
// [first, first + kSkHalfChunks)), into the partner's ring.
__device__ __forceinline__ void sk_epilogue_send(uint32_t t_row, int group, int w, int lane,
                                                 int first, uint32_t remote_base,
                                                 uint32_t remote_bar) {
  uint32_t next[16];
  tmem_ld16_start(t_row + sk_chunk_col(group, first), next);
#pragma unroll 1
  for (int il = 0; il < kSkHalfChunks; ++il) {
    tmem_wait16(next);
    uint32_t a[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) a[j] = next[j];
    if (il + 1 < kSkHalfChunks) tmem_ld16_start(t_row + sk_chunk_col(group, first + il + 1), next);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      st_async_v4(remote_base + sk_offset(w, il, j, lane), a[4 * j], a[4 * j + 1], a[4 * j + 2],
                  a[4 * j + 3], remote_bar);
    }
  }
}

// One 256 x 256 tile per cluster of four CTAs: p.num_m_blocks counts 256-row
// pair blocks, p.num_n_blocks 256-column blocks (B boxes at rows nb*256 and
// nb*256 + 128 of W, as the GELU-form pair kernel), grid = 4 * tiles.
template <int EPI, typename TOut>
__global__ void __cluster_dims__(4, 1, 1) __launch_bounds__(kCtaThreads, 1)
    gemm_bf16_sk_kernel(const __grid_constant__ GemmParams p) {
  static_assert(EPI == kEpiBiasGeluErf || EPI == kEpiBiasGeluTanh || EPI == kEpiResidual,
                "split-K cluster kernel: GELU-form B boxes");
  using Cfg = SkCfg;
  constexpr int kStages = Cfg::kStages;
  constexpr uint32_t kIdesc = idesc_bf16_f32(Cfg::kMmaM, Cfg::kMmaN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~static_cast<std::uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * Cfg::kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kStages;
  uint64_t* tfull_bar = bars + 2 * kStages;
  uint64_t* drain_bar = tfull_bar + 1;
  uint64_t* ready_bar = drain_bar + 1;
  uint64_t* red_bar = ready_bar + 1;  // kEpiWarps of them
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(red_bar + kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  static_assert((2 * kStages + 3 + kEpiWarps) * 8 + 8 <= Cfg::kBarrierBytes, "barrier space");

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();   // 0..3
  const uint32_t half = rank >> 1;           // 0: k-blocks [0, mid), 1: [mid, K)
  const uint32_t pair_base = rank & 2u;      // this pair's leader
  const bool leader = (rank & 1u) == 0u;
  const uint16_t pair_mask = static_cast<uint16_t>(0x3u << pair_base);
  const int tile = blockIdx.x >> 2;
  const int kb_mid = p.num_k_blocks / 2;
  const int kb_begin = half == 0 ? 0 : kb_mid;
  const int kb_end = half == 0 ? kb_mid : p.num_k_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(full_bar + s), 1);
      mbar_init(smem_u32(empty_bar + s), 1);
    }
    mbar_init(smem_u32(tfull_bar), 1);
    mbar_init(smem_u32(drain_bar), 1);
    mbar_init(smem_u32(ready_bar), 1);
    for (int w = 0; w < kEpiWarps; ++w) {
      mbar_init(smem_u32(red_bar + w), 1);
      // armed now for the partner's bytes: the phase completes when they land
      mbar_arrive_expect_tx_local(smem_u32(red_bar + w), kSkWarpBytes);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    grid_dependents_launch();
  }
  if (warp == 2) tmem_alloc_pair(smem_u32(tmem_holder), kSkTmemCols);
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  auto fail = [&](unsigned code) {
    atomicOr(p.status, code);
    *abort_flag = 1;
  };
  int mb, nb;
  tile_coords(tile, p, mb, nb);

  if (warp < 4) {
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer (every CTA): its rows of X, its half of B
      prefetch_tmap(&p.map_a);
      prefetch_tmap(&p.map_b0);
      grid_dependency_wait();
      const int a_row = mb * Cfg::kMmaM + static_cast<int>(rank & 1u) * kBlockM;
      const int b_row = nb * p.b_row_stride + static_cast<int>(rank & 1u) * p.b1_row_offset;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0;
      uint32_t issued_phase = 0;
      int filled = 0;
      bool ok = true;
      for (int kb = kb_begin; kb < kb_end; kb += kSkKps) {
        if (filled >= kStages && !mbar_wait(smem_u32(empty_bar + stage), phase ^ 1u, abort_flag)) {
          fail(kStatusProducer);
          ok = false;
          break;
        }
        const int nk = min(kSkKps, kb_end - kb);
        const uint32_t fb_local = smem_u32(full_bar + stage);
        if (leader) mbar_arrive_expect_tx(fb_local, 2 * nk * Cfg::kKBlockBytes);
        const uint32_t fb = map_to_cta(fb_local, pair_base);
#pragma unroll
        for (int j = 0; j < kSkKps; ++j) {
          if (j > 0 && j >= nk) break;
          const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes + j * Cfg::kKBlockBytes);
          tma_load_2d_pair(sa, &p.map_a, fb, (kb + j) * kBlockK, a_row);
          tma_load_2d_pair(sa + Cfg::kABytes, &p.map_b0, fb, (kb + j) * kBlockK, b_row);
        }
        if (filled < kStages) ++filled;
        issued_mask |= 1u << stage;
        issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok || *abort_flag) {
        if (leader) {
          for (int s = 0; s < kStages; ++s) {
            if ((issued_mask & (1u << s)) &&
                !mbar_wait_drain(smem_u32(full_bar + s), (issued_phase >> s) & 1u)) {
              atomicOr(p.status, kStatusDrain);
            }
          }
        } else {
          for (int i = 0; i < 200; ++i) __nanosleep(1000);
        }
      }
    } else if (warp == 1 && lane == 0 && leader) {
      // ---------------- MMA issuer (pair leaders, CTAs 0 and 2)
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int kb = kb_begin; kb < kb_end; kb += kSkKps) {
        if (!mbar_wait(smem_u32(full_bar + stage), phase, abort_flag)) {
          fail(kStatusMma);
          ok = false;
          break;
        }
        tc_fence_after();
        const int nk = min(kSkKps, kb_end - kb);
#pragma unroll
        for (int j = 0; j < kSkKps; ++j) {
          if (j > 0 && j >= nk) break;
          const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes + j * Cfg::kKBlockBytes);
          const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll
          for (int k = 0; k < kBlockK / 16; ++k) {
            umma_bf16_pair(tmem_base, sdesc_kmajor_sw128(sa + k * 32), sdesc_kmajor_sw128(sb + k * 32),
                           kIdesc, (kb + j != kb_begin || k != 0) ? 1u : 0u);
          }
        }
        issued_any = true;
        asm volatile(
            "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
            " [%0], %1;" ::"r"(smem_u32(empty_bar + stage)),
            "h"(pair_mask)
            : "memory");
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) {
        asm volatile(
            "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
            " [%0], %1;" ::"r"(smem_u32(tfull_bar)),
            "h"(pair_mask)
            : "memory");
      }
      if (issued_any) {
        umma_commit_pair_local(smem_u32(drain_bar));
        if (!mbar_wait_drain(smem_u32(drain_bar), 0)) atomicOr(p.status, kStatusDrain);
      }
    }
  } else {
    grid_dependency_wait();
    // ---------------- epilogue: this CTA's 128 rows of the tile
    const int q = warp & 3;
    const int group = (warp - 4) >> 2;
    const int w = warp - 4;
    const int row = mb * Cfg::kMmaM + static_cast<int>(rank & 1u) * kBlockM + q * 32 + lane;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t partner = rank ^ 2u;
    float* bias_tile = reinterpret_cast<float*>(smem + kStages * Cfg::kStageBytes + Cfg::kBarrierBytes);
    if constexpr (EPI != kEpiResidual) {
      // stage the tile's bias while the main loop runs (zero past n)
      const int t = threadIdx.x - 128;
      const int col = nb * kSkAccCols + t;
      if (t < kSkAccCols) bias_tile[t] = col < p.n ? __ldg(p.bias + col) : 0.0f;
      named_barrier_sync(kStartBarrier + 1, 32 * kEpiWarps);
    }
    bool ok = epi_wait(smem_u32(tfull_bar), 0, abort_flag, lane);
    if (!ok && lane == 0) fail(kStatusEpilogue);
    if (ok) {
      tc_fence_after();
      // every MMA of this pair has completed, so the ring is free: the
      // partner may send
      if (w == 0 && lane == 0) mbar_arrive_cluster(map_to_cta(smem_u32(ready_bar), partner));
    }
    const int own_first = half == 0 ? 0 : kSkHalfChunks;
    const int send_first = half == 0 ? kSkHalfChunks : 0;
    if (ok && !epi_wait_cluster(smem_u32(ready_bar), 0, abort_flag, lane)) {
      if (lane == 0) fail(kStatusEpilogue);
      ok = false;
    }
    if (ok) {
      sk_epilogue_send(t_row, group, w, lane, send_first, map_to_cta(smem_u32(smem), partner),
                       map_to_cta(smem_u32(red_bar + w), partner));
    }
    if (ok && !epi_wait_cluster(smem_u32(red_bar + w), 0, abort_flag, lane)) {
      if (lane == 0) fail(kStatusEpilogue);
      ok = false;
    }
    if (ok) sk_epilogue_finish<EPI, TOut>(p, row, nb, t_row, group, w, lane, own_first, smem, bias_tile);
    tc_fence_before();
  }

  // No CTA leaves while another may still address its shared memory (the
  // partner's st.async into the ring, the remote arrivals).
  tc_fence_before();
  cluster_sync();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kSkTmemCols);
  }
}

}  // namespace sm100
}  // namespace col
