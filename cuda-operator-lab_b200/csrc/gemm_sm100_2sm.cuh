// CTA-pair (2-SM) variant of the tensor-core GEMM: tcgen05.mma.cta_group::2.
//
// A cluster of two CTAs on two SMs computes a 256-row tile: each CTA loads
// its own 128 rows of X and HALF of the B tile (SwiGLU: CTA 0 the gate box,
// CTA 1 the up box; GELU: the two halves of the W box), and one MMA
// instruction issued by CTA 0 (M=256, N=2*BNH, K=16) reads A and B from both
// CTAs' shared memory and accumulates into both CTAs' TMEM (each CTA holds its
// 128 rows x N columns, so the epilogue is the same as the 1-CTA kernel).
// Per SM and k-block this moves 16 KB of X + BNH*128 B of W instead of
// 16 KB + 2*BNH*128 B: a third less L2->SM traffic per flop, which is what
// bounds the 1-CTA kernel when few M-blocks share each weight tile.
//
// Synchronisation (all mbarrier waits bounded as in the 1-CTA kernel):
//   full[s]   in CTA 0 only: CTA 0's producer posts the byte count of both
//             CTAs' loads; both CTAs' TMA loads complete on it;
//   empty[s]  in each CTA: the MMA's commit is multicast to both CTAs;
//   tfull[a]  in each CTA: MMA commit multicast, each epilogue waits locally;
//   tempty[a] in CTA 0: the epilogue warps of both CTAs arrive (remote
//             arrive for CTA 1).
// No TMA multicast: every load reads this GPU's memory into the issuing CTA.
#pragma once

#include "gemm_sm100.cuh"

namespace col {
namespace sm100 {

// KPS = k-blocks per pipeline stage, as in TileCfg.
template <int BNH, int KPS = 1, uint32_t RESERVE = 0>
struct TileCfg2;

// k-blocks per stage of the pair kernel: the most operand bytes in flight.
// Mid-size GEMMs wait on L2 round trips, so throughput per SM follows the
// bytes the ring holds: at BNH = 64 three-k-block stages hold 216 KB (three
// stages) where two-k-block stages hold 192 KB (four); elsewhere two.  FLUSH
// kernels keep one (their accumulation chunks end on k-block boundaries).
constexpr int pair_kps(int bnh, int epi, bool flush) {
  return flush ? 1 : (bnh == 64 && epi_smem_reserve(epi) == 0 ? 3 : 2);
}

template <int BNH, int KPS, uint32_t RESERVE>
struct TileCfg2 {
  static_assert(BNH % 16 == 0 && BNH >= 32 && BNH <= 128, "unsupported B box height");
  static_assert(KPS >= 1 && KPS <= 3, "one to three k-blocks per stage");
  static constexpr int kMmaM = 256;
  static constexpr int kMmaN = 2 * BNH;
  static constexpr uint32_t kABytes = kBlockM * kBlockK * 2;  // this CTA's 128 rows
  static constexpr uint32_t kBBytes = BNH * kBlockK * 2;      // this CTA's half of B
  static constexpr uint32_t kKBlockBytes = kABytes + kBBytes;  // [A | B] of one k-block
  static constexpr uint32_t kStageBytes = KPS * kKBlockBytes;
  static constexpr uint32_t kBarrierBytes = 256;
  static constexpr int kStagesFit =
      static_cast<int>((kSmemLimit - 1024 - kBarrierBytes - RESERVE) / kStageBytes);
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr uint32_t kAccStride = pow2_at_least(kMmaN);
  static constexpr uint32_t kTmemCols = 2 * kAccStride;
  static constexpr uint32_t kEpiSmemOffset = kStages * kStageBytes + kBarrierBytes;
  static constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024 + kBarrierBytes + RESERVE;
  static_assert(kTmemCols <= 512, "two accumulators must fit in TMEM");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t saddr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
  return out;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t cluster_bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at local offset `bar` in both CTAs of the pair once
// all previously issued MMAs of this thread complete.
__device__ __forceinline__ void umma_commit_pair_both(uint32_t bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

__device__ __forceinline__ void umma_commit_pair_local(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t holder, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}

// Pair tiles: p.num_m_blocks counts 256-row pair blocks here.
template <int BNH, int EPI, typename TOut, bool FLUSH = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kCtaThreads, 1)
    gemm_bf16_tc2_kernel(const __grid_constant__ GemmParams p) {
  constexpr int kKps = pair_kps(BNH, EPI, FLUSH);
  using Cfg = TileCfg2<BNH, kKps, epi_smem_reserve(EPI)>;
  static_assert(EPI != kEpiSwiGLUGather || (sizeof(TOut) == 2 && !FLUSH), "gather: bf16 out");
  constexpr int kStages = Cfg::kStages;
  constexpr uint32_t kIdesc = idesc_bf16_f32(Cfg::kMmaM, Cfg::kMmaN);

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
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int num_tiles = p.num_m_blocks * p.num_n_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(full_bar + s), 1);
      mbar_init(smem_u32(empty_bar + s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(tfull_bar + a), 1);
      mbar_init(smem_u32(tempty_bar + a), 2 * kEpiWarps);
    }
    mbar_init(smem_u32(drain_bar), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    grid_dependents_launch();
  }
  if (warp == 2) tmem_alloc_pair(smem_u32(tmem_holder), Cfg::kTmemCols);
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  auto fail = [&](unsigned code) {
    atomicOr(p.status, code);
    *abort_flag = 1;
  };

  // Warpgroup 0: producer, MMA issuer, TMEM owner; warpgroups 1-2: epilogue.
  if (warp < 4) {
    if constexpr (FLUSH && BNH > 96) regs_release<kRegsControl>();
    if (warp == 0) {
      if (lane == 0) {
        // ---------------- TMA producer (both CTAs)
        prefetch_tmap(&p.map_a);
        prefetch_tmap(leader ? &p.map_b0 : &p.map_b1);
        grid_dependency_wait();
        const CUtensorMap* map_b = leader ? &p.map_b0 : &p.map_b1;
        int stage = 0;
        uint32_t phase = 0;
        uint32_t issued_mask = 0;
        uint32_t issued_phase = 0;
        int filled = 0;  // loads issued so far, counted up to kStages
        bool ok = true;
        for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
          int mb, nb;
          tile_coords(tile, p, mb, nb);
          const int a_row = mb * Cfg::kMmaM + static_cast<int>(rank) * kBlockM;
          // SwiGLU: both CTAs use row nb*BNH (of the gate map / the up map);
          // GELU: CTA r loads rows nb*2*BNH + r*BNH of W.
          const int b_row = nb * p.b_row_stride + static_cast<int>(rank) * p.b1_row_offset;
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
            const uint32_t fb_local = smem_u32(full_bar + stage);
            if (leader) mbar_arrive_expect_tx(fb_local, 2 * nk * Cfg::kKBlockBytes);
            const uint32_t fb = map_to_cta(fb_local, 0);
#pragma unroll
            for (int j = 0; j < kKps; ++j) {
              if (j > 0 && j >= nk) break;  // k-block 0 of a stage always exists
              const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes + j * Cfg::kKBlockBytes);
              const uint32_t sb = sa + Cfg::kABytes;
              int ax, kx;
              k_block_coords(p, kb + j, ax, kx);
              tma_load_2d_pair(sa, &p.map_a, fb, ax, a_row);
              tma_load_2d_pair(sb, map_b, fb, kx, b_row);
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
          if (leader) {
            for (int s = 0; s < kStages; ++s) {
              if (issued_mask & (1u << s)) {
                if (!mbar_wait_drain(smem_u32(full_bar + s), (issued_phase >> s) & 1u)) {
                  atomicOr(p.status, kStatusDrain);
                }
              }
            }
          } else {
            // CTA 1 cannot observe CTA 0's barrier: give its copies time to land.
            for (int i = 0; i < 200; ++i) __nanosleep(1000);
          }
        }
      }
    } else if (warp == 1) {
      if (lane == 0 && leader) {
        // ---------------- MMA issuer (CTA 0 only)
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        bool ok = true;
        bool issued_any = false;
        const int chunks = tile_chunks<FLUSH>(p);
        for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
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
                  umma_bf16_pair(d_tmem, sdesc_kmajor_sw128(sa + k * 32),
                                 sdesc_kmajor_sw128(sb + k * 32), kIdesc,
                                 (kb + j != kb0 || k != 0) ? 1u : 0u);
                }
              }
              issued_any = true;
              umma_commit_pair_both(smem_u32(empty_bar + stage));
              if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
              }
            }
            if (!ok) break;
            umma_commit_pair_both(smem_u32(tfull_bar + acc));
          }
        }
        if (issued_any) {
          umma_commit_pair_local(smem_u32(drain_bar));
          if (!mbar_wait_drain(smem_u32(drain_bar), 0)) atomicOr(p.status, kStatusDrain);
        }
      }
    }
  } else {
    if constexpr (FLUSH && BNH > 96) regs_acquire<kRegsEpilogue>();
    grid_dependency_wait();
    // ---------------- epilogue (both CTAs): this CTA's 128 rows of the tile
    const int q = warp & 3;
    const int group = (warp - 4) >> 2;
    const int chunks = tile_chunks<FLUSH>(p);
    uint8_t* gather_stage = smem + Cfg::kEpiSmemOffset + (warp - 4) * kGatherWarpBytes;
    (void)gather_stage;
    int local = 0;
    bool ok = true;
    for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const int row = mb * Cfg::kMmaM + static_cast<int>(rank) * kBlockM + q * 32 + lane;
      ChunkSums<BNH, EPI> sums;
      for (int c = 0; c < chunks; ++c, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
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
        if (lane == 0) mbar_arrive_cluster(map_to_cta(smem_u32(tempty_bar + acc), 0));
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

  // Neither CTA leaves while the other may still address its shared memory.
  tc_fence_before();
  cluster_sync();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace sm100
}  // namespace col
