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

// ------------------------------------------------------------ stream-K tail
//
// Work of one CTA pair: whole tiles c, c + P, ... below p.sk_dp_tiles (all
// tiles when stream-K is off), then -- stream-K on -- an even share of the
// k-blocks of the remaining tiles, taken in tile order.  Every share is at
// least one tile long, so a tile is split at most once, between pairs c and
// c+1: pair c+1 computes the tile's last k-blocks first thing in its share
// (kind kWorkTail: the accumulator goes to global memory and a flag is set),
// pair c its first k-blocks last (kind kWorkHead: it adds c+1's partial and
// runs the epilogue).  All three roles walk the same sequence.
constexpr int kWorkFull = 0;
constexpr int kWorkTail = 1;
constexpr int kWorkHead = 2;

struct WorkItem {
  int tile;
  int kb0;
  int kb1;
  int kind;
};

struct WorkSched {
  int pair, pairs, dp_end, next_dp, kbs;
  uint64_t u, u_end;
  bool sk;

  __device__ __forceinline__ WorkSched(const GemmParams& p, int c, int num_pairs)
      : pair(c), pairs(num_pairs), next_dp(c), kbs(p.num_k_blocks), u(0), u_end(0) {
    const int num_tiles = p.num_m_blocks * p.num_n_blocks;
    sk = p.sk_flags != nullptr;
    dp_end = sk ? p.sk_dp_tiles : num_tiles;
    if (sk) {
      const uint64_t units = static_cast<uint64_t>(num_tiles - dp_end) * static_cast<uint64_t>(kbs);
      u = units * static_cast<uint64_t>(c) / static_cast<uint64_t>(num_pairs);
      u_end = units * static_cast<uint64_t>(c + 1) / static_cast<uint64_t>(num_pairs);
    }
  }

  __device__ __forceinline__ bool next(WorkItem& w) {
    if (next_dp < dp_end) {
      w.tile = next_dp;
      w.kb0 = 0;
      w.kb1 = kbs;
      w.kind = kWorkFull;
      next_dp += pairs;
      return true;
    }
    if (u < u_end) {
      const uint64_t t = u / static_cast<uint64_t>(kbs);
      w.tile = dp_end + static_cast<int>(t);
      w.kb0 = static_cast<int>(u - t * static_cast<uint64_t>(kbs));
      const uint64_t left = u_end - u;
      w.kb1 = static_cast<int>(min(static_cast<uint64_t>(kbs), static_cast<uint64_t>(w.kb0) + left));
      w.kind = w.kb0 > 0 ? kWorkTail : (w.kb1 < kbs ? kWorkHead : kWorkFull);
      u += static_cast<uint64_t>(w.kb1 - w.kb0);
      return true;
    }
    return false;
  }
};

// One CTA's partial accumulator (128 rows x 2*BNH fp32) is laid out as the
// epilogue deals its columns (16-column chunks round robin over the
// kEpiGroups warps of a lane quarter; partial_offset in gemm_sm100.cuh), so
// each warp writes -- and reads back -- 512 contiguous bytes per (chunk,
// segment).
template <int BNH>
constexpr uint32_t partial_cta_bytes() {
  return static_cast<uint32_t>(128 * 2 * BNH * 4);
}

// kWorkTail: this thread's accumulator row, every column, to global memory.
template <int BNH>
__device__ __forceinline__ void epilogue_dump_partial(uint32_t t_row, int q, int group, int lane,
                                                      uint8_t* part) {
#pragma unroll 1
  for (int c = group * 16; c < 2 * BNH; c += 16 * kEpiGroups) {
    uint32_t a[16];
    tmem_ld16(t_row + c, a);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      *reinterpret_cast<uint4*>(part + partial_offset<BNH>(q, c, j, lane)) =
          make_uint4(a[4 * j], a[4 * j + 1], a[4 * j + 2], a[4 * j + 3]);
    }
  }
}

// kWorkHead: the epilogue of epilogue_tile with the partner's partial (in
// shared memory, partial_offset layout) added to the accumulator first.
template <int BNH, int EPI, typename TOut>
__device__ __forceinline__ void epilogue_tile_with_partial(const GemmParams& p, int row, int nb,
                                                           uint32_t t_row, int q, int group,
                                                           int lane, const uint8_t* part) {
  if constexpr (EPI == kEpiSwiGLU || EPI == kEpiSwiGLURoundBf16 || EPI == kEpiSwiGLURowScale) {
    const int col_base = nb * BNH;
    float rs = 1.0f;
    if constexpr (EPI == kEpiSwiGLURowScale) rs = row < p.m ? __ldg(p.row_scale + row) : 0.0f;
#pragma unroll 1
    for (int c = group * 16; c < BNH; c += 16 * kEpiGroups) {
      uint32_t g[16], u[16];
      tmem_ld16x2(t_row + c, t_row + BNH + c, g, u);
      float gv[16], uv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        gv[j] = __uint_as_float(g[j]);
        uv[j] = __uint_as_float(u[j]);
      }
      add_partial16(part, partial_offset<BNH>(q, c, 0, lane), gv);
      add_partial16(part, partial_offset<BNH>(q, BNH + c, 0, lane), uv);
      float o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float a = gv[j], b = uv[j];
        if constexpr (EPI == kEpiSwiGLURoundBf16) {
          a = bf16_round(a);
          b = bf16_round(b);
        } else if constexpr (EPI == kEpiSwiGLURowScale) {
          a *= rs;
          b *= rs;
        }
        o[j] = silu_fast(a) * b;
      }
      store_chunk<TOut, 16>(p, row, col_base + c, o);
    }
  } else {
    const int col_base = nb * 2 * BNH;
#pragma unroll 1
    for (int c = group * 16; c < 2 * BNH; c += 16 * kEpiGroups) {
      uint32_t a[16];
      tmem_ld16(t_row + c, a);
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(a[j]);
      add_partial16(part, partial_offset<BNH>(q, c, 0, lane), v);
      float o[16];
      if constexpr (EPI == kEpiResidual) {
        float res[16];
        load_residual16(p, row, col_base + c, res);
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] = v[j] + res[j];
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int colj = col_base + c + j;
          const float z = v[j] + (colj < p.n ? __ldg(p.bias + colj) : 0.0f);
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
}

__device__ __forceinline__ void st_release_gpu(unsigned* addr, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* addr) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Bounded wait for a flag that another CTA pair sets.
__device__ __forceinline__ bool wait_flag(const unsigned* flag, volatile int* abort_flag) {
  uint64_t t0 = 0;
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_gpu(flag) != 0u) return true;
    __nanosleep(128);
    if ((i & 15u) == 0u) {
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

__device__ __forceinline__ void bulk_load_global(uint32_t dst, const void* src, uint32_t bytes,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
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
  // stream-K is never set up for the fp32 emulation
  constexpr bool kStreamK = !FLUSH;
  static_assert(!kStreamK || Cfg::kStages * Cfg::kStageBytes >= partial_cta_bytes<BNH>(),
                "a partial accumulator must fit in the operand ring");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~static_cast<std::uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * Cfg::kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kStages;
  uint64_t* tfull_bar = bars + 2 * kStages;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* part_bar = drain_bar + 1;  // the partner's partial landed (stream-K)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(part_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  static_assert((2 * kStages + 6) * 8 + 8 <= Cfg::kBarrierBytes, "barrier space");

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

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
    mbar_init(smem_u32(part_bar), 1);
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
        WorkSched sched(p, cluster_id, num_clusters);
        WorkItem w;
        while (ok && sched.next(w)) {
          int mb, nb;
          tile_coords(w.tile, p, mb, nb);
          const int a_row = mb * Cfg::kMmaM + static_cast<int>(rank) * kBlockM;
          // SwiGLU: both CTAs use row nb*BNH (of the gate map / the up map);
          // GELU: CTA r loads rows nb*2*BNH + r*BNH of W.
          const int b_row = nb * p.b_row_stride + static_cast<int>(rank) * p.b1_row_offset;
          for (int kb = w.kb0; kb < w.kb1; kb += kKps) {
            // The first pass over the ring needs no wait (every slot starts
            // empty), and skipping it saves the first wait on a barrier just
            // initialised (~0.4 us measured), which a one-k-block tile feels.
            if (filled >= kStages &&
                !mbar_wait(smem_u32(empty_bar + stage), phase ^ 1u, abort_flag)) {
              fail(kStatusProducer);
              ok = false;
              break;
            }
            const int nk = min(kKps, w.kb1 - kb);
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
        WorkSched sched(p, cluster_id, num_clusters);
        WorkItem w;
        while (ok && sched.next(w)) {
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
            if constexpr (FLUSH) {
              chunk_range<FLUSH>(p, c, kb0, kb1);
            } else {
              kb0 = w.kb0;
              kb1 = w.kb1;
            }
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
    WorkSched sched(p, cluster_id, num_clusters);
    WorkItem w;
    while (ok && sched.next(w)) {
      int mb, nb;
      tile_coords(w.tile, p, mb, nb);
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
        } else {
          if (w.kind == kWorkFull) {
            if constexpr (EPI == kEpiSwiGLUGather) {
              epilogue_gather_local<BNH>(p, row, nb, t_row, group, lane, gather_stage);
            } else {
              epilogue_tile<BNH, EPI, TOut>(p, row, nb, t_row, group);
            }
          } else if (w.kind == kWorkTail) {
            // the tile's last k-blocks: the accumulator goes to this pair's
            // partial buffer; the flag says it is complete
            uint8_t* part = p.sk_partials +
                            (static_cast<std::size_t>(cluster_id) * 2 + rank) * partial_cta_bytes<BNH>();
            epilogue_dump_partial<BNH>(t_row, q, group, lane, part);
            // every lane's stores are visible GPU-wide before its warp's flag
            __threadfence();
            __syncwarp();
            if (lane == 0) {
              st_release_gpu(p.sk_flags + (cluster_id * 2 + rank) * kEpiWarps + (warp - 4), 1u);
            }
          } else {
            // the tile's first k-blocks, the pair's last item: every MMA of
            // this pair is complete, so the operand ring is free to receive
            // the next pair's partial (same tile, its last k-blocks)
            bool got = true;
            if (warp == 4 && lane == 0) {
              // every warp of the partner CTA has written its part
              const unsigned* flags = p.sk_flags + ((cluster_id + 1) * 2 + rank) * kEpiWarps;
              for (int f = 0; got && f < kEpiWarps; ++f) got = wait_flag(flags + f, abort_flag);
              if (got) {
                asm volatile("fence.proxy.async.global;" ::: "memory");
                const uint8_t* src = p.sk_partials + (static_cast<std::size_t>(cluster_id + 1) * 2 + rank) *
                                                         partial_cta_bytes<BNH>();
                mbar_arrive_expect_tx(smem_u32(part_bar), partial_cta_bytes<BNH>());
                bulk_load_global(smem_u32(smem), src, partial_cta_bytes<BNH>(), smem_u32(part_bar));
              } else {
                fail(kStatusEpilogue);
              }
            }
            got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
            if (got && !epi_wait(smem_u32(part_bar), 0, abort_flag, lane)) {
              if (lane == 0) fail(kStatusEpilogue);
              got = false;
            }
            if (got) {
              if constexpr (EPI == kEpiSwiGLUGather) {
                epilogue_gather_local<BNH>(p, row, nb, t_row, group, lane, gather_stage, q, smem);
              } else {
                epilogue_tile_with_partial<BNH, EPI, TOut>(p, row, nb, t_row, q, group, lane, smem);
              }
            } else {
              ok = false;
            }
          }
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
        // while this tile travels to the peers (a stream-K tail part has no
        // output of its own)
        if (ok && w.kind != kWorkTail) {
          epilogue_gather_peers<BNH>(p, row - lane, nb, group, lane, gather_stage);
        }
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
