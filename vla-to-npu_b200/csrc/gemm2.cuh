// Two-CTA (cta_group::2) variant of the persistent bf16 GEMM.
//
// A cluster of two CTAs on neighbouring SMs computes a 256 x BN tile with
// UMMA 256 x BN x 16 issued by the pair's leader (rank 0):
//   - each CTA TMA-loads its own 128 rows of A and its own BN/2 rows of B
//     (plain loads, no multicast); both CTAs' loads complete on the leader's
//     `full` barrier, so every SM stages 16 KB of A + BN*64 B of B per
//     k-block instead of 16 KB + BN*128 B (half the B traffic per SM, six
//     pipeline stages in 192 KB at BN = 256);
//   - the leader's commits are multicast to both CTAs' `empty` (smem slot free)
//     and `tfull` (accumulator ready) barriers;
//   - each CTA's epilogue warps drain the 128 accumulator rows that live in its
//     own tensor memory and arrive on the leader's `tempty` barrier (one
//     relaxed cluster-scope arrive per warp: release arrives cost a fence each).
// Epilogue semantics are those of the one-CTA kernel (gemm.cuh).
#pragma once
#include "gemm.cuh"

namespace vla {
namespace gemm {

// KPS k-blocks per stage: with KPS > 1 a stage is filled by one k-slab TMA box
// per operand (gemm_skinny.cuh explains the per-stage costs this amortises).
template <int BN, int KPS = 1>
struct Cfg2 {
  static constexpr int A_KB = BM * BK * 2;           // 128 rows of A per CTA and k-block
  static constexpr int B_KB = (BN / 2) * BK * 2;     // half of the B tile per CTA and k-block
  static constexpr int A_BYTES = KPS * A_KB;
  static constexpr int B_BYTES = KPS * B_KB;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BUDGET = kSmemLimit - 1024 - kBarrierBytes - kEpiStoreBytes;
  static constexpr int STAGES = (BUDGET / STAGE_BYTES) > 8 ? 8 : (BUDGET / STAGE_BYTES);
  static constexpr int TMEM_COLS = (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + kEpiStoreBytes + kBarrierBytes + 1024;
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "UMMA N");
  static_assert(B_KB % 1024 == 0, "B half-tile alignment (BN/2 multiple of 8)");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the variable at local shared address `a` in CTA `rank`
__device__ __forceinline__ uint32_t map_to_rank(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t bar_cluster_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.relaxed.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(bar_cluster_addr),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* smem_dst, const void* tmap, uint32_t bar_cluster_addr, int x,
                                                 int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(bar_cluster_addr)
      : "memory");
}

// Relaxed remote arrive: used only to hand a tensor-memory accumulator back to
// the MMA issuer, whose ordering comes from tcgen05.wait::ld and the tcgen05
// thread-sync fences; no shared or global data is published through it.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

// TMA load into this CTA's smem whose completion is counted on a barrier of
// either CTA of the pair (cta_group::2 form, no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap, uint32_t bar_cluster_addr, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar_cluster_addr)
      : "memory");
}

__device__ __forceinline__ void tc_mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// arrive once on the barrier at the same smem offset in both CTAs of the pair
// when the previously issued MMAs completed
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)0x3)
      : "memory");
}

// tmA3 / tmB3: k-slab maps (64, rows, K / 64) with (64, 128, KPS) and
// (64, BN / 2, KPS) boxes, used when KPS > 1 for units of whole k-blocks.
template <int BN, int KPS = 1>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmA3, const __grid_constant__ CUtensorMap tmB3,
                         const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR, DevEpi ep,
                         int M, int N, int K) {
  using Cf = Cfg2<BN, KPS>;
  constexpr int STAGES = Cf::STAGES;
  static_assert(STAGES >= 2, "pair GEMM: two stages");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + STAGES * Cf::A_BYTES;
  uint8_t* sC = sB + STAGES * Cf::B_BYTES;  // output staging (1024-byte aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(sC + kEpiStoreBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* rbar = tempty + 2;  // [kEpiWarps][2]: residual chunk landed (this CTA's)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 2 * kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int cluster = blockIdx.x >> 1;
  const int n_clusters = gridDim.x >> 1;
  const int num_m = (M + 2 * BM - 1) / (2 * BM);
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  const int nfull = K / BK;
  const int nunits = (num_kb + KPS - 1) / KPS;
  auto unit_kbs = [&](int u) { return min(KPS, num_kb - u * KPS); };
  auto unit_slab = [&](int u) { return KPS > 1 && u * KPS + KPS <= nfull; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 2);   // one expect_tx arrival per CTA (leader's copy is used)
      mbar_init(&empty[s], 1);  // multicast MMA commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);                    // multicast MMA commit
      mbar_init(&tempty[i], 2 * kEpiWarps);  // one arrival per epilogue warp of both CTAs (leader's copy)
    }
    *abort_flag = 0;
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&rbar[i], 1);
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (KPS > 1) {
      tma_prefetch_desc(&tmA3);
      tma_prefetch_desc(&tmB3);
    }
    if (ep.tma_c) tma_prefetch_desc(&tmC);
    if (ep.tma_r) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)Cf::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_prologue();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = cluster; t < num_tiles && ok; t += n_clusters) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        const int arow = mb * 2 * BM + (int)rank * BM, brow = nb * BN + (int)rank * (BN / 2);
        for (int u = 0; u < nunits; ++u) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t leader_full = map_to_rank(smem_u32(&full[s]), 0);
          const int cnt = unit_kbs(u);
          if (unit_slab(u)) {
            mbar_arrive_expect_tx_cluster(leader_full, Cf::STAGE_BYTES);
            tma_load_3d_pair(sA + s * Cf::A_BYTES, &tmA3, leader_full, 0, arow, u * KPS);
            tma_load_3d_pair(sB + s * Cf::B_BYTES, &tmB3, leader_full, 0, brow, u * KPS);
          } else {
            mbar_arrive_expect_tx_cluster(leader_full, (uint32_t)(cnt * (Cf::A_KB + Cf::B_KB)));
            for (int i = 0; i < cnt; ++i) {
              const int kb = u * KPS + i;
              tma_load_2d_pair(sA + s * Cf::A_BYTES + i * Cf::A_KB, &tmA, leader_full, kb * BK, arow);
              tma_load_2d_pair(sB + s * Cf::B_BYTES + i * Cf::B_KB, &tmB, leader_full, kb * BK, brow);
            }
          }
          ++it;
        }
      }
      if (!ok) {
        if (!*abort_flag) vla_record_error(VLA_DERR_GEMM_PRODUCER_TIMEOUT);
        *abort_flag = 1;
      }
      // Let this CTA's issued copies land before it can exit: a slot is free again
      // only after the MMAs that read it, which read after the copies completed.
      const int first = it > STAGES ? it - STAGES : 0;
      for (int j = first; j < it; ++j)
        mbar_wait_bounded(&empty[j % STAGES], (uint32_t)(j / STAGES) & 1u, nullptr, 20000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(2 * BM, BN);
      int it = 0, tc = 0;
      bool ok = true;
      for (int t = cluster; t < num_tiles && ok; t += n_clusters) {
        const int as = tc & 1;
        const uint32_t aph = (uint32_t)(tc >> 1) & 1u;
        if (!mbar_wait_bounded(&tempty[as], aph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(as * BN);
        for (int u = 0; u < nunits; ++u) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int cnt = unit_kbs(u);
#pragma unroll
          for (int i = 0; i < KPS; ++i) {
            if (i < cnt) {
              const uint64_t adesc = make_sw128_desc(smem_u32(sA + s * Cf::A_BYTES + i * Cf::A_KB));
              const uint64_t bdesc = make_sw128_desc(smem_u32(sB + s * Cf::B_BYTES + i * Cf::B_KB));
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                tc_mma_bf16_pair(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                                 (u | i | k) != 0 ? 1u : 0u);
            }
          }
          tc_commit_pair(&empty[s]);
          ++it;
        }
        if (!ok) break;
        tc_commit_pair(&tfull[as]);
        ++tc;
      }
      if (!ok) {
        if (!*abort_flag) vla_record_error(VLA_DERR_GEMM_MMA_TIMEOUT);
        *abort_flag = 1;
      }
    }
  } else {
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;
    const uint32_t leader_tempty0 = map_to_rank(smem_u32(&tempty[0]), 0);
    const uint32_t leader_tempty1 = map_to_rank(smem_u32(&tempty[1]), 0);
    EpiStore es{smem_u32(sC) + (uint32_t)((warp - 2) * 2 * kStageC), 0, 0, rbar + 2 * (warp - 2), 0u, abort_flag};
    int tc = 0;
    for (int t = cluster; t < num_tiles; t += n_clusters) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const int as = tc & 1;
      const uint32_t aph = (uint32_t)(tc >> 1) & 1u;
      bool ok = mbar_wait_bounded(&tfull[as], aph, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) {
          if (!*abort_flag) vla_record_error(VLA_DERR_GEMM_EPILOGUE_TIMEOUT);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      const int m = mb * 2 * BM + (int)rank * BM + q * 32 + lane;
      es.row0 = mb * 2 * BM + (int)rank * BM + q * 32;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(as * BN);
      epilogue_tile<BN>(ep, taddr, m, nb * BN, part, kEpiWarps / 4, &tmC, &tmR, es, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_relaxed(as ? leader_tempty1 : leader_tempty0);
      ++tc;
    }
    if (ep.tma_c) stage_drain(lane);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the pair's MMAs or signals may still touch it
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"((uint32_t)Cf::TMEM_COLS)
                 : "memory");
  }
}

}  // namespace gemm
}  // namespace vla
