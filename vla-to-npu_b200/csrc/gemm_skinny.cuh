// One-CTA tcgen05 GEMM for skinny problems (one row tile: M <= 64 rows, one
// observation's action rows, copied as 64-row boxes; or M <= 128, its prefix
// tokens, as 128-row boxes), whose time is the per-k-block cost of the main loop.
//
// Measured on B200 with the one-k-block-per-stage ring of gemm.cuh at M = 50:
// a launch costs ~3 us plus ~530 SM cycles per 64-wide k-block whatever the
// ring depth (4, 8 or 16 stages), tile width (32 or 64) or where the operands
// sit (L2 or HBM).  The pace is set by fixed per-stage costs, not bandwidth:
// each barrier round trip and each TMA instruction of the producer (~210
// cycles for a stage of one box, ~75 per further box), and on the issuer side
// the wait, fence and commit around four 128 x BN x 16 MMAs (~46 cycles each
// at BN <= 64, the instruction's own floor).
//
// Here a stage carries KPS = 4 consecutive k-blocks, fetched with ONE
// three-dimensional TMA box per operand: the tensor map views a row-major
// [rows, K] matrix as (64 columns, rows, K / 64 k-blocks) with strides
// (ld * 2 bytes, 128 bytes), so a (64, R, 4) box lands in shared memory as four
// consecutive R x 128-byte tiles in the 128-byte swizzle (R a multiple of 8:
// each tile starts on a 1024-byte boundary), exactly what four single-k-block
// stages would hold.  One barrier wait, one commit and two TMA instructions
// then serve 16 MMAs: ~300 cycles per k-block in the same measurement.  The
// k-blocks of a partial unit (K not a multiple of 256, or a K tail that is
// not a whole k-block) use the two-dimensional maps, one box per k-block, with
// TMA's zero fill past K.
//
// Roles, epilogue, weight prefetch ahead of the launch-overlap wait and the
// error handling are those of gemm_bf16_tc_kernel.
#pragma once
#include "gemm.cuh"

namespace vla {
namespace gemm {

constexpr int kSkinnyRows = 64;  // A rows of every copy for M <= 64; M <= 128 copies 128 rows
constexpr int kSkinnyKps = 4;    // k-blocks per stage

template <int BN, int AR, int KPS_ = kSkinnyKps>
struct CfgK {
  static constexpr int KPS = KPS_;
  static constexpr int A_KB = AR * BK * 2;  // 8 or 16 KB
  static constexpr int B_KB = BN * BK * 2;
  static constexpr int A_UNIT = KPS * A_KB;
  static constexpr int B_UNIT = KPS * B_KB;
  static constexpr int UNIT_BYTES = A_UNIT + B_UNIT;
  static constexpr int BUDGET = kSmemLimit - 1024 - kBarrierBytes - kEpiStoreBytes;
  static constexpr int STAGES = (BUDGET / UNIT_BYTES) > 4 ? 4 : (BUDGET / UNIT_BYTES);
  static constexpr int TMEM_COLS = Cfg<BN>::TMEM_COLS;
  static constexpr int SMEM_BYTES = STAGES * UNIT_BYTES + kEpiStoreBytes + kBarrierBytes + 1024;

  static_assert(A_UNIT % 1024 == 0 && B_UNIT % 1024 == 0, "unit alignment");
};

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Second accumulator of a DUAL launch, added to each TMEM chunk the epilogue
// loads (the partial-sum hook of epilogue_tile).
struct TmemPartial {
  uint32_t base2;  // TMEM address of the second accumulator (this warp's lanes)
  __device__ __forceinline__ void add16(int c, float* v) const {
    float w[16];
    tmem_ld16(base2 + (uint32_t)c, w);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] += w[i];
  }
};

// tmA / tmB: two-dimensional maps (64 x 64-row and 64 x BN boxes) for partial
// units; tmA3 / tmB3: the k-slab maps (64, rows, K / 64) with (64, R, KPS) boxes.
// DUAL: two threads issue the MMAs, warp 1 the even units into one
// accumulator, lane 0 of epilogue warp 2 the odd units into a second one
// (before it joins the epilogue), and the epilogue adds the two.  At these
// tile sizes one thread's issue cost (~46 cycles per MMA plus the wait, fence
// and commit of every unit) sets the main loop's pace.  The host uses it only
// for one tile per CTA and at least two units.
template <int BN, int AR, int KPS_ = kSkinnyKps, bool DUAL = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_skinny_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmA3, const __grid_constant__ CUtensorMap tmB3,
                            const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR, DevEpi ep,
                            int M, int N, int K) {
  using Cf = CfgK<BN, AR, KPS_>;
  constexpr int NACC = DUAL ? 2 : 1;  // accumulators per tile
  constexpr int TCOLS = !DUAL ? Cf::TMEM_COLS : (4 * BN <= 128) ? 128 : (4 * BN <= 256) ? 256 : 512;
  static_assert(!DUAL || 4 * BN <= 512, "DUAL: four BN-wide accumulators");
  constexpr int STAGES = Cf::STAGES;
  static_assert(STAGES >= 2, "unit GEMM: two stages must fit");
  constexpr int KPS = Cf::KPS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // With 64-row copies (AR = 64) the MMA reads 128 A rows from each tile: the
  // upper 64 come from the next tile (the last one's from the B units); those
  // rows only produce accumulator rows >= 64 > M, which are never stored.
  uint8_t* sA = base;
  uint8_t* sB = base + STAGES * Cf::A_UNIT;
  uint8_t* sC = sB + STAGES * Cf::B_UNIT;
  uint64_t* full = reinterpret_cast<uint64_t*>(sC + kEpiStoreBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* rbar = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 2 * kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  const int nfull = K / BK;  // k-blocks entirely inside K (the k-slab maps' depth)
  const int nunits = (num_kb + KPS - 1) / KPS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], NACC);
      mbar_init(&tempty[i], 32 * kEpiWarps);
    }
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&rbar[i], 1);
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmA3);
    tma_prefetch_desc(&tmB3);
    if (ep.tma_c) tma_prefetch_desc(&tmC);
    if (ep.tma_r) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // k-blocks of unit u, and whether one k-slab box per operand covers them
  auto unit_kbs = [&](int u) { return min(KPS, num_kb - u * KPS); };
  auto unit_slab = [&](int u) { return u * KPS + KPS <= nfull; };
  auto unit_tx = [&](int u) { return (uint32_t)((unit_slab(u) ? KPS : unit_kbs(u)) * (Cf::A_KB + Cf::B_KB)); };
  auto load_a = [&](int s, int u, int mb) {
    uint8_t* dst = sA + s * Cf::A_UNIT;
    if (unit_slab(u)) {
      tma_load_3d(dst, &tmA3, &full[s], 0, mb * BM, u * KPS);
    } else {
      for (int i = 0; i < unit_kbs(u); ++i) tma_load_2d(dst + i * Cf::A_KB, &tmA, &full[s], (u * KPS + i) * BK, mb * BM);
    }
  };
  auto load_b = [&](int s, int u, int nb) {
    uint8_t* dst = sB + s * Cf::B_UNIT;
    if (unit_slab(u)) {
      tma_load_3d(dst, &tmB3, &full[s], 0, nb * BN, u * KPS);
    } else {
      for (int i = 0; i < unit_kbs(u); ++i) tma_load_2d(dst + i * Cf::B_KB, &tmB, &full[s], (u * KPS + i) * BK, nb * BN);
    }
  };

  // weights of the first tile's first units before waiting for the previous kernel
  int prefetched = 0;
  if (warp == 0 && lane == 0 && ep.b_static && (int)blockIdx.x < num_tiles) {
    int mb, nb;
    tile_coords(blockIdx.x, num_m, num_n, mb, nb);
    for (; prefetched < STAGES && prefetched < nunits; ++prefetched) {
      mbar_arrive_expect_tx(&full[prefetched], unit_tx(prefetched));
      load_b(prefetched, prefetched, nb);
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // MMA issuing of accumulator h: the units u with u % NACC == h of every tile
  auto issue = [&](int h) {
    constexpr uint32_t idesc = make_idesc_bf16(BM, BN);
    int it = 0, tc = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      const int as = tc & 1;
      const uint32_t aph = (uint32_t)(tc >> 1) & 1u;
      if (!mbar_wait_bounded(&tempty[as], aph ^ 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)((as * NACC + h) * BN);
      for (int u = 0; u < nunits; ++u, ++it) {
        if (u % NACC != h) continue;
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
            const uint64_t adesc = make_sw128_desc(smem_u32(sA + s * Cf::A_UNIT + i * Cf::A_KB));
            const uint64_t bdesc = make_sw128_desc(smem_u32(sB + s * Cf::B_UNIT + i * Cf::B_KB));
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              tc_mma_bf16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                          ((u / NACC) | i | k) != 0 ? 1u : 0u);
          }
        }
        tc_commit(&empty[s]);
      }
      if (!ok) break;
      tc_commit(&tfull[as]);
      ++tc;
    }
    if (!ok) {
      if (!*abort_flag) vla_record_error(VLA_DERR_GEMM_MMA_TIMEOUT);
      *abort_flag = 1;
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        for (int u = 0; u < nunits; ++u) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (it < prefetched) {
            load_a(s, u, mb);
            ++it;
            continue;
          }
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], unit_tx(u));
          load_a(s, u, mb);
          load_b(s, u, nb);
          ++it;
        }
      }
      if (!ok) {
        if (!*abort_flag) vla_record_error(VLA_DERR_GEMM_PRODUCER_TIMEOUT);
        *abort_flag = 1;
      }
      const int issued = it > prefetched ? it : prefetched;
      const int first = issued > STAGES ? issued - STAGES : 0;
      for (int j = first; j < issued; ++j)
        mbar_wait_bounded(&full[j % STAGES], (uint32_t)(j / STAGES) & 1u, nullptr, 20000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) issue(0);
  } else {
    if (DUAL && warp == 2 && lane == 0) issue(1);
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;
    EpiStore es{smem_u32(sC) + (uint32_t)((warp - 2) * 2 * kStageC), 0, 0, rbar + 2 * (warp - 2), 0u, abort_flag};
    int tc = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
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
      const int m = mb * BM + q * 32 + lane;
      es.row0 = mb * BM + q * 32;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(as * NACC * BN);
      if constexpr (DUAL)
        epilogue_tile<BN>(ep, taddr, m, nb * BN, part, kEpiWarps / 4, &tmC, &tmR, es, lane,
                          TmemPartial{taddr + (uint32_t)BN});
      else
        epilogue_tile<BN>(ep, taddr, m, nb * BN, part, kEpiWarps / 4, &tmC, &tmR, es, lane);
      tc_fence_before();
      mbar_arrive(&tempty[as]);
      ++tc;
    }
    if (ep.tma_c) stage_drain(lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TCOLS);
  }
}

}  // namespace gemm
}  // namespace vla
