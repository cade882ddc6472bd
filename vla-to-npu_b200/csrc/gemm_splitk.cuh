// Split-K variant of the persistent tcgen05 GEMM for problems with few output
// tiles (single-observation inference: M = 50 action rows or 113 prefix rows,
// where a 128 x BN tiling of the output gives only tens of tiles and most SMs
// would idle while each busy one streams the whole K extent).
//
// A cluster of S CTAs (S <= 8) owns one output tile at a time; CTA rank r
// computes the tile's product over k-blocks [r * KB / S, (r + 1) * KB / S) with
// the one-CTA machinery of gemm.cuh (TMA ring, single-thread tcgen05.mma into
// TMEM).  The ranks r > 0 then write their fp32 accumulators into the leader's
// (rank 0's) shared memory through distributed shared memory (st.shared::cluster)
// and arrive on a leader barrier with release semantics at cluster scope; the
// leader's epilogue adds those partial tiles to its own accumulator as it reads
// each TMEM chunk (the PS hook of epilogue_tile) and runs the ordinary fused
// epilogue, then signals the ranks that their partial slots are free again.
// No global scratch, no second kernel; the reduction order (leader's partial,
// then ranks 1..S-1) is fixed, so results are deterministic.
#pragma once
#include "gemm2.cuh"

namespace vla {
namespace gemm {

constexpr int kMaxSplit = 8;
constexpr int kMaxStagesS = 8;  // barrier slots reserved for the stage ring

template <int BN>
struct CfgS {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int ROW_FLOATS = BN + 4;                // padded row: 16-byte loads hit distinct banks
  static constexpr int SLOT_BYTES = BM * ROW_FLOATS * 4;   // one rank's partial tile
  static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static_assert(BN == 32 || BN == 64 || BN == 128, "split-K tile widths");
  // smem: stages | epilogue staging | partial slots | barriers
  static constexpr int fixed_bytes(int slots) { return kEpiStoreBytes + slots * SLOT_BYTES + kBarrierBytes + 1024; }
  static constexpr int stages_for(int slots) {
    return (kSmemLimit - fixed_bytes(slots)) / STAGE_BYTES > 6 ? 6 : (kSmemLimit - fixed_bytes(slots)) / STAGE_BYTES;
  }
  static constexpr int smem_bytes(int slots) { return stages_for(slots) * STAGE_BYTES + fixed_bytes(slots); }
};

// The leader's view of the other ranks' partial tiles (its own shared memory).
struct SmemPartial {
  uint32_t base;    // slot 0, row 0 of this thread's tile
  uint32_t row_off; // this thread's row
  uint32_t slot_bytes;
  int nslots;
  __device__ __forceinline__ void add16(int col, float* v) const {
    for (int s = 0; s < nslots; ++s) {
      const uint32_t a = base + (uint32_t)s * slot_bytes + row_off + (uint32_t)col * 4u;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float4 f;
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(f.x), "=f"(f.y), "=f"(f.z), "=f"(f.w)
                     : "r"(a + 16u * i));
        v[4 * i] += f.x;
        v[4 * i + 1] += f.y;
        v[4 * i + 2] += f.z;
        v[4 * i + 3] += f.w;
      }
    }
  }
};

__device__ __forceinline__ void mbar_arrive_release_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

// Bounded wait with acquire semantics at cluster scope (the arrivals come from
// other CTAs of the cluster and order their distributed shared memory writes).
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t a = smem_u32(bar);
  auto try_once = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (try_once()) return true;
  const uint64_t t0 = vla_globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (try_once()) return true;
    if ((i & 255u) == 0u) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (vla_globaltimer() - t0 > VLA_WAIT_LIMIT_NS) return false;
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_splitk_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR,
                            DevEpi ep, int M, int N, int K, int S, int STAGES) {
  using Cf = CfgS<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + STAGES * Cf::A_BYTES;
  uint8_t* sC = sB + STAGES * Cf::B_BYTES;  // output staging (1024-byte aligned)
  uint8_t* sP = sC + kEpiStoreBytes;        // partial slots (leader only)
  uint64_t* full = reinterpret_cast<uint64_t*>(sP + (S - 1) * Cf::SLOT_BYTES);
  uint64_t* empty = full + kMaxStagesS;
  uint64_t* tfull = empty + kMaxStagesS;
  uint64_t* tempty = tfull + 2;
  uint64_t* rbar = tempty + 2;               // [kEpiWarps][2]
  uint64_t* pfull = rbar + 2 * kEpiWarps;    // leader: partials of the current tile have arrived
  uint64_t* pfree = pfull + 1;               // ranks > 0: the leader has consumed the previous partial
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pfree + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int cluster = blockIdx.x / S;
  const int n_clusters = gridDim.x / S;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  const int kb0 = (int)rank * num_kb / S, kb1 = ((int)rank + 1) * num_kb / S;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 32 * kEpiWarps);
    }
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&rbar[i], 1);
    mbar_init(pfull, (uint32_t)((S - 1) * kEpiWarps));
    mbar_init(pfree, (uint32_t)kEpiWarps);
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (ep.tma_c) tma_prefetch_desc(&tmC);
    if (ep.tma_r) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cf::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  cluster_sync();  // every rank's barriers exist before any remote arrive
  pdl_prologue();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = cluster; t < num_tiles && ok; t += n_clusters) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        for (int kb = kb0; kb < kb1; ++kb) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cf::STAGE_BYTES);
          tma_load_2d(sA + s * Cf::A_BYTES, &tmA, &full[s], kb * BK, mb * BM);
          tma_load_2d(sB + s * Cf::B_BYTES, &tmB, &full[s], kb * BK, nb * BN);
          ++it;
        }
      }
      if (!ok) {
        if (!*abort_flag) vla_record_error(VLA_DERR_GEMM_PRODUCER_TIMEOUT);
        *abort_flag = 1;
      }
      const int first = it > STAGES ? it - STAGES : 0;
      for (int j = first; j < it; ++j)
        mbar_wait_bounded(&full[j % STAGES], (uint32_t)(j / STAGES) & 1u, nullptr, 20000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN);
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
        for (int kb = kb0; kb < kb1; ++kb) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = make_sw128_desc(smem_u32(sA + s * Cf::A_BYTES));
          const uint64_t bdesc = make_sw128_desc(smem_u32(sB + s * Cf::B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma_bf16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                        (kb != kb0 || k != 0) ? 1u : 0u);
          tc_commit(&empty[s]);
          ++it;
        }
        if (!ok) break;
        tc_commit(&tfull[as]);
        ++tc;
      }
      if (!ok) {
        if (!*abort_flag) vla_record_error(VLA_DERR_GEMM_MMA_TIMEOUT);
        *abort_flag = 1;
      }
    }
  } else {
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int part = (warp - 2) >> 2;  // which column share of that quarter
    const int row = q * 32 + lane;     // this thread's tile row
    EpiStore es{smem_u32(sC) + (uint32_t)((warp - 2) * 2 * kStageC), 0, 0, rbar + 2 * (warp - 2), 0u, abort_flag};
    // the leader's partial area, as seen from this CTA (rank r writes slot r - 1)
    const uint32_t leader_slots = map_to_rank(smem_u32(sP), 0);
    const uint32_t leader_pfull = map_to_rank(smem_u32(pfull), 0);
    int tc = 0;
    bool ok = true;
    for (int t = cluster; t < num_tiles; t += n_clusters) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const int as = tc & 1;
      const uint32_t aph = (uint32_t)(tc >> 1) & 1u;
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(&tfull[as], aph, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(as * BN);
      if (rank == 0) {
        // every rank's partial of this tile is in our shared memory
        ok = __all_sync(0xffffffffu, mbar_wait_cluster_bounded(pfull, (uint32_t)tc & 1u, abort_flag));
        if (!ok) break;
        const int m = mb * BM + row;
        es.row0 = mb * BM + q * 32;
        const SmemPartial ps{smem_u32(sP), (uint32_t)(row * Cf::ROW_FLOATS * 4), (uint32_t)Cf::SLOT_BYTES, S - 1};
        epilogue_tile<BN, SmemPartial>(ep, taddr, m, nb * BN, part, kEpiWarps / 4, &tmC, &tmR, es, lane, ps);
        // this warp has read its share of the partial slots: let the ranks refill them
        __syncwarp();
        if (lane == 0)
          for (uint32_t r = 1; r < (uint32_t)S; ++r) mbar_arrive_release_cluster(map_to_rank(smem_u32(pfree), r));
      } else {
        // slot rank-1 of the leader must be free (the leader read the previous tile's partial)
        ok = __all_sync(0xffffffffu, mbar_wait_cluster_bounded(pfree, ((uint32_t)tc & 1u) ^ 1u, abort_flag));
        if (!ok) break;
        const uint32_t dst = leader_slots + (rank - 1) * (uint32_t)Cf::SLOT_BYTES + (uint32_t)(row * Cf::ROW_FLOATS * 4);
#pragma unroll 1
        for (int c = 32 * part; c < BN; c += 32 * (kEpiWarps / 4)) {
          float v[32];
          tmem_ld16(taddr + c, v);
          tmem_ld16(taddr + c + 16, v + 16);
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst + (uint32_t)(c + i) * 4u),
                         "f"(v[i]), "f"(v[i + 1]), "f"(v[i + 2]), "f"(v[i + 3])
                         : "memory");
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_release_cluster(leader_pfull);
      }
      tc_fence_before();
      mbar_arrive(&tempty[as]);
      ++tc;
    }
    if (!ok && lane == 0) {
      if (!*abort_flag) vla_record_error(VLA_DERR_GEMM_EPILOGUE_TIMEOUT);
      *abort_flag = 1;
    }
    if (ep.tma_c && rank == 0) stage_drain(lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cf::TMEM_COLS);
  }
  cluster_sync();  // no rank leaves while a peer may still touch its shared memory
}

}  // namespace gemm
}  // namespace vla
