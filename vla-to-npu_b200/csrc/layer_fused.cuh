// One Llama-style layer (text decoder / action-expert block, self or cross
// attention) as ONE persistent cooperative kernel, for the small row counts of
// single-observation inference.
//
// At one observation a layer is seven short dependent kernels (RMSNorm, QKV
// GEMM + RoPE, attention, O GEMM + residual, RMSNorm, gate/up GEMM + SwiGLU,
// down GEMM + residual), each a few microseconds of work behind several
// microseconds of launch-to-launch latency.  Here the seven phases run inside
// one launch of one CTA per SM, separated by grid-wide barriers (an atomic
// counter, bounded spin):
//   norm phases   every warp of the grid normalises rows (norm::norm_rows_reg);
//   GEMM phases   the tcgen05 machinery of gemm.cuh: warp 0 TMA producer, warp 1
//                 single-thread tcgen05.mma into double-buffered TMEM, warps
//                 2..9 the fused epilogue (epilogue_tile: RoPE / residual /
//                 SwiGLU, TMA stores); the stage ring, TMEM accumulators and
//                 barrier phases carry over from phase to phase;
//   attention     warps 2..5 of CTA i run work item i of the short-sequence
//                 tcgen05 attention (the G query heads of a kv head stacked into
//                 128-row tiles, S = Q K^T into TMEM, softmax in registers,
//                 O = P V with P from TMEM), Q / K / V staged with cp.async.
// Between phases each CTA drains its TMA stores, fences (generic and async
// proxies) and arrives on the barrier; after it, the TMA loads of the next phase
// see every CTA's results.  Semantics (and bits) are those of the unfused layer.
// Measured at one observation it is slower than the seven launches (the
// phases' own latency dominates), so the library uses it only on request
// (vla_set_fused_layers).
#pragma once
#include "attention_short.cuh"
#include "gemm.cuh"
#include "norm.cuh"

namespace vla {
namespace lfused {

using gemm::BK;
using gemm::BM;
using gemm::DevEpi;
using gemm::EpiStore;
using gemm::kEpiWarps;
using gemm::kStageC;
using gemm::kThreads;

constexpr int A_BYTES = BM * BK * 2;       // 16 KB
constexpr int B_BYTES = 64 * BK * 2;       // room for BN <= 64
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int STAGES = 6;
constexpr uint32_t TMEM_COLS = 256;        // GEMM accumulators [0, 128), attention [128, 256)
constexpr uint32_t ATT_COL = 128;
constexpr int kAttThreads = 128;           // warps 2..5
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + gemm::kEpiStoreBytes + 1024 /*barriers*/ + 1024 /*align*/;
static_assert(3 * attn_sq::TILE <= STAGES * STAGE_BYTES, "attention tiles alias the stage ring");

struct GemmArgs {
  DevEpi ep;
  int M, N, K;
};

struct Params {
  CUtensorMap a_h, a_attn, a_mlp;         // A operands: normalised rows, attention output, SwiGLU output
  CUtensorMap b_qkv, b_o, b_gu, b_down;   // weights (K-major)
  CUtensorMap c_qkv, c_x, c_mlp, r_x;     // output stores and the residual loads
  GemmArgs g_qkv, g_o, g_gu, g_down;
  const bf16* norm1;
  const bf16* norm2;
  bf16* x;
  bf16* h;
  int rows, H;
  float eps;
  attn_sq::Params att;
  unsigned int* barrier;   // grid barrier counter, zero at launch
};

struct Bars {
  uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2];
  uint64_t rbar[2 * kEpiWarps];
  uint64_t abar;           // attention MMA completion
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Bars) <= 1024, "barrier block");

// Grid-wide barrier number `k` (0-based) of this launch.
__device__ __forceinline__ bool grid_barrier(unsigned int* ctr, unsigned int k, volatile int* abort_flag) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __threadfence();
    atomicAdd(ctr, 1u);
    const unsigned int target = (k + 1) * gridDim.x;
    const uint64_t t0 = vla_globaltimer();
    int ok = 1;
    for (uint32_t i = 0;; ++i) {
      unsigned int v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= target) break;
      if ((i & 63u) == 63u && (*abort_flag || vla_globaltimer() - t0 > VLA_WAIT_LIMIT_NS)) {
        ok = 0;
        break;
      }
    }
    __threadfence();
    s_ok = ok;
  }
  __syncthreads();
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return s_ok != 0;
}

// Persistent-across-phases state of the three GEMM roles.
struct RoleState {
  int it = 0;   // stage ring position (producer and MMA)
  int tc = 0;   // accumulator buffer position (MMA and epilogue)
};

template <int BN>
__device__ __forceinline__ bool gemm_phase(const GemmArgs& g, const CUtensorMap* tA, const CUtensorMap* tB,
                                           const CUtensorMap* tC, const CUtensorMap* tR, uint8_t* base, Bars& bb,
                                           uint32_t tmem_base, RoleState& rs, EpiStore& es) {
  constexpr int B_TILE = BN * BK * 2;
  constexpr uint32_t TX = (uint32_t)(A_BYTES + B_TILE);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &bb.abort;
  const int num_m = (g.M + BM - 1) / BM, num_n = (g.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n, num_kb = (g.K + BK - 1) / BK;
  bool ok = true;
  if (warp == 0) {
    if (lane == 0) {
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        gemm::tile_coords(t, num_m, num_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          const int s = rs.it % STAGES;
          if (!mbar_wait_bounded(&bb.empty[s], ((uint32_t)(rs.it / STAGES) & 1u) ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = base + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&bb.full[s], TX);
          tma_load_2d(st, tA, &bb.full[s], kb * BK, mb * BM);
          tma_load_2d(st + A_BYTES, tB, &bb.full[s], kb * BK, nb * BN);
          ++rs.it;
        }
      }
      if (!ok) vla_record_error(VLA_DERR_GEMM_PRODUCER_TIMEOUT);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN);
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int as = rs.tc & 1;
        if (!mbar_wait_bounded(&bb.tempty[as], ((uint32_t)(rs.tc >> 1) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(as * 64);
        for (int kb = 0; kb < num_kb; ++kb) {
          const int s = rs.it % STAGES;
          if (!mbar_wait_bounded(&bb.full[s], (uint32_t)(rs.it / STAGES) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* st = base + s * STAGE_BYTES;
          const uint64_t adesc = make_sw128_desc(smem_u32(st)), bdesc = make_sw128_desc(smem_u32(st + A_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma_bf16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc, (kb | k) != 0 ? 1u : 0u);
          tc_commit(&bb.empty[s]);
          ++rs.it;
        }
        if (!ok) break;
        tc_commit(&bb.tfull[as]);
        ++rs.tc;
      }
      if (!ok) vla_record_error(VLA_DERR_GEMM_MMA_TIMEOUT);
    }
  } else {
    const int q = warp & 3, part = (warp - 2) >> 2;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int mb, nb;
      gemm::tile_coords(t, num_m, num_n, mb, nb);
      const int as = rs.tc & 1;
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bb.tfull[as], (uint32_t)(rs.tc >> 1) & 1u, abort_flag));
      if (!ok) break;
      tc_fence_after();
      es.row0 = mb * BM + q * 32;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(as * 64);
      gemm::epilogue_tile<BN>(g.ep, taddr, mb * BM + q * 32 + lane, nb * BN, part, kEpiWarps / 4, tC, tR, es, lane);
      tc_fence_before();
      mbar_arrive(&bb.tempty[as]);
      ++rs.tc;
    }
    if (!ok && lane == 0) vla_record_error(VLA_DERR_GEMM_EPILOGUE_TIMEOUT);
    if (g.ep.tma_c) gemm::stage_drain(lane);  // this phase's stores are complete before the barrier
  }
  if (!ok) *abort_flag = 1;
  return ok;
}

// cp.async copy of `nrows` 128-byte rows into a 128-byte-swizzled tile (rows at
// or past `valid` zero-filled); tid in [0, 128).
template <typename RowPtr>
__device__ __forceinline__ void stage_rows128(uint32_t tile, int valid, int tid, RowPtr src) {
  const int c = tid & 7;
#pragma unroll
  for (int i = 0; i < attn_sq::MT / 16; ++i) {
    const int r = (tid >> 3) + 16 * i;
    const bool ok = r < valid;
    const bf16* gp = ok ? src(r) + c * 8 : src(0);
    attn_sq::cp16(tile + (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)), gp, ok);
  }
}

// Attention work items of this CTA on warps 2..5 (tid = threadIdx.x - 64).
template <int NK>
__device__ __forceinline__ bool attention_phase(const attn_sq::Params& p, uint8_t* base, Bars& bb, uint32_t tmem,
                                                uint32_t& phase) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x - 64;
  const int q4 = warp & 3;
  const int row = q4 * 32 + lane;  // TMEM lane of this thread
  const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
  const uint32_t sq = smem_u32(base), sk = sq + attn_sq::TILE, sv = sk + attn_sq::TILE;
  constexpr uint32_t idesc_s = make_idesc_bf16(attn_sq::MT, NK);
  constexpr uint32_t idesc_pv = make_idesc_bf16(attn_sq::MT, attn_sq::HD) | (1u << 16);
  const int n_items = p.batch * p.Hkv * p.n_mt;
  const int G = p.G, Lq = p.Lq, rows_valid = G * Lq;
  const uint32_t tmem_a = tmem + ATT_COL;
  bool ok = true;
  for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
    const attn_sq::Item w = attn_sq::item_at(p, it);
    const bf16* qb = p.q + (long long)w.b * p.q_batch;
    const bf16* kb = p.k + (long long)w.b * p.k_batch + (long long)w.kvh * 64;
    const bf16* vb = p.v + (long long)w.b * p.v_batch + (long long)w.kvh * 64;
    stage_rows128(sq, rows_valid - w.s0, tid, [&](int r) {
      const int s = w.s0 + r;
      return qb + (long long)(s % Lq) * p.q_row + (long long)(w.kvh * G + s / Lq) * 64;
    });
    stage_rows128(sk, w.lk, tid, [&](int r) { return kb + (long long)r * p.k_row; });
    stage_rows128(sv, w.lk, tid, [&](int r) { return vb + (long long)r * p.v_row; });
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    asm volatile("bar.sync 1, %0;" ::"r"(kAttThreads) : "memory");
    tc_fence_after();
    if (tid == 0) {
      const uint64_t qd = make_sw128_desc(sq), kd = make_sw128_desc(sk);
#pragma unroll
      for (int k = 0; k < 4; ++k) tc_mma_bf16(tmem_a, qd + 2 * k, kd + 2 * k, idesc_s, k > 0 ? 1u : 0u);
      tc_commit(&bb.abar);
    }
    ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bb.abar, phase, &bb.abort));
    phase ^= 1u;
    tc_fence_after();
    const int s = w.s0 + row;
    int kend = w.lk;
    if (p.causal) kend = min(kend, s % Lq + 1);
    const uint32_t srow = tmem_a + lane_base;
    float m = -INFINITY;
#pragma unroll
    for (int h = 0; h < NK / 64; ++h) {
      float v[64];
      tmem_ld64(srow + 64 * h, v);
#pragma unroll
      for (int c = 0; c < 64; ++c)
        if (64 * h + c < kend) m = fmaxf(m, v[c]);
    }
    const float mb = m == -INFINITY ? 0.f : m * p.scale_log2;
    float l = 0.f;
#pragma unroll
    for (int h = 0; h < NK / 64; ++h) {
      float v[64];
      tmem_ld64(srow + 64 * h, v);
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float e0 = 64 * h + c < kend ? attn_sq::ex2f(fmaf(v[c], p.scale_log2, -mb)) : 0.f;
        const float e1 = 64 * h + c + 1 < kend ? attn_sq::ex2f(fmaf(v[c + 1], p.scale_log2, -mb)) : 0.f;
        l += e0 + e1;
        pk[c >> 1] = pack_bf16x2(e0, e1);
      }
      attn_sq::tmem_st32u(srow + 32 * h, pk);
    }
    tc_fence_before();
    asm volatile("bar.sync 1, %0;" ::"r"(kAttThreads) : "memory");
    tc_fence_after();
    if (tid == 0 && ok) {
#pragma unroll
      for (int k = 0; k < NK / 16; ++k)
        attn_sq::mma_ts(tmem_a + attn_sq::O_COL, tmem_a + (uint32_t)k * 8u, attn_sq::mn_desc(sv + (uint32_t)k * 2048u),
                        idesc_pv, k > 0 ? 1u : 0u);
      tc_commit(&bb.abar);
    }
    ok = ok && __all_sync(0xffffffffu, mbar_wait_bounded(&bb.abar, phase, &bb.abort));
    phase ^= 1u;
    tc_fence_after();
    {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      float o[64];
      tmem_ld64(srow + attn_sq::O_COL, o);
      const int sr = w.s0 + row;
      if (ok && sr < rows_valid) {
        const int hh = w.kvh * G + sr / Lq;
        bf16* dst = p.o + (long long)w.b * p.o_batch + (long long)(sr % Lq) * p.o_row + (long long)hh * 64;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          float t8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) t8[i] = o[8 * c8 + i] * inv;
          reinterpret_cast<uint4*>(dst)[c8] = pack_bf16x8(t8);
        }
      }
    }
    tc_fence_before();
    asm volatile("bar.sync 1, %0;" ::"r"(kAttThreads) : "memory");
    tc_fence_after();
    if (!ok) break;
  }
  if (!ok && tid == 0) {
    vla_record_error(VLA_DERR_ATTN_TIMEOUT);
    bb.abort = 1;
  }
  return ok;
}

__device__ __forceinline__ void norm_phase(const bf16* x, const bf16* g, bf16* y, int rows, int H, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = kThreads / 32;
  for (int r = blockIdx.x * nw + warp; r < rows; r += gridDim.x * nw)
    norm::norm_rows_reg<0, 1>(x, H, g, nullptr, y, H, r, rows, H, eps, lane);
}

template <int NK>
__global__ void __launch_bounds__(kThreads, 1) llama_layer_fused_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sC = base + STAGES * STAGE_BYTES;
  Bars& bb = *reinterpret_cast<Bars*>(sC + gemm::kEpiStoreBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bb.full[s], 1);
      mbar_init(&bb.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bb.tfull[i], 1);
      mbar_init(&bb.tempty[i], 32 * kEpiWarps);
    }
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&bb.rbar[i], 1);
    mbar_init(&bb.abar, 1);
    bb.abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&bb.tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bb.tmem_base;
  pdl_prologue();
  volatile int* abort_flag = &bb.abort;
  RoleState rs;
  EpiStore es{smem_u32(sC) + (uint32_t)((warp >= 2 ? warp - 2 : 0) * 2 * kStageC), 0, 0,
              bb.rbar + 2 * (warp >= 2 ? warp - 2 : 0), 0u, abort_flag};
  uint32_t att_phase = 0;
  unsigned int nb = 0;  // grid barriers passed
  bool ok = true;
  const int H = p.H;

  // 1. RMSNorm of x into h
  norm_phase(p.x, p.norm1, p.h, p.rows, H, p.eps);
  ok = grid_barrier(p.barrier, nb++, abort_flag);
  // 2. QKV (or Q) GEMM with the RoPE epilogue
  if (ok) ok = gemm_phase<64>(p.g_qkv, &p.a_h, &p.b_qkv, &p.c_qkv, &p.r_x, base, bb, tmem, rs, es);
  ok = grid_barrier(p.barrier, nb++, abort_flag) && ok;
  // 3. attention
  if (ok && warp >= 2 && warp < 6) ok = attention_phase<NK>(p.att, base, bb, tmem, att_phase);
  ok = grid_barrier(p.barrier, nb++, abort_flag) && ok;
  // 4. O GEMM + residual into x
  if (ok) ok = gemm_phase<32>(p.g_o, &p.a_attn, &p.b_o, &p.c_x, &p.r_x, base, bb, tmem, rs, es);
  ok = grid_barrier(p.barrier, nb++, abort_flag) && ok;
  // 5. RMSNorm of x into h
  if (ok) norm_phase(p.x, p.norm2, p.h, p.rows, H, p.eps);
  ok = grid_barrier(p.barrier, nb++, abort_flag) && ok;
  // 6. gate / up GEMM with the SwiGLU epilogue
  if (ok) ok = gemm_phase<32>(p.g_gu, &p.a_h, &p.b_gu, &p.c_mlp, &p.r_x, base, bb, tmem, rs, es);
  ok = grid_barrier(p.barrier, nb++, abort_flag) && ok;
  // 7. down GEMM + residual into x
  if (ok) gemm_phase<32>(p.g_down, &p.a_mlp, &p.b_down, &p.c_x, &p.r_x, base, bb, tmem, rs, es);

  // copies that a failed phase left in flight land before the CTA exits
  if (warp == 0 && lane == 0 && *abort_flag) {
    const int first = rs.it > STAGES ? rs.it - STAGES : 0;
    for (int j = first; j < rs.it; ++j)
      mbar_wait_bounded(&bb.full[j % STAGES], (uint32_t)(j / STAGES) & 1u, nullptr, 20000000ull);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace lfused
}  // namespace vla
