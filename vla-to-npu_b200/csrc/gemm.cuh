// Persistent, warp-specialised bf16 GEMM for sm_100a.
//
//   C[M, N] = epilogue(A[M, K] . B[N, K]^T)
//
// warp 0      : TMA producer (one elected lane) filling a STAGES-deep ring of
//               128x64 A tiles and BNx64 B tiles (128-byte swizzle)
// warp 1      : TMEM allocator + single-thread tcgen05.mma issuer
//               (UMMA 128 x BN x 16, fp32 accumulators in tensor memory,
//               double-buffered so the epilogue of tile i overlaps the
//               mainloop of tile i+1)
// warps 2..5  : epilogue — tcgen05.ld 32 lanes x 16 columns, fused bias /
//               GELU-tanh / SwiGLU / RoPE / Euler / residual, bf16 stores.
//
// This is the replacement for the reference's Allo GEMM module plus the host
// loops that sum its bf16 K-chunks (vla/text_encoder_bf16.py:583-590,
// vla/vision_block_bf16.py:406-416): the whole K reduction stays in fp32 TMEM.
#pragma once
#include "common.cuh"
#include "vla_b200.h"

namespace vla {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpiWarps = 8;                 // two warps per TMEM lane quarter, splitting the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kGroupM = 16;  // tile raster: groups of 16 M-blocks sweep all N-blocks

struct DevEpi {
  bf16* C;
  long long ldc;
  const bf16* bias;
  const bf16* residual;
  long long ldr;
  int res_row_mod;
  int act;
  float alpha;
  const float* rope_cs;
  int rope_seq;
  int rope_ncols;
  int out_grp;
  long long out_grp_stride;
  float* euler_x;
  long long ldx;
  float euler_dt;
  int M, N;
};

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN <= 64) ? 8 : (BN <= 128 ? 6 : 4);
  static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 256 + 1024;
  static_assert(BN % 16 == 0 && BN >= 32 && BN <= 256, "UMMA N");
  static_assert(B_BYTES % 1024 == 0, "B tile alignment");
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int group_size = kGroupM * num_n;
  const int g = t / group_size;
  const int first_m = g * kGroupM;
  const int gm = min(num_m - first_m, kGroupM);
  const int r = t - g * group_size;
  mb = first_m + r % gm;
  nb = r / gm;
}

__device__ __forceinline__ long long out_row(const DevEpi& ep, int m) {
  if (ep.out_grp > 0) return (long long)(m / ep.out_grp) * ep.out_grp_stride + (m % ep.out_grp);
  return m;
}

// Finish 16 consecutive columns [n, n+16) of row m held in v[] (fp32).
__device__ __forceinline__ void finish16(const DevEpi& ep, int m, int n, long long orow, float* v, bool row_ok) {
  if (ep.bias != nullptr) {
    float b[16];
    const uint4* bp = reinterpret_cast<const uint4*>(ep.bias + n);
    unpack_bf16x8(__ldg(bp), b);
    unpack_bf16x8(__ldg(bp + 1), b + 8);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] += b[i];
  }
  if (ep.act == VLA_ACT_GELU_TANH) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = gelu_tanh_f(v[i]);
  }
  if (!row_ok) return;
  if (ep.act == VLA_ACT_EULER) {
    float* xp = ep.euler_x + (long long)m * ep.ldx + n;
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      float4 x = *reinterpret_cast<float4*>(xp + i);
      x.x += ep.euler_dt * v[i];
      x.y += ep.euler_dt * v[i + 1];
      x.z += ep.euler_dt * v[i + 2];
      x.w += ep.euler_dt * v[i + 3];
      *reinterpret_cast<float4*>(xp + i) = x;
      v[i] = x.x;
      v[i + 1] = x.y;
      v[i + 2] = x.z;
      v[i + 3] = x.w;
    }
  }
  if (ep.residual != nullptr) {
    const long long rr = ep.res_row_mod > 0 ? (long long)(m % ep.res_row_mod) : (long long)m;
    const uint4* rp = reinterpret_cast<const uint4*>(ep.residual + rr * ep.ldr + n);
    float r[16];
    unpack_bf16x8(rp[0], r);
    unpack_bf16x8(rp[1], r + 8);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] += r[i];
  }
  uint4* cp = reinterpret_cast<uint4*>(ep.C + orow * ep.ldc + n);
  cp[0] = pack_bf16x8(v);
  cp[1] = pack_bf16x8(v + 8);
}

// Epilogue of one 128 x BN accumulator tile for one row m; warps that share a
// lane quarter split the column chunks round-robin (part of nparts).
template <int BN>
__device__ __forceinline__ void epilogue_tile(const DevEpi& ep, uint32_t taddr, int m, int n0, int part,
                                              int nparts) {
  const bool row_ok = m < ep.M;
  const long long orow = out_row(ep, m);
  if (ep.act == VLA_ACT_ROPE) {
#pragma unroll 1
    for (int h = 64 * part; h < BN; h += 64 * nparts) {
      float x[64];
#pragma unroll
      for (int j = 0; j < 4; ++j) tmem_ld16(taddr + h + 16 * j, x + 16 * j);
      const int n = n0 + h;
      if (n >= ep.N) continue;
#pragma unroll
      for (int i = 0; i < 64; ++i) x[i] *= ep.alpha;
      if (ep.bias != nullptr) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float b[8];
          unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(ep.bias + n) + j), b);
#pragma unroll
          for (int i = 0; i < 8; ++i) x[8 * j + i] += b[i];
        }
      }
      if (n < ep.rope_ncols && row_ok) {
        const float* cs = ep.rope_cs + (long long)(m % ep.rope_seq) * 64;
#pragma unroll
        for (int d = 0; d < 32; ++d) {
          const float c = __ldg(cs + d), s = __ldg(cs + 32 + d);
          const float a = x[d], b = x[d + 32];
          x[d] = a * c - b * s;
          x[d + 32] = b * c + a * s;
        }
      }
      if (!row_ok) continue;
      if (ep.residual != nullptr) {
        const long long rr = ep.res_row_mod > 0 ? (long long)(m % ep.res_row_mod) : (long long)m;
        const uint4* rp = reinterpret_cast<const uint4*>(ep.residual + rr * ep.ldr + n);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float r[8];
          unpack_bf16x8(rp[j], r);
#pragma unroll
          for (int i = 0; i < 8; ++i) x[8 * j + i] += r[i];
        }
      }
      uint4* cp = reinterpret_cast<uint4*>(ep.C + orow * ep.ldc + n);
#pragma unroll
      for (int j = 0; j < 8; ++j) cp[j] = pack_bf16x8(x + 8 * j);
    }
  } else if (ep.act == VLA_ACT_SWIGLU) {
#pragma unroll 1
    for (int c = 32 * part; c < BN; c += 32 * nparts) {
      float g[16], u[16];
      tmem_ld16(taddr + c, g);
      tmem_ld16(taddr + c + 16, u);
      const int n = n0 + c;
      if (n >= ep.N || !row_ok) continue;
#pragma unroll
      for (int i = 0; i < 16; ++i) g[i] = silu_f(g[i] * ep.alpha) * (u[i] * ep.alpha);
      const int nc = n >> 1;
      if (ep.residual != nullptr) {
        const long long rr = ep.res_row_mod > 0 ? (long long)(m % ep.res_row_mod) : (long long)m;
        const uint4* rp = reinterpret_cast<const uint4*>(ep.residual + rr * ep.ldr + nc);
        float r[16];
        unpack_bf16x8(rp[0], r);
        unpack_bf16x8(rp[1], r + 8);
#pragma unroll
        for (int i = 0; i < 16; ++i) g[i] += r[i];
      }
      uint4* cp = reinterpret_cast<uint4*>(ep.C + orow * ep.ldc + nc);
      cp[0] = pack_bf16x8(g);
      cp[1] = pack_bf16x8(g + 8);
    }
  } else {
#pragma unroll 1
    for (int c = 32 * part; c < BN; c += 32 * nparts) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float v[16];
        tmem_ld16(taddr + c + 16 * half, v);
        const int n = n0 + c + 16 * half;
        if (n >= ep.N) continue;
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] *= ep.alpha;
        finish16(ep, m, n, orow, v, row_ok);
      }
    }
  }
}


template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, DevEpi ep,
                        int M, int N, int K) {
  using Cf = Cfg<BN>;
  constexpr int STAGES = Cf::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + STAGES * Cf::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cf::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 32 * kEpiWarps);
    }
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cf::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
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
      // Let the copies already issued land before the CTA can exit.
      const int first = it > STAGES ? it - STAGES : 0;
      for (int j = first; j < it; ++j)
        mbar_wait_bounded(&full[j % STAGES], (uint32_t)(j / STAGES) & 1u, nullptr, 20000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
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
        const uint32_t d_tmem = tmem_base + (uint32_t)(as * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
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
          for (int k = 0; k < BK / 16; ++k) {
            // +32 bytes along K inside the 128-byte swizzle atom = +2 in the address field
            tc_mma_bf16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc, (kb | k) != 0 ? 1u : 0u);
          }
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
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int part = (warp - 2) >> 2;     // which column share of that quarter
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
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(as * BN);
      epilogue_tile<BN>(ep, taddr, m, nb * BN, part, kEpiWarps / 4);
      tc_fence_before();
      mbar_arrive(&tempty[as]);
      ++tc;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cf::TMEM_COLS);
  }
}

}  // namespace gemm
}  // namespace vla
