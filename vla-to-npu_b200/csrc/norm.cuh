// Row normalisation kernels: RMSNorm and LayerNorm over bf16 rows, fp32
// statistics, one warp per row, 16-byte vector loads, warp-shuffle
// reductions.  HBM-bound: each row is read once and written once.
//
// Replace the reference's AIE kernels rms_norm_960_bf16
// (cc/bf16/rms_norm_960_bf16.cc:18-62), rms_norm_bf16
// (cc/bf16_old/rms_norm_bf16.cc:16-64) and layer_norm_bf16 + bias region
// (cc/bf16_old/layer_norm_bf16.cc:16-70, vla/vision_block_bf16.py:101-127)
// and their host tiling loops (vla/text_encoder_bf16.py:398-404).
#pragma once
#include "common.cuh"

namespace vla {
namespace norm {

constexpr int kWarps = 8;
constexpr int kMaxVec = 4;  // rows up to 32 lanes x 4 x 8 = 1024 elements stay in registers

// mode 0: RMSNorm  y = x * rsqrt(mean(x^2) + eps) * g
// mode 1: LayerNorm y = (x - mean) * rsqrt(var + eps) * g + b
// Normalise one row whose 16-byte vectors stay in registers as packed bf16
// (N <= 1024; 4 registers per 8 values keep the kernel at ~46 registers, so
// more warps are resident to cover the load latency).
// gp / bp: the lane's gain / bias vectors already in registers (or null).
template <int MODE, int R>
__device__ __forceinline__ void norm_rows_reg(const bf16* __restrict__ x, long long ldx, const bf16* __restrict__ g,
                                              const bf16* __restrict__ b, bf16* __restrict__ y, long long ldy,
                                              long long row0, int M, int N, float eps, int lane,
                                              const uint4* gp = nullptr, const uint4* bp = nullptr) {
  const int nvec = N >> 3;
  const float inv_n = 1.f / (float)N;
  uint4 raw[R][kMaxVec];  // rows kept as packed bf16 (4 registers per 8 values)
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const long long row = row0 + r;
    const uint4* xr = reinterpret_cast<const uint4*>(x + (row < M ? row : 0) * ldx);
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = lane + 32 * i;
      raw[r][i] = (c < nvec && row < M) ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  float mean[R], rs[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      if (lane + 32 * i < nvec) {
        float v[8];
        unpack_bf16x8(raw[r][i], v);
#pragma unroll
        for (int j = 0; j < 8; ++j) s += MODE == 0 ? v[j] * v[j] : v[j];
      }
    }
    s = warp_sum(s);
    mean[r] = 0.f;
    if (MODE == 0) {
      rs[r] = rsqrtf(s * inv_n + eps);
    } else {
      mean[r] = s * inv_n;
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i) {
        if (lane + 32 * i < nvec) {
          float v[8];
          unpack_bf16x8(raw[r][i], v);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float d = v[j] - mean[r];
            q += d * d;
          }
        }
      }
      q = warp_sum(q);
      rs[r] = rsqrtf(q * inv_n + eps);
    }
  }
  const uint4* gv = reinterpret_cast<const uint4*>(g);
  const uint4* bv = reinterpret_cast<const uint4*>(b);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      float gg[8], bb[8];
      unpack_bf16x8(gp != nullptr ? gp[i] : __ldg(gv + c), gg);
      if (MODE == 1) unpack_bf16x8(bp != nullptr ? bp[i] : __ldg(bv + c), bb);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const long long row = row0 + r;
        if (row >= M) continue;
        float v[8], o[8];
        unpack_bf16x8(raw[r][i], v);
        if (MODE == 0) {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = (v[j] * rs[r]) * gg[j];
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = (v[j] - mean[r]) * rs[r] * gg[j] + bb[j];
        }
        reinterpret_cast<uint4*>(y + row * ldy)[c] = pack_bf16x8(o);
      }
    }
  }
}

// wide rows (N > 1024): statistics pass, then a normalise pass re-reading the
// row (L1/L2 hit)
template <int MODE>
__device__ __forceinline__ void norm_row_wide(const bf16* __restrict__ x, long long ldx, const bf16* __restrict__ g,
                                              const bf16* __restrict__ b, bf16* __restrict__ y, long long ldy,
                                              long long row, int N, float eps, int lane) {
  const int nvec = N >> 3;
  const float inv_n = 1.f / (float)N;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  uint4* yr = reinterpret_cast<uint4*>(y + row * ldy);
  const uint4* gv = reinterpret_cast<const uint4*>(g);
  const uint4* bv = reinterpret_cast<const uint4*>(b);
  float s = 0.f;
  for (int c = lane; c < nvec; c += 32) {
    float t[8];
    unpack_bf16x8(xr[c], t);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += MODE == 0 ? t[j] * t[j] : t[j];
  }
  s = warp_sum(s);
  float mean = 0.f, rs;
  if (MODE == 0) {
    rs = rsqrtf(s * inv_n + eps);
  } else {
    mean = s * inv_n;
    float q = 0.f;
    for (int c = lane; c < nvec; c += 32) {
      float t[8];
      unpack_bf16x8(xr[c], t);
#pragma unroll
      for (int j = 0; j < 8; ++j) q += (t[j] - mean) * (t[j] - mean);
    }
    q = warp_sum(q);
    rs = rsqrtf(q * inv_n + eps);
  }
  for (int c = lane; c < nvec; c += 32) {
    float t[8], gg[8], o[8];
    unpack_bf16x8(xr[c], t);
    unpack_bf16x8(__ldg(gv + c), gg);
    if (MODE == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (t[j] * rs) * gg[j];
    } else {
      float bb[8];
      unpack_bf16x8(__ldg(bv + c), bb);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (t[j] - mean) * rs * gg[j] + bb[j];
    }
    yr[c] = pack_bf16x8(o);
  }
}

// MODE 0 = RMSNorm, 1 = LayerNorm; one warp per row, the grid striding over
// the rows.  STATIC: g and b are weights no earlier kernel in the stream
// writes, so rows of at most 1024 take them into registers before waiting for
// the previous kernel (their load latency overlaps its tail).
template <int MODE, bool STATIC>
__global__ void __launch_bounds__(kWarps * 32) rownorm_kernel(const bf16* __restrict__ x, long long ldx,
                                                              const bf16* __restrict__ g, const bf16* __restrict__ b,
                                                              bf16* __restrict__ y, long long ldy, int M, int N,
                                                              float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool reg_rows = (N >> 3) <= 32 * kMaxVec;
  uint4 gp[kMaxVec], bp[kMaxVec];
  if (STATIC && reg_rows) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = lane + 32 * i;
      gp[i] = c < (N >> 3) ? __ldg(reinterpret_cast<const uint4*>(g) + c) : make_uint4(0u, 0u, 0u, 0u);
      bp[i] = (MODE == 1 && c < (N >> 3)) ? __ldg(reinterpret_cast<const uint4*>(b) + c) : make_uint4(0u, 0u, 0u, 0u);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
  } else {
    pdl_prologue();
  }
  for (long long row = (long long)blockIdx.x * kWarps + warp; row < M; row += (long long)gridDim.x * kWarps) {
    if (reg_rows)
      norm_rows_reg<MODE, 1>(x, ldx, g, b, y, ldy, row, M, N, eps, lane, STATIC ? gp : nullptr,
                             STATIC ? bp : nullptr);
    else
      norm_row_wide<MODE>(x, ldx, g, b, y, ldy, row, N, eps, lane);
  }
}

}  // namespace norm
}  // namespace vla
