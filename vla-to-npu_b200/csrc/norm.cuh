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
template <int MODE>
__global__ void __launch_bounds__(kWarps * 32) rownorm_kernel(const bf16* __restrict__ x, long long ldx,
                                                              const bf16* __restrict__ g, const bf16* __restrict__ b,
                                                              bf16* __restrict__ y, long long ldy, int M, int N,
                                                              float eps) {
  pdl_prologue();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kWarps + warp;
  if (row >= M) return;
  const int nvec = N >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  uint4* yr = reinterpret_cast<uint4*>(y + row * ldy);
  const uint4* gv = reinterpret_cast<const uint4*>(g);
  const uint4* bv = reinterpret_cast<const uint4*>(b);
  const float inv_n = 1.f / (float)N;

  if (nvec <= 32 * kMaxVec) {
    float v[kMaxVec][8];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        unpack_bf16x8(xr[c], v[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) s += MODE == 0 ? v[i][j] * v[i][j] : v[i][j];
      }
    }
    s = warp_sum(s);
    float mean = 0.f, rs;
    if (MODE == 0) {
      rs = rsqrtf(s * inv_n + eps);
    } else {
      mean = s * inv_n;
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i) {
        const int c = lane + 32 * i;
        if (c < nvec) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float d = v[i][j] - mean;
            q += d * d;
          }
        }
      }
      q = warp_sum(q);
      rs = rsqrtf(q * inv_n + eps);
    }
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        float gg[8], o[8];
        unpack_bf16x8(__ldg(gv + c), gg);
        if (MODE == 0) {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = (v[i][j] * rs) * gg[j];
        } else {
          float bb[8];
          unpack_bf16x8(__ldg(bv + c), bb);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = (v[i][j] - mean) * rs * gg[j] + bb[j];
        }
        yr[c] = pack_bf16x8(o);
      }
    }
  } else {
    // wide rows: statistics pass, then a normalise pass re-reading the row (L1/L2 hit)
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
}

}  // namespace norm
}  // namespace vla
