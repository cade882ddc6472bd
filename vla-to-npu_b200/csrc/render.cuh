// PushT scene rasteriser: the camera of the closed-loop demo, drawn on the GPU
// straight into uint8 frames (the model's camera input), one thread per pixel.
// Scene per environment (fp32 [8]): end effector x, y; block x, y, theta;
// target x, y, theta, in a 512 x 512 workspace with y pointing up (row 0 is
// y = 512).  Layers, back to front: background, target T outline (2-unit band
// around the target's boundary), block T (1.5-unit darker boundary band), end
// effector disc of radius 15 (1.5-unit darker rim).  The T is the union of a
// bar (80 x 30, centred) and a stem (15 wide, 32 long) below it.
#pragma once
#include "common.cuh"

namespace vla {
namespace render {

constexpr float kWorkspace = 512.f;
constexpr float kHalfBarW = 40.f, kHalfBarH = 15.f, kHalfStemW = 7.5f, kStemLen = 32.f, kEeR = 15.f;

// Point (u, v) in the T's own frame, the T grown by `grow` units (negative: shrunk).
__device__ __forceinline__ bool in_t(float u, float v, float grow) {
  const bool bar = fabsf(u) <= kHalfBarW + grow && fabsf(v) <= kHalfBarH + grow;
  // the stem is extended up through the bar so that shrinking keeps the joint inside
  const bool stem = fabsf(u) <= kHalfStemW + grow && v >= -kHalfBarH - kStemLen - grow && v <= kHalfBarH + grow;
  return bar || stem;
}

__device__ __forceinline__ void to_frame(float x, float y, float cx, float cy, float th, float& u, float& v) {
  const float c = cosf(th), s = sinf(th);
  const float dx = x - cx, dy = y - cy;
  u = __fadd_rn(__fmul_rn(c, dx), __fmul_rn(s, dy));
  v = __fsub_rn(__fmul_rn(c, dy), __fmul_rn(s, dx));
}

__global__ void pusht_render_kernel(const float* __restrict__ scene, int n, int S, uint8_t* __restrict__ out) {
  pdl_prologue();
  const long long total = (long long)n * S * S;
  const float scale = kWorkspace / (float)S;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % S);
    const int r = (int)((i / S) % S);
    const long long e = i / ((long long)S * S);
    const float* sc = scene + e * 8;
    const float x = ((float)c + 0.5f) * scale, y = kWorkspace - ((float)r + 0.5f) * scale;
    uint8_t R = 240, G = 240, B = 240;
    float u, v;
    to_frame(x, y, sc[5], sc[6], sc[7], u, v);
    if (in_t(u, v, 1.f) && !in_t(u, v, -1.f)) R = 144, G = 238, B = 144;
    to_frame(x, y, sc[2], sc[3], sc[4], u, v);
    if (in_t(u, v, 0.f)) {
      if (in_t(u, v, -1.5f)) R = 74, G = 144, B = 217;
      else R = 44, G = 95, B = 138;
    }
    const float dx = x - sc[0], dy = y - sc[1];
    const float d2 = __fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy));
    if (d2 <= kEeR * kEeR) {
      if (d2 <= (kEeR - 1.5f) * (kEeR - 1.5f)) R = 255, G = 107, B = 107;
      else R = 204, G = 68, B = 68;
    }
    uint8_t* p = out + i * 3;
    p[0] = R;
    p[1] = G;
    p[2] = B;
  }
}

}  // namespace render
}  // namespace vla
