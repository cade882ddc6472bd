// Bandwidth-bound elementwise / layout kernels of the hot path.  Each is a
// grid-stride loop over 16-byte vectors (8 bf16) so that reads and writes are
// fully coalesced; the grid is sized to a multiple of the SM count.
#pragma once
#include "common.cuh"

namespace vla {
namespace ew {

// ---------------------------------------------------------------------------
// RoPE on packed heads, in place: x [M, ld], columns [0, ncols) in 64-wide heads,
// row m has position m % seq.  cs = fp32 table [seq][64] (cos k<32 | sin k<32).
// Replaces rope_apply_packed (vla/text_encoder_bf16.py:422-475) and its ~11
// AIE calls per head and 64-row tile (cc/float/rope_vec_ops.cc:8-95,
// cc/float/sine.cc, cc/float/cosine.cc).
// ---------------------------------------------------------------------------
__global__ void rope_kernel(bf16* __restrict__ x, long long ld, long long M, int ncols, int seq,
                            const float* __restrict__ cs) {
  pdl_prologue();
  // one thread per (row, head, 8-pair group): handles d in [8j, 8j+8) and d+32
  const int groups_per_row = (ncols / 64) * 4;
  const long long total = M * groups_per_row;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / groups_per_row;
    const int r = (int)(i % groups_per_row);
    const int head = r >> 2, j = r & 3;
    bf16* base = x + m * ld + head * 64 + j * 8;
    float a[8], bb[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(base), a);
    unpack_bf16x8(*reinterpret_cast<const uint4*>(base + 32), bb);
    const float* c = cs + (long long)(m % seq) * 64 + j * 8;
    float lo[8], hi[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float co = __ldg(c + e), si = __ldg(c + 32 + e);
      lo[e] = a[e] * co - bb[e] * si;
      hi[e] = bb[e] * co + a[e] * si;
    }
    *reinterpret_cast<uint4*>(base) = pack_bf16x8(lo);
    *reinterpret_cast<uint4*>(base + 32) = pack_bf16x8(hi);
  }
}

// ---------------------------------------------------------------------------
// Row softmax, bf16 in/out, fp32 math; one warp per row.  causal_row_start >= 0
// masks column c of local row r when c > causal_row_start + r (the reference's
// masked_softmax_128_bf16 row_start argument, cc/bf16/masked_softmax_128_bf16.cc:251-398;
// unmasked: cc/bf16_old/v2_softmax_bf16.cc:552-664, cc/float/v1_softmax_float.cc:117-179).
// Masked columns are written as exact zeros.
// ---------------------------------------------------------------------------
__global__ void softmax_kernel(const bf16* __restrict__ x, long long ldx, bf16* __restrict__ y, long long ldy, int M,
                               int N, float scale, int causal_row_start) {
  pdl_prologue();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= M) return;
  const bf16* xr = x + (long long)row * ldx;
  bf16* yr = y + (long long)row * ldy;
  const int limit = causal_row_start >= 0 ? min(N, causal_row_start + row + 1) : N;
  float mx = -INFINITY;
  for (int c = lane; c < limit; c += 32) mx = fmaxf(mx, __bfloat162float(xr[c]) * scale);
  mx = warp_max(mx);
  float s = 0.f;
  for (int c = lane; c < limit; c += 32) s += expf(__bfloat162float(xr[c]) * scale - mx);
  s = warp_sum(s);
  const float inv = s > 0.f ? 1.f / s : 0.f;
  for (int c = lane; c < N; c += 32) {
    const float v = c < limit ? expf(__bfloat162float(xr[c]) * scale - mx) * inv : 0.f;
    yr[c] = __float2bfloat16(v);
  }
}

// ---------------------------------------------------------------------------
// Activations on [M, ld] bf16 (vector path needs N % 8 == 0).
//   op 0: GELU-tanh (cc/bf16_old/gelu_bf16.cc:83-102)
//   op 1: SiLU      (cc/bf16/silu_160_bf16.cc:29-127)
//   op 2: SiLU(x) * y  (silu then the numpy Hadamard, vla/text_encoder_bf16.py:581)
//   op 3: x + y
// ---------------------------------------------------------------------------
__global__ void act_kernel(const bf16* __restrict__ x, long long ldx, const bf16* __restrict__ y2, long long ldy2,
                           bf16* __restrict__ out, long long ldo, long long M, int N, int op) {
  pdl_prologue();
  const int vpr = N >> 3;
  const long long total = M * vpr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / vpr;
    const int c = (int)(i % vpr) * 8;
    float a[8], r[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(x + m * ldx + c), a);
    if (op >= 2) {
      float b[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(y2 + m * ldy2 + c), b);
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = op == 2 ? silu_f(a[e]) * b[e] : a[e] + b[e];
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = op == 0 ? gelu_tanh_f(a[e]) : silu_f(a[e]);
    }
    *reinterpret_cast<uint4*>(out + m * ldo + c) = pack_bf16x8(r);
  }
}

// ---------------------------------------------------------------------------
// Pixel shuffle (scale s) of B images of grid x grid tokens with C channels:
//   out[b, h4*(grid/s) + w4, (h%s)*s*C + (w%s)*C + c] = in[b, h*grid + w, c]
// the reshape/transpose chain of con_ref (vla/vla.py:434-436) and the copy
// regions of fused_op (vla/connector_bf16.py:97-111).  Vectorised over c.
// ---------------------------------------------------------------------------
// I: index type of the vector counter (32-bit when the total fits: the
// divisions below dominate the kernel's cost in 64-bit arithmetic)
template <typename I>
__global__ void pixel_shuffle_kernel(const bf16* __restrict__ in, bf16* __restrict__ out, int B, int grid, int s,
                                     int C) {
  pdl_prologue();
  const int cv = C >> 3;
  const I total = (I)B * grid * grid * cv;
  const int g2 = grid / s;
  for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (I)gridDim.x * blockDim.x) {
    const int c = (int)(i % cv) * 8;
    I tok = i / cv;
    const int w = (int)(tok % grid);
    tok /= grid;
    const int h = (int)(tok % grid);
    const long long b = tok / grid;
    const long long orow = b * g2 * g2 + (h / s) * g2 + (w / s);
    const long long ocol = (long long)(h % s) * s * C + (long long)(w % s) * C + c;
    const uint4 v = *reinterpret_cast<const uint4*>(in + ((b * grid + h) * grid + w) * (long long)C + c);
    *reinterpret_cast<uint4*>(out + orow * ((long long)s * s * C) + ocol) = v;
  }
}

// ---------------------------------------------------------------------------
// Patch im2col (stride == kernel): image [B, Cin, H, W] bf16 ->
// A [B * (H/p) * (W/p), Cin*p*p], column = cin*p*p + ky*p + kx, the order of
// Conv2d weight.reshape(out, -1) (vla/vit_emb.py:199-200;
// cc/bf16_old/conv_bf16.cc:12-55 computes the same dot products per patch).
// Vectorised over 8 consecutive kx.
// ---------------------------------------------------------------------------
template <typename I>
__global__ void im2col_kernel(const bf16* __restrict__ img, bf16* __restrict__ out, int B, int Cin, int H, int W,
                              int p) {
  pdl_prologue();
  const int gh = H / p, gw = W / p;
  const int kdim = Cin * p * p;
  const int vec_per_row = kdim >> 3;
  const I total = (I)B * gh * gw * vec_per_row;
  for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (I)gridDim.x * blockDim.x) {
    const int col = (int)(i % vec_per_row) * 8;
    const I tok = i / vec_per_row;
    const int px = (int)(tok % gw);
    const int py = (int)((tok / gw) % gh);
    const long long b = tok / ((I)gw * gh);
    const int cin = col / (p * p);
    const int ky = (col / p) % p;
    const int kx = col % p;
    const bf16* src = img + ((b * Cin + cin) * H + (py * p + ky)) * (long long)W + px * p + kx;
    *reinterpret_cast<uint4*>(out + (long long)tok * kdim + col) = *reinterpret_cast<const uint4*>(src);
  }
}

// ---------------------------------------------------------------------------
// Token embedding gather with scale (create_text_emb, vla/vla.py:169-174):
//   out[(b*rows_per_seq + row_offset + t), :] = table[ids[b*T + t], :] * scale
// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// Camera frames in: uint8 [B, H, W, 3] (HWC, the usual camera / video layout)
// -> bilinear resize to S x S (half-pixel centres, no antialiasing: the rule of
// torch.nn.functional.interpolate(mode="bilinear", align_corners=False)) ->
// scaled to [-1, 1] as v * 2/255 - 1 -> bf16, written either as the NCHW image
// [B, 3, S, S] (mode 0) or directly as the patch-embedding GEMM's A operand
// [B * (S/p)^2, 3 p p] with column cin*p*p + ky*p + kx (mode 1: resize,
// normalisation and im2col in one pass).  One thread makes 8 horizontally
// adjacent output pixels of one channel (one 16-byte store).
// ---------------------------------------------------------------------------
template <typename I>
__global__ void camera_preprocess_kernel(const uint8_t* __restrict__ img, bf16* __restrict__ out, int B, int H, int W,
                                         int S, int p, int mode, float scale_y, float scale_x) {
  pdl_prologue();
  const int xv = S >> 3;
  const I total = (I)B * 3 * S * xv;
  for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (I)gridDim.x * blockDim.x) {
    const int x0 = (int)(i % xv) * 8;
    const I r = i / xv;
    const int y = (int)(r % S);
    const int c = (int)((r / S) % 3);
    const long long b = (long long)(r / ((I)S * 3));
    float sy = ((float)y + 0.5f) * scale_y - 0.5f;
    sy = sy < 0.f ? 0.f : sy;
    const int y0 = (int)sy;
    const int y1 = y0 + (y0 < H - 1 ? 1 : 0);
    const float ly = sy - (float)y0, hy = 1.f - ly;
    const uint8_t* row0 = img + ((b * H + y0) * (long long)W) * 3 + c;
    const uint8_t* row1 = img + ((b * H + y1) * (long long)W) * 3 + c;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float sx = ((float)(x0 + j) + 0.5f) * scale_x - 0.5f;
      sx = sx < 0.f ? 0.f : sx;
      const int xa = (int)sx;
      const int xb = xa + (xa < W - 1 ? 1 : 0);
      const float lx = sx - (float)xa, hx = 1.f - lx;
      const float top = hx * (float)__ldg(row0 + 3 * xa) + lx * (float)__ldg(row0 + 3 * xb);
      const float bot = hx * (float)__ldg(row1 + 3 * xa) + lx * (float)__ldg(row1 + 3 * xb);
      v[j] = __fadd_rn(__fmul_rn(hy * top + ly * bot, 2.f / 255.f), -1.f);  // x * 2/255 - 1, two roundings
    }
    bf16* dst;
    if (mode == 0) {
      dst = out + ((b * 3 + c) * S + y) * (long long)S + x0;
    } else {
      const int g = S / p;
      const long long tok = (b * g + y / p) * g + x0 / p;
      dst = out + tok * (3ll * p * p) + c * p * p + (y % p) * p + (x0 % p);
    }
    *reinterpret_cast<uint4*>(dst) = pack_bf16x8(v);
  }
}

__global__ void embed_kernel(const int* __restrict__ ids, const bf16* __restrict__ table, int vocab, int H, int B,
                             int T, float scale, bf16* __restrict__ out, long long ldo, int rows_per_seq,
                             int row_offset) {
  pdl_prologue();
  const int hv = H >> 3;
  const long long total = (long long)B * T * hv;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % hv) * 8;
    const long long bt = i / hv;
    const int t = (int)(bt % T);
    const long long b = bt / T;
    int id = __ldg(ids + bt);
    id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
    float v[8];
    unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(table + (long long)id * H + c)), v);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] *= scale;
    *reinterpret_cast<uint4*>(out + (b * rows_per_seq + row_offset + t) * ldo + c) = pack_bf16x8(v);
  }
}

// fp32 -> bf16 copy of a [M, N] matrix (row strides in elements)
__global__ void f32_to_bf16_kernel(const float* __restrict__ x, long long ldx, bf16* __restrict__ y, long long ldy,
                                   long long M, int N) {
  pdl_prologue();
  const long long total = M * N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / N;
    const int n = (int)(i % N);
    y[m * ldy + n] = __float2bfloat16(x[m * ldx + n]);
  }
}

}  // namespace ew
}  // namespace vla
