// Flash-style attention, head_dim 64, bf16 in / fp32 softmax / bf16 out.
//
// One CTA = 64 query rows of one (sequence, head); 4 warps x 16 rows.  K/V
// tiles of 64 keys stream through a double-buffered cp.async ring; S = Q K^T
// and O += P V run on mma.sync m16n8k16 with fp32 accumulators; the online
// softmax keeps row max / row sum in fp32 registers and P is rounded to bf16
// for the P.V product (as the reference rounds the probabilities to bf16
// before P.V, vla/text_encoder_bf16.py:124-126).
//
// Replaces, per layer, the reference's per-head score GEMMs
// (vla/text_encoder_bf16.py:505-511), the masked softmax kernels
// (cc/bf16/masked_softmax_128_bf16.cc:251-398, cc/float/v1_softmax_float.cc:117-179,
// cc/bf16_old/v2_softmax_bf16.cc:627-645) and the per-head P.V GEMMs
// (vla/text_encoder_bf16.py:519-526).  GQA: head h reads kv head
// h * Hkv / Hq (vla/text_encoder_bf16.py:117).
#pragma once
#include "common.cuh"

namespace vla {
namespace attn {

constexpr int BQ = 64;   // query rows per CTA
constexpr int BKV = 64;  // keys per tile
constexpr int HD = 64;   // head dim
constexpr int kThreads = 128;

struct Params {
  const bf16* q;
  const bf16* k;
  const bf16* v;
  bf16* o;
  long long q_row, k_row, v_row, o_row;          // row strides (elements)
  long long q_batch, k_batch, v_batch, o_batch;  // sequence strides (elements)
  int Lq, Lk, Hq, Hkv;
  int causal;
  const int* kv_len;  // per-sequence valid key count, or null
  float scale_log2;   // softmax scale * log2(e)
};

__device__ __forceinline__ int swz(int r, int c) {  // element offset of (row, 8-col chunk)
  return r * HD + ((c ^ (r & 7)) << 3);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Load a [64 x 64] bf16 tile (rows r0.. of a strided matrix) into swizzled smem,
// zero-filling rows >= nrows.
__device__ __forceinline__ void load_tile(bf16* s, const bf16* g, long long row_stride, int r0, int nrows) {
  const uint32_t sbase = smem_u32(s);
#pragma unroll
  for (int i = 0; i < (BKV * 8) / kThreads; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    const int r = idx >> 3, c = idx & 7;
    const bool ok = (r0 + r) < nrows;
    const bf16* src = ok ? g + (long long)(r0 + r) * row_stride + c * 8 : g;
    cp_async16(sbase + 2u * (uint32_t)swz(r, c), src, ok);
  }
}

__global__ void __launch_bounds__(kThreads, 4) flash_attn_kernel(Params p) {
  pdl_prologue();
  __shared__ __align__(128) bf16 sQ[BQ * HD];
  __shared__ __align__(128) bf16 sK[2][BKV * HD];
  __shared__ __align__(128) bf16 sV[2][BKV * HD];

  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = (int)((long long)h * p.Hkv / p.Hq);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int m0 = qt * BQ;
  int Lk = p.Lk;
  if (p.kv_len != nullptr) Lk = min(Lk, __ldg(p.kv_len + b));

  const bf16* qg = p.q + (long long)b * p.q_batch + (long long)h * HD;
  const bf16* kg = p.k + (long long)b * p.k_batch + (long long)kvh * HD;
  const bf16* vg = p.v + (long long)b * p.v_batch + (long long)kvh * HD;

  int n_tiles = (Lk + BKV - 1) / BKV;
  if (p.causal) n_tiles = min(n_tiles, (m0 + BQ - 1) / BKV + 1);

  load_tile(sQ, qg, p.q_row, m0, p.Lq);
  if (n_tiles > 0) {
    load_tile(sK[0], kg, p.k_row, 0, Lk);
    load_tile(sV[0], vg, p.v_row, 0, Lk);
  }
  cp_async_commit();

  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY};
  float lrow[2] = {0.f, 0.f};
  uint32_t qa[4][4];
  const int qrow0 = m0 + warp * 16 + g;  // this thread's rows: qrow0, qrow0 + 8

  for (int j = 0; j < n_tiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_tiles) {
      load_tile(sK[buf ^ 1], kg, p.k_row, (j + 1) * BKV, Lk);
      load_tile(sV[buf ^ 1], vg, p.v_row, (j + 1) * BKV, Lk);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    if (j == 0) {
      const uint32_t qb = smem_u32(sQ);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int r = warp * 16 + (lane & 15);
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(qb + 2u * (uint32_t)swz(r, c), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
      }
    }

    // S = Q K^T for 64 keys
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    const uint32_t kb = smem_u32(sK[buf]);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int mi = lane >> 3;
        const int r = np * 16 + (lane & 7) + (mi >> 1) * 8;
        const int c = ks * 2 + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + 2u * (uint32_t)swz(r, c), b0, b1, b2, b3);
        mma_bf16(s[2 * np], qa[ks], b0, b1);
        mma_bf16(s[2 * np + 1], qa[ks], b2, b3);
      }
    }

    // mask + online softmax (base-2 exponent, scale folded in)
    const int n0 = j * BKV;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = n0 + nt * 8 + 2 * t + (e & 1);
        const int qrow = qrow0 + (e >> 1) * 8;
        bool masked = key >= Lk;
        if (p.causal) masked = masked || key > qrow;
        const float v = masked ? -INFINITY : s[nt][e] * p.scale_log2;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mnew = fmaxf(mrow[r], mx[r]);
      const float mbase = mnew == -INFINITY ? 0.f : mnew;
      alpha[r] = exp2f(mrow[r] - mbase);
      mrow[r] = mnew;
      mx[r] = mbase;
    }
    float ls[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pe = exp2f(s[nt][e] - mx[e >> 1]);
        s[nt][e] = pe;
        ls[e >> 1] += pe;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) lrow[r] = lrow[r] * alpha[r] + ls[r];
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      o[dt][0] *= alpha[0];
      o[dt][1] *= alpha[0];
      o[dt][2] *= alpha[1];
      o[dt][3] *= alpha[1];
    }

    // O += P V
    const uint32_t vb = smem_u32(sV[buf]);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * ks][0], s[2 * ks][1]);
      pa[1] = pack_bf16x2(s[2 * ks][2], s[2 * ks][3]);
      pa[2] = pack_bf16x2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
      pa[3] = pack_bf16x2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        const int mi = lane >> 3;
        const int r = ks * 16 + (lane & 7) + (mi & 1) * 8;
        const int c = dp * 2 + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + 2u * (uint32_t)swz(r, c), b0, b1, b2, b3);
        mma_bf16(o[2 * dp], pa, b0, b1);
        mma_bf16(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  const float inv0 = lrow[0] > 0.f ? 1.f / lrow[0] : 0.f;
  const float inv1 = lrow[1] > 0.f ? 1.f / lrow[1] : 0.f;
  bf16* og = p.o + (long long)b * p.o_batch + (long long)h * HD;
  if (qrow0 < p.Lq) {
    bf16* orow = og + (long long)qrow0 * p.o_row;
#pragma unroll
    for (int dt = 0; dt < 8; ++dt)
      *reinterpret_cast<uint32_t*>(orow + dt * 8 + 2 * t) = pack_bf16x2(o[dt][0] * inv0, o[dt][1] * inv0);
  }
  if (qrow0 + 8 < p.Lq) {
    bf16* orow = og + (long long)(qrow0 + 8) * p.o_row;
#pragma unroll
    for (int dt = 0; dt < 8; ++dt)
      *reinterpret_cast<uint32_t*>(orow + dt * 8 + 2 * t) = pack_bf16x2(o[dt][2] * inv1, o[dt][3] * inv1);
  }
}

}  // namespace attn
}  // namespace vla
