// Short-sequence attention on the tensor cores (tcgen05): every key of a
// sequence (Lk <= 128) fits one tile, so the softmax needs no running max.
//
// Work item = 128 query rows of one (sequence, kv head): the G = Hq / Hkv query
// heads that share the kv head are stacked (stacked row s -> head kvh*G + s/Lq,
// query s % Lq), so K and V are staged once for all of them and the padding is
// at most one partial tile per (sequence, kv head) instead of one per head.
// Persistent CTAs of 4 warps (4 per SM: 48 KB smem, 128 TMEM columns; four
// independent CTAs per SM hide each other's copy latency better than two CTAs
// that prefetch their next item, measured):
//   1. all threads copy Q (stacked rows), K and V into 128-byte-swizzled smem
//      tiles (cp.async, zero-filled past the valid rows / keys);
//   2. one thread issues S = Q K^T (128 x NK x 64) into TMEM columns [0, NK);
//   3. thread r owns row r: reads S, masks keys past kv_len / above the causal
//      diagonal, takes the row max, writes P = 2^(s*scale - m) as bf16 pairs
//      over the S columns it has read, keeps the fp32 row sum;
//   4. one thread issues O = P V (A from TMEM, V MN-major from smem) into
//      columns [64, 128);
//   5. thread r reads its O row, divides by the row sum and writes it into the
//      (no longer needed) Q tile; each warp then stores its 32 rows with whole
//      128-byte rows per 8 lanes.
// Semantics are those of the mma.sync kernel (attention.cuh): fp32 scores and
// softmax, exp2 with the scale folded in, P rounded to bf16 for P.V, causal
// masking key > query index, kv_len limiting the keys of each sequence.
#pragma once
#include "common.cuh"

namespace vla {
namespace attn_sq {

constexpr int HD = 64;
constexpr int MT = 128;            // stacked query rows per item
constexpr int kThreads = 128;
constexpr int TILE = MT * HD * 2;  // 16 KB
constexpr uint32_t TMEM_COLS = 128;
constexpr uint32_t O_COL = 64;

struct Params {
  const bf16* q;
  const bf16* k;
  const bf16* v;
  bf16* o;
  long long q_row, k_row, v_row, o_row;
  long long q_batch, k_batch, v_batch, o_batch;
  int Lq, Lk, Hq, Hkv, G, n_mt, batch, causal;
  const int* kv_len;
  float scale_log2;
};

struct Stage {
  uint8_t q[TILE];  // stacked query rows; after S = Q K^T the output rows are staged here
  uint8_t k[TILE];
  uint8_t v[TILE];
};

struct Smem {
  Stage st;
  uint64_t bar;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// D[tmem] (+)= A[tmem] * B[smem desc] (A: two bf16 K-elements per 32-bit column)
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// MN-major SW128 descriptor of a [keys x 64] bf16 tile read along the keys
__device__ __forceinline__ uint64_t mn_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((uint32_t)TILE >> 4) << 16;  // leading byte offset (single 64-wide atom along N)
  d |= (uint64_t)(1024u >> 4) << 32;           // 8 key rows x 128 B
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Copy `nrows` rows (row i at src(i), 128 bytes each) into a swizzled tile;
// rows at or past `valid` are zero-filled.  Thread t copies chunk t & 7 of rows
// t >> 3, +16, ... (8 consecutive threads read one 128-byte row).
template <typename RowPtr>
__device__ __forceinline__ void stage_rows(uint32_t tile, int valid, RowPtr src) {
  const int c = threadIdx.x & 7;
#pragma unroll
  for (int i = 0; i < MT / 16; ++i) {
    const int r = (threadIdx.x >> 3) + 16 * i;
    const bool ok = r < valid;
    const bf16* g = ok ? src(r) + c * 8 : src(0);
    cp16(tile + (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)), g, ok);
  }
}

struct Item {
  int b, kvh, s0, lk;
};

__device__ __forceinline__ Item item_at(const Params& p, int it) {
  Item r;
  const int mt = it % p.n_mt;
  const int rest = it / p.n_mt;
  r.kvh = rest % p.Hkv;
  r.b = rest / p.Hkv;
  r.s0 = mt * MT;
  r.lk = p.Lk;
  if (p.kv_len != nullptr) r.lk = max(0, min(r.lk, __ldg(p.kv_len + r.b)));
  return r;
}

// issue (and commit as one group) the copies of item `w` into stage `st`
__device__ __forceinline__ void stage_item(const Params& p, const Item& w, const Stage& st) {
  const bf16* qb = p.q + (long long)w.b * p.q_batch;
  const bf16* kb = p.k + (long long)w.b * p.k_batch + (long long)w.kvh * HD;
  const bf16* vb = p.v + (long long)w.b * p.v_batch + (long long)w.kvh * HD;
  const int G = p.G, Lq = p.Lq, s0 = w.s0, kvh = w.kvh;
  stage_rows(smem_u32(st.q), G * Lq - s0, [&](int r) {
    const int s = s0 + r;
    const int h = kvh * G + s / Lq;
    return qb + (long long)(s % Lq) * p.q_row + (long long)h * HD;
  });
  stage_rows(smem_u32(st.k), w.lk, [&](int r) { return kb + (long long)r * p.k_row; });
  stage_rows(smem_u32(st.v), w.lk, [&](int r) { return vb + (long long)r * p.v_row; });
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int NK>
__global__ void __launch_bounds__(kThreads, 4) attn_short_kernel(Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&sm.bar, 1);
    sm.abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(&sm.tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  pdl_prologue();

  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const int row = warp * 32 + lane;  // this thread's tile row = TMEM lane
  constexpr uint32_t idesc_s = make_idesc_bf16(MT, NK);
  constexpr uint32_t idesc_pv = make_idesc_bf16(MT, HD) | (1u << 16);  // B (V) MN-major
  const int n_items = p.batch * p.Hkv * p.n_mt;
  const int rows_valid = p.G * p.Lq;
  const int G = p.G, Lq = p.Lq;
  uint32_t phase = 0;
  bool ok = true;

  for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
    const Item w = item_at(p, it);
    const Stage& st = sm.st;
    stage_item(p, w, st);
    asm volatile("cp.async.wait_group 0;" ::: "memory");         // this item's copies landed
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t sq = smem_u32(st.q), sk = smem_u32(st.k), sv = smem_u32(st.v);

    // S = Q K^T
    if (threadIdx.x == 0) {
      const uint64_t qd = make_sw128_desc(sq), kd = make_sw128_desc(sk);
#pragma unroll
      for (int k = 0; k < HD / 16; ++k) tc_mma_bf16(tmem, qd + 2 * k, kd + 2 * k, idesc_s, k > 0 ? 1u : 0u);
      tc_commit(&sm.bar);
    }
    ok = mbar_wait_bounded(&sm.bar, phase, &sm.abort);
    if (!ok) *(volatile int*)&sm.abort = 1;  // the other warps stop waiting at once
    phase ^= 1u;
    tc_fence_after();

    // softmax of this thread's row
    const int s = w.s0 + row;
    const int qi = s % Lq;
    int kend = w.lk;  // keys [0, kend) are visible to this row
    if (p.causal) kend = min(kend, qi + 1);
    const uint32_t srow = tmem + lane_base;
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
        const float e0 = 64 * h + c < kend ? ex2f(fmaf(v[c], p.scale_log2, -mb)) : 0.f;
        const float e1 = 64 * h + c + 1 < kend ? ex2f(fmaf(v[c + 1], p.scale_log2, -mb)) : 0.f;
        l += e0 + e1;
        pk[c >> 1] = pack_bf16x2(e0, e1);
      }
      // P (keys 64h .. 64h+63) over S columns 32h .. 32h+31, already read
      tmem_st32u(srow + 32 * h, pk);
    }
    tc_fence_before();
    ok = __syncthreads_and(ok) != 0;  // one verdict for the whole block
    tc_fence_after();

    // O = P V
    if (threadIdx.x == 0 && ok) {
#pragma unroll
      for (int k = 0; k < NK / 16; ++k)
        mma_ts(tmem + O_COL, tmem + (uint32_t)k * 8u, mn_desc(sv + (uint32_t)k * 2048u), idesc_pv, k > 0 ? 1u : 0u);
      tc_commit(&sm.bar);
    }
    ok = ok && mbar_wait_bounded(&sm.bar, phase, &sm.abort);
    if (!ok) *(volatile int*)&sm.abort = 1;
    phase ^= 1u;
    tc_fence_after();

    // O row / l into the Q tile (row r at r * 128 bytes, 16-byte chunks swizzled
    // by r & 7), then this warp's 32 rows out as whole 128-byte rows
    {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      float o[64];
      tmem_ld64(srow + O_COL, o);
#pragma unroll
      for (int c8 = 0; c8 < HD / 8; ++c8) {
        float t8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) t8[i] = o[8 * c8 + i] * inv;
        const uint4 u = pack_bf16x8(t8);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sq + (uint32_t)(row * 128 + ((c8 ^ (row & 7)) << 4))),
                     "r"(u.x), "r"(u.y), "r"(u.z), "r"(u.w)
                     : "memory");
      }
      __syncwarp();
      const int c = lane & 7;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = warp * 32 + 4 * i + (lane >> 3);
        const int sr = w.s0 + r;
        if (ok && sr < rows_valid) {
          uint4 u;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                       : "r"(sq + (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4))));
          const int h = w.kvh * G + sr / Lq;
          bf16* dst = p.o + (long long)w.b * p.o_batch + (long long)(sr % Lq) * p.o_row + (long long)h * HD + c * 8;
          *reinterpret_cast<uint4*>(dst) = u;
        }
      }
    }
    // the next item's copies overwrite the tiles and its MMA the TMEM columns;
    // the barrier also makes `ok` block-uniform, so every warp leaves the loop
    // on the same iteration
    tc_fence_before();
    ok = __syncthreads_and(ok) != 0;
    tc_fence_after();
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  if (!ok && threadIdx.x == 0) vla_record_error(VLA_DERR_ATTN_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace attn_sq
}  // namespace vla
