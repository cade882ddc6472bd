// Flash attention on the 5th-generation tensor cores (tcgen05), head_dim 64.
//
// Work item = 128 query rows of one (sequence, head); a persistent CTA per SM
// walks the work items.  Warp roles:
//   warp 0     TMA producer: Q (double-buffered across items), K and V tiles of
//              128 keys into separate 3-stage rings (K is released as soon as
//              S = Q K^T completes, V after P.V)
//   warp 1     TMEM allocator + single-thread MMA issuer:
//                S_j  = Q . K_j^T         (UMMA 128x128x16, A = Q, B = K, both K-major)
//                O   += P_j . [V_j | 1]   (UMMA 128x80x16, A = P from tensor memory,
//                                          B = V from smem MN-major, no transpose pass)
//   warps 2..5 softmax: thread r owns query row r; reads its S row from TMEM
//              (so the row max needs no shuffles), P = exp2(S*scale*log2e - m)
//              rounded to bf16 and stored back into the S columns of TMEM (no
//              shared-memory round trip) for the P.V MMA.
// The output accumulator O lives in TMEM (double-buffered across items) and is
// accumulated by the tensor core over the item's key tiles.  The B operand of
// P.V is V extended by a 16-column block of ones (a constant smem block reached
// through the descriptor's leading byte offset), so O column 64 accumulates the
// row sum of P: the softmax threads neither add up P nor touch O per tile.  The
// running max m only moves when a row's max grows by more than 2^8 (log2 units),
// and only then is that row of O rescaled in TMEM (P values stay below 2^8,
// exact in fp32 and bf16 alike).
// S is double-buffered in TMEM (S_{j+1} is computed while row j is in softmax).
// TMEM: 2 x 128 (S) + 2 x 80 (O | row sum) columns.
//
// Used for the non-causal SigLIP attention (1024 keys per head); the small
// text / expert attentions run on the mma.sync kernel (attention.cuh).
#pragma once
#include "common.cuh"

namespace vla {
namespace attn_tc {

constexpr int BQ = 128;   // query rows per work item (UMMA M)
constexpr int BKV = 128;  // keys per tile (UMMA N of S, K of P.V)
constexpr int HD = 64;
constexpr int kKStages = 3;
constexpr int kVStages = 3;
constexpr int kThreads = 192;
constexpr int TILE_BYTES = BKV * HD * 2;  // 16 KB: a [128 x 64] bf16 tile (Q, K or V)
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t S_COL0 = 0;    // S buffers at columns 0 and 128
constexpr uint32_t O_COL0 = 256;  // O buffers at columns 256 and 336
constexpr int ON = HD + 16;       // O columns: 64 outputs + 16 copies of the row sum
constexpr float kRescaleLog2 = 8.f;

struct Params {
  int Lq, Lk, Hq, Hkv, batch;
  int n_qt;                                  // query tiles per (sequence, head)
  long long q_rows_per_seq, k_rows_per_seq;  // row offset of sequence b = b * rows_per_seq
  bf16* o;
  long long o_row, o_batch;
  const int* kv_len;
  float scale_log2;
};

struct Smem {
  uint8_t q[2][TILE_BYTES];
  uint8_t k[kKStages][TILE_BYTES];
  uint8_t v[kVStages][TILE_BYTES];
  uint8_t ones[TILE_BYTES];  // bf16 1.0: the extra N atom of every P.V B operand
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t v_full[kVStages], v_empty[kVStages];
  uint64_t s_full[2], p_full[2], o_empty[2];
  uint64_t pv_done;  // completes once per P.V, in the CTA's tile order
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 32 lanes x 16 consecutive 32-bit TMEM columns from registers, then wait.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 32 lanes x 64 consecutive 32-bit TMEM columns from registers, then wait.
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, "
      "%33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, "
      "%49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "r"(r[32]), "r"(r[33]), "r"(r[34]), "r"(r[35]), "r"(r[36]),
      "r"(r[37]), "r"(r[38]), "r"(r[39]), "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]), "r"(r[45]),
      "r"(r[46]), "r"(r[47]), "r"(r[48]), "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]), "r"(r[54]),
      "r"(r[55]), "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]), "r"(r[62]), "r"(r[63])
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]: A (M x K) read from tensor memory with
// two bf16 K-elements per 32-bit column (element 2c in the low half).
__device__ __forceinline__ void tc_mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// MN-major SW128 descriptor for a [rows x 64] bf16 tile read along the row
// (K) direction: 8-row groups 1024 bytes apart (stride byte offset); the next
// 64-element atom along N starts `next_atom` bytes after this one (leading
// byte offset), which is where the ones block sits for the N = 80 P.V MMA.
__device__ __forceinline__ uint64_t make_sw128_mn_desc(uint32_t smem_addr, uint32_t next_atom) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((next_atom >> 4) & 0x3FFFu) << 16;  // leading byte offset: next N atom
  d |= (uint64_t)(1024u >> 4) << 32;   // stride byte offset: next 8 K-rows
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// work item w -> (query tile, head, sequence); consecutive items share K/V
__device__ __forceinline__ void item_coords(const Params& p, int w, int& qt, int& h, int& b) {
  qt = w % p.n_qt;
  h = (w / p.n_qt) % p.Hq;
  b = w / (p.n_qt * p.Hq);
}

__device__ __forceinline__ int item_keys(const Params& p, int b) {
  int Lk = p.Lk;
  if (p.kv_len != nullptr) Lk = min(Lk, __ldg(p.kv_len + b));
  return max(Lk, 0);
}

// Persistent kernel: CTA i processes work items i, i + gridDim.x, ...  Every
// pipeline counter (K/V ring slots, S/P/PV buffers) runs over the CTA's global
// tile index, so loads and MMAs of the next item overlap the tail of this one.
__global__ void __launch_bounds__(kThreads, 1)
    flash_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* abort_flag = &sm.abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.n_qt * p.Hq * p.batch;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.q_full[i], 1);
      mbar_init(&sm.q_empty[i], 1);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.p_full[i], 128);
      mbar_init(&sm.o_empty[i], 128);
    }
    mbar_init(&sm.pv_done, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    sm.abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, TMEM_COLS);
  {
    // the ones block, written through the generic proxy and read by the tensor core
    uint4* o4 = reinterpret_cast<uint4*>(sm.ones);
    const uint4 one8 = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
    for (int i = threadIdx.x; i < TILE_BYTES / 16; i += kThreads) o4[i] = one8;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  pdl_prologue();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      bool ok = true;
      int tk = 0, tv = 0, it = 0;  // K / V tiles issued, items started
      for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++it) {
        int qt, h, b;
        item_coords(p, w, qt, h, b);
        const int kvh = (int)((long long)h * p.Hkv / p.Hq);
        const int n = (item_keys(p, b) + BKV - 1) / BKV;
        const int qb = it & 1;
        if (!mbar_wait_bounded(&sm.q_empty[qb], ((it >> 1) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.q_full[qb], TILE_BYTES);
        tma_load_2d(sm.q[qb], &tmQ, &sm.q_full[qb], h * HD, (int)(b * p.q_rows_per_seq) + qt * BQ);
        const int k_row0 = (int)(b * p.k_rows_per_seq);
        for (int j = 0; j < n; ++j) {
          const int sk = tk % kKStages;
          if (!mbar_wait_bounded(&sm.k_empty[sk], ((tk / kKStages) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.k_full[sk], TILE_BYTES);
          tma_load_2d(sm.k[sk], &tmK, &sm.k_full[sk], kvh * HD, k_row0 + j * BKV);
          ++tk;
          const int sv = tv % kVStages;
          if (!mbar_wait_bounded(&sm.v_empty[sv], ((tv / kVStages) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.v_full[sv], TILE_BYTES);
          tma_load_2d(sm.v[sv], &tmV, &sm.v_full[sv], kvh * HD, k_row0 + j * BKV);
          ++tv;
        }
      }
      if (!ok) {
        if (!*abort_flag) vla_record_error(VLA_DERR_ATTN_TIMEOUT);
        *abort_flag = 1;
      }
      // let issued copies land before the CTA can exit
      for (int i = (tk > kKStages ? tk - kKStages : 0); i < tk; ++i)
        mbar_wait_bounded(&sm.k_full[i % kKStages], (i / kKStages) & 1, nullptr, 20000000ull);
      for (int i = (tv > kVStages ? tv - kVStages : 0); i < tv; ++i)
        mbar_wait_bounded(&sm.v_full[i % kVStages], (i / kVStages) & 1, nullptr, 20000000ull);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BQ, BKV);
      constexpr uint32_t idesc_pv = make_idesc_bf16(BQ, ON) | (1u << 16);  // B (V | 1) is MN-major
      const uint32_t ones = smem_u32(sm.ones);
      bool ok = true;
      int t = 0, it = 0, io = 0;  // tiles, items, items with at least one key tile
      for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++it) {
        int qt, h, b;
        item_coords(p, w, qt, h, b);
        const int n = (item_keys(p, b) + BKV - 1) / BKV;
        const int qb = it & 1;
        ok = mbar_wait_bounded(&sm.q_full[qb], (it >> 1) & 1, abort_flag);
        if (!ok) break;
        const int ob = io & 1;
        const uint64_t qdesc = make_sw128_desc(smem_u32(sm.q[qb]));
        // S of tile j, then P.V of tile j-1; finally P.V of the item's last tile
        for (int j = 0; ok && j <= n && n > 0; ++j) {
          if (j < n) {
            const int tt = t + j;
            const int sk = tt % kKStages;
            ok = mbar_wait_bounded(&sm.k_full[sk], (tt / kKStages) & 1, abort_flag);
            // S buffer tt%2 was last read by the softmax of tile tt-2 (released with P_{tt-2})
            if (ok && tt >= 2) ok = mbar_wait_bounded(&sm.p_full[tt & 1], ((tt - 2) >> 1) & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            const uint64_t kdesc = make_sw128_desc(smem_u32(sm.k[sk]));
            const uint32_t d = tmem + S_COL0 + (uint32_t)(tt & 1) * BKV;
#pragma unroll
            for (int k = 0; k < HD / 16; ++k) tc_mma_bf16(d, qdesc + 2 * k, kdesc + 2 * k, idesc_s, k > 0);
            tc_commit(&sm.s_full[tt & 1]);
            tc_commit(&sm.k_empty[sk]);
          }
          if (j >= 1) {
            const int tp = t + j - 1;
            const int sv = tp % kVStages;
            // O buffer ob was last read out by the softmax for item io-2
            if (j == 1 && io >= 2) ok = mbar_wait_bounded(&sm.o_empty[ob], ((io - 2) >> 1) & 1, abort_flag);
            if (ok) ok = mbar_wait_bounded(&sm.p_full[tp & 1], (tp >> 1) & 1, abort_flag);
            if (ok) ok = mbar_wait_bounded(&sm.v_full[sv], (tp / kVStages) & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            // P (bf16, packed in pairs) lives in the first 64 columns of S buffer tp%2
            const uint32_t pt = tmem + S_COL0 + (uint32_t)(tp & 1) * BKV;
            const uint32_t vbase = smem_u32(sm.v[sv]);
            const uint32_t d = tmem + O_COL0 + (uint32_t)ob * ON;
#pragma unroll
            for (int k = 0; k < BKV / 16; ++k) {
              const uint32_t a = vbase + (uint32_t)k * 2048u;
              const uint64_t bdesc = make_sw128_mn_desc(a, ones - vbase);
              tc_mma_bf16_ts(d, pt + (uint32_t)k * 8u, bdesc, idesc_pv, (j > 1 || k > 0) ? 1u : 0u);
            }
            tc_commit(&sm.pv_done);
            tc_commit(&sm.v_empty[sv]);
          }
        }
        if (!ok) break;
        tc_commit(&sm.q_empty[qb]);  // every S of this item has been issued before this point
        t += n;
        if (n > 0) ++io;
      }
      if (!ok) {
        if (!*abort_flag) vla_record_error(VLA_DERR_ATTN_TIMEOUT);
        *abort_flag = 1;
      }
    }
  } else {
    // ---------------- softmax / output warps ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    bool ok = true;
    int t = 0, io = 0;
    // the previous item's output is read out of TMEM while this item's first
    // tile is in softmax (its P.V is then certainly done)
    bool pending = false;
    int pend_b = 0, pend_h = 0, pend_qt = 0, pend_ob = 0, pend_tp = 0;
    auto finish_item = [&]() -> bool {
      // completion of the item's last P.V; no later P.V can have completed, as it
      // needs a P this thread has not yet released
      bool good = mbar_wait_bounded(&sm.pv_done, (uint32_t)pend_tp & 1u, abort_flag);
      good = __all_sync(0xffffffffu, good);
      if (!good) return false;
      tc_fence_after();
      const uint32_t oadr = tmem + lane_base + O_COL0 + (uint32_t)pend_ob * ON;
      float o[HD], lsum[16];
      tmem_ld64(oadr, o);
      tmem_ld16(oadr + HD, lsum);
      tc_fence_before();
      mbar_arrive(&sm.o_empty[pend_ob]);
      const int qrow = pend_qt * BQ + row;
      if (qrow < p.Lq) {
        const float inv = lsum[0] > 0.f ? 1.f / lsum[0] : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(p.o + (long long)pend_b * p.o_batch + (long long)qrow * p.o_row +
                                              (long long)pend_h * HD);
#pragma unroll
        for (int c8 = 0; c8 < HD / 8; ++c8) {
          float tv8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) tv8[i] = o[c8 * 8 + i] * inv;
          dst[c8] = pack_bf16x8(tv8);
        }
      }
      return true;
    };
    for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
      int qt, h, b;
      item_coords(p, w, qt, h, b);
      const int Lk = item_keys(p, b);
      const int n = (Lk + BKV - 1) / BKV;
      if (n == 0) {
        const int qrow = qt * BQ + row;
        if (qrow < p.Lq) {
          uint4* dst = reinterpret_cast<uint4*>(p.o + (long long)b * p.o_batch + (long long)qrow * p.o_row +
                                                (long long)h * HD);
#pragma unroll
          for (int c8 = 0; c8 < HD / 8; ++c8) dst[c8] = make_uint4(0u, 0u, 0u, 0u);
        }
        continue;
      }
      const int ob = io & 1;
      float m = -INFINITY;  // running max of S * scale * log2(e), moved in steps > kRescaleLog2
      for (int j = 0; j < n; ++j) {
        const int tt = t + j;
        ok = mbar_wait_bounded(&sm.s_full[tt & 1], (tt >> 1) & 1, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const uint32_t sadr = tmem + lane_base + S_COL0 + (uint32_t)(tt & 1) * BKV;
        const int key0 = j * BKV;
        float s[BKV];
        tmem_ld128(sadr, s);
        if (key0 + BKV > Lk) {
#pragma unroll
          for (int c = 0; c < BKV; ++c)
            if (key0 + c >= Lk) s[c] = -INFINITY;
        }
        // row max with 8 independent three-input max chains
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = s[i];
#pragma unroll
        for (int c = 8; c < BKV; c += 16) {
#pragma unroll
          for (int i = 0; i < 8; ++i) mx8[i] = max3f(mx8[i], s[c + i], s[c + 8 + i]);
        }
        const float mx = max3f(max3f(mx8[0], mx8[1], mx8[2]), max3f(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])) *
                         p.scale_log2;
        const bool grow = mx > m + kRescaleLog2;
        const float alpha = grow ? ex2_fast(m - mx) : 1.f;
        if (grow) m = mx;
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
          // rescale this warp's rows of O (and the row sums) once P.V of tile tt-1 is done
          ok = mbar_wait_bounded(&sm.pv_done, (uint32_t)(tt - 1) & 1u, abort_flag);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          tc_fence_after();
          const uint32_t oadr = tmem + lane_base + O_COL0 + (uint32_t)ob * ON;
          float o[HD];
          uint32_t u[HD];
          tmem_ld64(oadr, o);
#pragma unroll
          for (int i = 0; i < HD; ++i) u[i] = __float_as_uint(o[i] * alpha);
          tmem_st64(oadr, u);
          tmem_ld16(oadr + HD, o);
#pragma unroll
          for (int i = 0; i < 16; ++i) u[i] = __float_as_uint(o[i] * alpha);
          tmem_st16(oadr + HD, u);
        }
        const float mbase = m == -INFINITY ? 0.f : m;
        // P row (128 keys): exp2(s * scale*log2e - m) as one FFMA + MUFU.EX2, packed
        // as 64 bf16 pairs into the first 64 TMEM columns of this S buffer
        uint32_t pk[BKV / 2];
#pragma unroll
        for (int c = 0; c < BKV; c += 2) {
          const float e0 = ex2_fast(fmaf(s[c], p.scale_log2, -mbase));
          const float e1 = ex2_fast(fmaf(s[c + 1], p.scale_log2, -mbase));
          pk[c >> 1] = pack_bf16x2(e0, e1);
        }
        tmem_st64(sadr, pk);
        if (j == 0 && pending) {
          ok = finish_item();
          if (!ok) break;
          pending = false;
        }
        tc_fence_before();
        mbar_arrive(&sm.p_full[tt & 1]);
      }
      if (!ok) break;
      pending = true;
      pend_b = b, pend_h = h, pend_qt = qt, pend_ob = ob, pend_tp = t + n - 1;
      t += n;
      ++io;
    }
    if (ok && pending) ok = finish_item();
    if (!ok && lane == 0) {
      if (!*abort_flag) vla_record_error(VLA_DERR_ATTN_TIMEOUT);
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace attn_tc
}  // namespace vla
