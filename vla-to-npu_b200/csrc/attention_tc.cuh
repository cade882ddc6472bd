// Flash attention on the 5th-generation tensor cores (tcgen05), head_dim 64.
//
// Work item = 256 query rows (two 128-row tiles Q0, Q1) of one (sequence,
// head); a persistent CTA per SM walks the work items.  Warp roles:
//   warp 0      TMA producer: Q0/Q1 (double-buffered across items), K and V
//               tiles of 128 keys into separate 3-stage rings (K is released
//               once both S_g = Q_g K^T are done, V after both P.V)
//   warps 1, 2  S issuers, one per softmax group g, following the group's
//               tile order with blocking waits, an elected lane issuing per
//               key tile j:
//                 S_g(j)     = Q_g . K_j^T    (UMMA 128x128x16, both K-major)
//   warp 3      P.V issuer for both groups (SPLITPV, the default), per key
//               tile group 0 then group 1 (the order in which their
//               alternating exp phases finish P):
//                 O_g       += P_g . V_j      (UMMA 128x64x16, A = P from tensor
//                                              memory, B = V MN-major, no transpose)
//               With SPLITPV off, each S issuer also issues its group's P.V
//               of tile j-1 after S_g(j) (measured 1.8 % slower: the P.V
//               waited behind the S issue on the softmax warps' path).
//               K, V and Q slots are released by both groups' commits.
//   warps 4..7  softmax group 0 (rows of Q0), warps 8..11 softmax group 1 (Q1):
//               thread r of a group owns query row r; reads its S row from TMEM
//               (the row max needs no shuffles), writes P = exp2(S*scale*log2e - m)
//               as bf16 pairs into the group's P columns.
// S_g, P_g and O_g have their own tensor-memory columns, so the tensor core
// computes S_g(j+1) while group g is still turning S_g(j) into P (a group
// releases S_g as soon as it has read it), and P.V runs behind the softmax.
// Each SM sub-partition runs two softmax warps (one per group), so the TMEM
// loads, exp chains and barrier waits of one overlap the other's work.  The
// two warps on a sub-partition pass a token so that their exp phases alternate
// (MUFU.EX2 is the sub-partition's scarcest pipe: left alone the two groups
// fall into step and both wait on it, then both leave it idle).
// Registers: the block is launched at kLaunchRegs per thread; warpgroup 0
// (producer, S issuers, P.V issuer) gives most of its share to the two softmax warpgroups
// with setmaxnreg (kLowRegs x 128 + kHighRegs x 256 = kLaunchRegs x 384), so a
// softmax thread holds its whole 128-key S row in registers.
// O_g is accumulated by the tensor core over the item's key tiles; the running
// max m only moves when a row's max grows by more than 2^8 (log2 units), and
// only then is that row of O_g (and its row sum, kept in a register) rescaled
// (P values stay below 2^8).  An item's O_g is read out before the next item's
// first P_g is released, which the next item's first P.V (overwriting O_g)
// waits for.
// TMEM: S_0 | S_1 (2 x 128 columns), P_0 | P_1 (2 x 64), O_0 | O_1 (2 x 64).
//
// Used for the non-causal SigLIP attention (1024 keys per head); the small
// text / expert attentions run on the mma.sync kernel (attention.cuh).
#pragma once
#include "common.cuh"

namespace vla {
namespace attn_tc {

constexpr int BQ = 128;   // query rows per tile (UMMA M)
constexpr int ITEM_ROWS = 2 * BQ;  // query rows per work item (two tiles)
constexpr int BKV = 128;  // keys per tile (UMMA N of S, K of P.V)
constexpr int HD = 64;
constexpr int kKStages = 3;
constexpr int kVStages = 3;
constexpr int kThreads = 384;
constexpr int kLaunchRegs = 168;  // 65536 / 384, rounded down to a multiple of 8
constexpr int kLowRegs = 88;      // warpgroup 0 after setmaxnreg.dec
constexpr int kHighRegs = 208;    // softmax warpgroups after setmaxnreg.inc
static_assert(kLowRegs * 128 + kHighRegs * 256 == kLaunchRegs * 384, "register split must equal the launch total");
static_assert((kLowRegs + 2 * kHighRegs) * 32 <= 16384, "per sub-partition register file");
constexpr int TILE_BYTES = BKV * HD * 2;  // 16 KB: a [128 x 64] bf16 tile (Q, K or V)
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t S_COL0 = 0;    // S_0, S_1 at columns 0 and 128
constexpr uint32_t P_COL0 = 256;  // P_0, P_1 (bf16 pairs) at columns 256 and 320
constexpr uint32_t O_COL0 = 384;  // O_0, O_1 at columns 384 and 448
constexpr float kRescaleLog2 = 8.f;

struct Params {
  int Lq, Lk, Hq, Hkv, batch;
  int n_qt;                                  // work items (256 query rows) per (sequence, head)
  long long q_rows_per_seq, k_rows_per_seq;  // row offset of sequence b = b * rows_per_seq
  bf16* o;
  long long o_row, o_batch;
  const int* kv_len;
  float scale_log2;
};

struct Smem {
  uint8_t q[2][2][TILE_BYTES];  // [item buffer][tile]
  uint8_t k[kKStages][TILE_BYTES];
  uint8_t v[kVStages][TILE_BYTES];
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t v_full[kVStages], v_empty[kVStages];
  uint64_t s_full[2], s_free[2], p_full[2];  // per softmax group, once per key tile
  uint64_t pv_done[2];                       // per group: completes once per P.V, in tile order
  uint64_t mufu_tok[2][4];  // [group][sub-partition]: the exp phase token of each softmax warp
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (one instruction for two lanes' worth of FMA-pipe work):
// (x0, x1) = (a0, a1) * b + c, and (s0, s1) += (e0, e1).
__device__ __forceinline__ void fma2(float a0, float a1, float b, float c, float& x0, float& x1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %4};\n\tmov.b64 rc, {%5, %5};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(x0), "=f"(x1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
__device__ __forceinline__ void add2(float& s0, float& s1, float e0, float e1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(s0), "+f"(s1)
      : "f"(e0), "f"(e1));
}

// 2^x of a pair on the FMA pipe (packed fp32 pairs), for part of the keys:
// MUFU.EX2 serves 16 lanes per clock per SM, the FMA pipe 128, and the exp
// phase leaves issue slots free.  Method (Cody-Waite split plus polynomial):
// x is clamped to >= -126 (the cubic is just below 1 at f = 0, so its
// exponent field is 126 there and n = -126 keeps the sum >= 0); r = x + 1.5 * 2^23 rounded toward -inf holds
// n = floor(x) in its low mantissa bits, f = x - n lies in [0, 1), 2^f comes
// from the cubic minimax fit (in relative error) of 2^f on [0, 1]
// (0.99992514 + 0.695834 f + 0.22606707 f^2 + 0.07802403 f^3, max relative
// error 7.5e-5, well under the 2^-9 rounding of the bf16 P it feeds), and
// 2^n is added into the exponent field: bits(r) << 23 equals n << 23 modulo
// 2^32 because the low nine bits of bits(1.5 * 2^23) are zero.
__device__ __forceinline__ void ex2_poly2(float x0, float x1, float& e0, float& e1) {
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  uint32_t r0, r1, p0, p1;
  asm("{\n\t.reg .b64 x, c, r, t, f, p, k;\n\t"
      "mov.b64 x, {%4, %5};\n\t"
      "mov.b64 c, {%6, %6};\n\t"
      "add.rm.f32x2 r, x, c;\n\t"
      "sub.rn.f32x2 t, r, c;\n\t"
      "sub.rn.f32x2 f, x, t;\n\t"
      "mov.b64 p, {%7, %7};\n\t"
      "mov.b64 k, {%8, %8};\n\t"
      "fma.rn.f32x2 p, p, f, k;\n\t"
      "mov.b64 k, {%9, %9};\n\t"
      "fma.rn.f32x2 p, p, f, k;\n\t"
      "mov.b64 k, {%10, %10};\n\t"
      "fma.rn.f32x2 p, p, f, k;\n\t"
      "mov.b64 {%0, %1}, r;\n\t"
      "mov.b64 {%2, %3}, p;\n\t}"
      : "=r"(r0), "=r"(r1), "=r"(p0), "=r"(p1)
      : "f"(x0), "f"(x1), "f"(12582912.f), "f"(0.07802403f), "f"(0.22606707f), "f"(0.695834f), "f"(0.99992514f));
  e0 = __uint_as_float(r0 * 8388608u + p0);
  e1 = __uint_as_float(r1 * 8388608u + p1);
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

// 32 lanes x 32 consecutive 32-bit TMEM columns from registers, then wait.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
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
// byte offset; unused for the N = 64 P.V MMA).
__device__ __forceinline__ uint64_t make_sw128_mn_desc(uint32_t smem_addr, uint32_t next_atom) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((next_atom >> 4) & 0x3FFFu) << 16;  // leading byte offset: next N atom
  d |= (uint64_t)(1024u >> 4) << 32;   // stride byte offset: next 8 K-rows
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Read one finished row of O_g out of tensor memory and store it divided by
// the row sum l.  The caller has waited for the item's last P.V.
__device__ __forceinline__ void finish_row(const Params& p, uint32_t o_adr, float l, int b, int h, int qrow) {
  const float inv = l > 0.f ? 1.f / l : 0.f;
  uint4* dst = reinterpret_cast<uint4*>(p.o + (long long)b * p.o_batch + (long long)qrow * p.o_row + (long long)h * HD);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    float o[HD / 2];
    tmem_ld32(o_adr + (uint32_t)half * (HD / 2), o);  // warp-collective: every lane loads
    if (qrow < p.Lq) {
#pragma unroll
      for (int c8 = 0; c8 < HD / 16; ++c8) {
        float tv8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) tv8[i] = o[c8 * 8 + i] * inv;
        dst[half * (HD / 16) + c8] = pack_bf16x8(tv8);
      }
    }
  }
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
// P8 of every 8 key pairs take their exponentials from ex2_poly2 (FMA pipe),
// the rest from MUFU.EX2; SPLITPV: warp 3 issues the P.V products.
template <int P8, bool SPLITPV>
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
      mbar_init(&sm.q_empty[i], 2);  // one commit per MMA issuer
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], 128);
      mbar_init(&sm.p_full[i], 128);
      mbar_init(&sm.pv_done[i], 1);
      for (int q = 0; q < 4; ++q) mbar_init(&sm.mufu_tok[i][q], 1);
    }
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 2);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 2);
    }
    sm.abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  pdl_prologue();

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kLowRegs));
    if (warp == 0) {
      // ---------------- TMA producer ----------------
      if (lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        bool ok = true;
        int tk = 0, tv = 0, it = 0;  // K / V tiles issued, items with keys started
        for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
          int qt, h, b;
          item_coords(p, w, qt, h, b);
          const int kvh = (int)((long long)h * p.Hkv / p.Hq);
          const int n = (item_keys(p, b) + BKV - 1) / BKV;
          if (n == 0) continue;
          const int qb = it & 1;
          ++it;
          if (!mbar_wait_bounded(&sm.q_empty[qb], (((it - 1) >> 1) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.q_full[qb], 2 * TILE_BYTES);
          const int q_row0 = (int)(b * p.q_rows_per_seq) + qt * ITEM_ROWS;
          tma_load_2d(sm.q[qb][0], &tmQ, &sm.q_full[qb], h * HD, q_row0);
          tma_load_2d(sm.q[qb][1], &tmQ, &sm.q_full[qb], h * HD, q_row0 + BQ);
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
    } else if (warp == 1 || warp == 2) {
      // ------- S issuers, one per softmax group (and its P.V without SPLITPV) -------
      // The whole warp walks the loop; one elected lane issues the tcgen05 ops.
      const int g = warp - 1;
      constexpr uint32_t idesc_s = make_idesc_bf16(BQ, BKV);
      constexpr uint32_t idesc_pv = make_idesc_bf16(BQ, HD) | (1u << 16);  // B (V) is MN-major
      const uint32_t s_tmem = tmem + S_COL0 + (uint32_t)g * BKV;
      const uint32_t p_tmem = tmem + P_COL0 + (uint32_t)g * (BKV / 2);
      const uint32_t o_tmem = tmem + O_COL0 + (uint32_t)g * HD;
      bool ok = true;
      int t = 0, it = 0;  // key tiles, items with keys
      for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
        int qt, h, b;
        item_coords(p, w, qt, h, b);
        const int n = (item_keys(p, b) + BKV - 1) / BKV;
        if (n == 0) continue;
        const int qb = it & 1;
        ok = mbar_wait_bounded(&sm.q_full[qb], (it >> 1) & 1, abort_flag);
        const uint64_t qdesc = make_sw128_desc(smem_u32(sm.q[qb][g]));
        // S_g of tile j, then P.V of tile j-1 (the order in which group g releases
        // S_g and then P_g); finally P.V of the item's last tile
        for (int j = 0; ok && j <= n; ++j) {
          if (j < n) {
            const int tt = t + j;
            const int sk = tt % kKStages;
            ok = mbar_wait_bounded(&sm.k_full[sk], (tt / kKStages) & 1, abort_flag);
            // S_g's columns are free once group g has read S_g(tt-1)
            if (ok && tt > 0) ok = mbar_wait_bounded(&sm.s_free[g], (uint32_t)(tt - 1) & 1u, abort_flag);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
              const uint64_t kdesc = make_sw128_desc(smem_u32(sm.k[sk]));
  #pragma unroll
              for (int k = 0; k < HD / 16; ++k) tc_mma_bf16(s_tmem, qdesc + 2 * k, kdesc + 2 * k, idesc_s, k > 0);
              tc_commit(&sm.s_full[g]);
              tc_commit(&sm.k_empty[sk]);
            }
            __syncwarp();
          }
          if (!SPLITPV && j >= 1) {
            const int tp = t + j - 1;
            const int sv = tp % kVStages;
            ok = mbar_wait_bounded(&sm.p_full[g], (uint32_t)tp & 1u, abort_flag);
            if (ok) ok = mbar_wait_bounded(&sm.v_full[sv], (tp / kVStages) & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
              const uint32_t vbase = smem_u32(sm.v[sv]);
  #pragma unroll
              for (int k = 0; k < BKV / 16; ++k) {
                const uint64_t bdesc = make_sw128_mn_desc(vbase + (uint32_t)k * 2048u, 16384u);
                tc_mma_bf16_ts(o_tmem, p_tmem + (uint32_t)k * 8u, bdesc, idesc_pv, (j > 1 || k > 0) ? 1u : 0u);
              }
              tc_commit(&sm.pv_done[g]);
              tc_commit(&sm.v_empty[sv]);
            }
            __syncwarp();
          }
        }
        if (!ok) break;
        if (elect_one()) tc_commit(&sm.q_empty[qb]);  // every S_g of this item has been issued
        __syncwarp();
        t += n;
        ++it;
      }
      if (!ok && lane == 0) {
        if (!*abort_flag) vla_record_error(VLA_DERR_ATTN_TIMEOUT);
        *abort_flag = 1;
      }
    } else if (SPLITPV && warp == 3) {
      // ---------------- P.V issuer for both groups ----------------
      // Per key tile, group 0's P.V then group 1's: the order in which the
      // groups finish their P (their exp phases alternate, group 0 first), so
      // the blocking waits follow the softmax warps instead of queueing behind
      // an S issue.
      constexpr uint32_t idesc_pv = make_idesc_bf16(BQ, HD) | (1u << 16);  // B (V) is MN-major
      bool ok = true;
      int t = 0;
      for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
        int qt, h, b;
        item_coords(p, w, qt, h, b);
        const int n = (item_keys(p, b) + BKV - 1) / BKV;
        if (n == 0) continue;
        for (int j = 0; ok && j < n; ++j) {
          const int tp = t + j;
          const int sv = tp % kVStages;
          for (int g = 0; g < 2; ++g) {
            ok = mbar_wait_bounded(&sm.p_full[g], (uint32_t)tp & 1u, abort_flag);
            if (ok) ok = mbar_wait_bounded(&sm.v_full[sv], (tp / kVStages) & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
              const uint32_t p_tmem = tmem + P_COL0 + (uint32_t)g * (BKV / 2);
              const uint32_t o_tmem = tmem + O_COL0 + (uint32_t)g * HD;
              const uint32_t vbase = smem_u32(sm.v[sv]);
  #pragma unroll
              for (int k = 0; k < BKV / 16; ++k) {
                const uint64_t bdesc = make_sw128_mn_desc(vbase + (uint32_t)k * 2048u, 16384u);
                tc_mma_bf16_ts(o_tmem, p_tmem + (uint32_t)k * 8u, bdesc, idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
              }
              tc_commit(&sm.pv_done[g]);
              tc_commit(&sm.v_empty[sv]);
            }
            __syncwarp();
          }
        }
        t += n;
      }
      if (!ok && lane == 0) {
        if (!*abort_flag) vla_record_error(VLA_DERR_ATTN_TIMEOUT);
        *abort_flag = 1;
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kHighRegs));
    // ---------------- softmax / output warps ----------------
    const int g = (warp - 4) >> 2;  // softmax group: query tile of the item
    const int q = warp & 3;         // TMEM lane quarter this warp may access
    const int row = g * BQ + q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t s_adr = tmem + lane_base + S_COL0 + (uint32_t)g * BKV;
    const uint32_t p_adr = tmem + lane_base + P_COL0 + (uint32_t)g * (BKV / 2);
    const uint32_t o_adr = tmem + lane_base + O_COL0 + (uint32_t)g * HD;
    bool ok = true;
    int t = 0;
    // the previous item's O_g is read out before this item's first P_g is
    // released (the next P.V, which overwrites O_g, waits for that P)
    bool pending = false;
    int pend_b = 0, pend_h = 0, pend_qt = 0;
    float pend_l = 0.f;
    for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
      int qt, h, b;
      item_coords(p, w, qt, h, b);
      const int Lk = item_keys(p, b);
      const int n = (Lk + BKV - 1) / BKV;
      if (n == 0) {
        const int qrow = qt * ITEM_ROWS + row;
        if (qrow < p.Lq) {
          uint4* dst = reinterpret_cast<uint4*>(p.o + (long long)b * p.o_batch + (long long)qrow * p.o_row +
                                                (long long)h * HD);
#pragma unroll
          for (int c8 = 0; c8 < HD / 8; ++c8) dst[c8] = make_uint4(0u, 0u, 0u, 0u);
        }
        continue;
      }
      float m = -INFINITY;  // running max of S * scale * log2(e), moved in steps > kRescaleLog2
      float l = 0.f;        // running row sum of P (at the scale of m)
      for (int j = 0; j < n; ++j) {
        const int tt = t + j;
        ok = mbar_wait_bounded(&sm.s_full[g], (uint32_t)tt & 1u, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const int key0 = j * BKV;
        float sr[BKV];
        tmem_ld128(s_adr, sr);
        tc_fence_before();
        mbar_arrive(&sm.s_free[g]);  // S_g(tt) is in registers: the tensor core may overwrite it
        if (key0 + BKV > Lk) {
#pragma unroll
          for (int c = 0; c < BKV; ++c)
            if (key0 + c >= Lk) sr[c] = -INFINITY;
        }
        // row max with 8 independent three-input max chains
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = sr[i];
#pragma unroll
        for (int c = 8; c < BKV; c += 16) {
#pragma unroll
          for (int i = 0; i < 8; ++i) mx8[i] = max3f(mx8[i], sr[c + i], sr[c + 8 + i]);
        }
        const float mx = max3f(max3f(mx8[0], mx8[1], mx8[2]), max3f(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])) *
                         p.scale_log2;
        const bool grow = mx > m + kRescaleLog2;
        const float alpha = grow ? ex2_fast(m - mx) : 1.f;
        if (grow) {
          m = mx;
          l *= alpha;
        }
        if (tt > 0) {
          // P_g and O_g were last used by P.V of tile tt-1 (no later P.V can have
          // completed: it needs the P this thread has not yet released)
          ok = mbar_wait_bounded(&sm.pv_done[g], (uint32_t)(tt - 1) & 1u, abort_flag);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          tc_fence_after();
        }
        if (j == 0 && pending) {
          finish_row(p, o_adr, pend_l, pend_b, pend_h, pend_qt * ITEM_ROWS + row);
          pending = false;
        }
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll 1
          for (int c = 0; c < HD; c += 16) {
            float o[16];
            uint32_t u[16];
            tmem_ld16(o_adr + c, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) u[i] = __float_as_uint(o[i] * alpha);
            tmem_st16(o_adr + c, u);
          }
        }
        const float mbase = m == -INFINITY ? 0.f : m;
        // the exp phase of tile tt: group 0 goes first (its first wait passes on
        // the fresh barrier), then the two groups alternate
        ok = mbar_wait_bounded(&sm.mufu_tok[g][q], g == 0 ? (((uint32_t)tt & 1u) ^ 1u) : ((uint32_t)tt & 1u),
                               abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        // P = exp2(s * scale*log2e - m) as one FFMA + MUFU.EX2, packed as bf16
        // pairs (keys 2c, 2c+1 in column c); row sum in 8 partial accumulators
        float rs8[8];
        uint32_t pk[BKV / 2];
#pragma unroll
        for (int c = 0; c < BKV; c += 2) {
          float x0, x1;
          fma2(sr[c], sr[c + 1], p.scale_log2, -mbase, x0, x1);
          float e0, e1;
          if (P8 > 0 && ((c >> 1) & 7) < P8) {
            ex2_poly2(x0, x1, e0, e1);
          } else {
            e0 = ex2_fast(x0);
            e1 = ex2_fast(x1);
          }
          if (c < 8) {
            rs8[c & 7] = e0;
            rs8[(c + 1) & 7] = e1;
          } else {
            add2(rs8[c & 7], rs8[(c + 1) & 7], e0, e1);
          }
          pk[c >> 1] = pack_bf16x2(e0, e1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.mufu_tok[g ^ 1][q]);  // the other group's warp on this sub-partition
        tmem_st32(p_adr, pk);
        tmem_st32(p_adr + BKV / 4, pk + BKV / 4);
        l += ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
        tc_fence_before();
        mbar_arrive(&sm.p_full[g]);
      }
      if (!ok) break;
      pending = true;
      pend_b = b, pend_h = h, pend_qt = qt, pend_l = l;
      t += n;
    }
    if (ok && pending) {
      ok = mbar_wait_bounded(&sm.pv_done[g], (uint32_t)(t - 1) & 1u, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        finish_row(p, o_adr, pend_l, pend_b, pend_h, pend_qt * ITEM_ROWS + row);
      }
    }
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
