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
// warps 2..9  : epilogue — tcgen05.ld 32 lanes x 16 columns, fused bias /
//               GELU-tanh / SwiGLU / RoPE / Euler / residual.  Output chunks
//               of 32 rows x 32 columns go through a per-warp shared-memory
//               staging buffer and a TMA tensor store (full-line global writes;
//               direct per-row stores touch 32 lines per warp instruction and
//               made the epilogue the bound of short-K GEMMs); Euler and
//               row-scatter epilogues store directly.
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
  int b_static;  // B is not written by earlier work in the stream (prefetched before the PDL wait)
  int a_rows;    // rows of each A copy (0 = BM); 64 when M <= 64: the MMA still reads BM rows,
                 // the rows past 64 are stale shared memory whose outputs (rows >= M) are never stored
  int tma_c;  // stores go through shared memory and the C tensor map
  int tma_r;  // the residual arrives in the same staging buffers through its tensor map
  int M, N;
};

// Per-warp output staging for the TMA store: two 2 KB buffers (32 rows x 64 B),
// used alternately; one bulk-async group per stored chunk.
constexpr int kStageC = 32 * 64;
constexpr int kEpiStoreBytes = kEpiWarps * 2 * kStageC;
constexpr int kSmemLimit = 232448;  // dynamic shared memory per block on sm_100
constexpr int kBarrierBytes = 512;  // mbarriers, TMEM slot and abort flag

struct EpiStore {
  uint32_t buf;   // shared address of this warp's two staging buffers
  int sb;         // buffer the next chunk uses
  int row0;       // output row of the warp's lane 0
  uint64_t* rbar; // two barriers: residual chunk landed in buffer 0 / 1
  uint32_t rpar;  // bit b: phase parity of the next residual arrival in buffer b
  volatile int* abort_flag;
};

// Issue the TMA load of the residual chunk at (col, res_row) into staging
// buffer `b` (lane 0).  `pending_ok` stores may still be reading staging
// buffers: 1 when `b` is the buffer used two chunks ago, 0 when it is the one
// the previous chunk used.
__device__ __forceinline__ void res_load(const CUtensorMap* tmR, EpiStore& es, int b, int col, int res_row,
                                         int pending_ok, int lane) {
  if (lane == 0) {
    if (pending_ok)
      asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    else
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    mbar_arrive_expect_tx(&es.rbar[b], (uint32_t)kStageC);
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            es.buf + (uint32_t)b * (uint32_t)kStageC),
        "l"(reinterpret_cast<uint64_t>(tmR)), "r"(col), "r"(res_row), "r"(smem_u32(&es.rbar[b]))
        : "memory");
  }
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, uint32_t smem, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(smem), "r"(x), "r"(y)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t a, const uint4& v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// Stage this warp's 32 rows x (NVEC * 8) columns (lane = row) and store them
// with TMA at column `col`.  The layout matches the tensor map's swizzle
// (64-byte for 4 vectors a row, 32-byte for 2), which also keeps the 16-byte
// shared stores of 8 consecutive rows on distinct banks.
template <int NVEC>
__device__ __forceinline__ void stage_store(const CUtensorMap* tm, EpiStore& es, const uint4* v, int lane, int col) {
  const uint32_t b = es.buf + (uint32_t)es.sb * (uint32_t)kStageC;
  // the store that last read this buffer (two chunks ago) must have finished reading
  if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
  __syncwarp();
#pragma unroll
  for (int i = 0; i < NVEC; ++i) {
    const int phys = NVEC == 4 ? (i ^ ((lane >> 1) & 3)) : (i ^ ((lane >> 2) & 1));
    st_shared_v4(b + (uint32_t)(lane * NVEC * 16 + phys * 16), v[i]);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) tma_store_2d(tm, b, col, es.row0);
  es.sb ^= 1;
}

// RoPE's two 16-column pieces of one head (v0: columns col0.., v1: col1..),
// staged in the warp's two buffers and stored as one bulk group: one wait, one
// proxy fence and one commit per pair instead of per piece.
__device__ __forceinline__ void stage_store_pair16(const CUtensorMap* tm, EpiStore& es, const uint4* v0, const uint4* v1,
                                                   int lane, int col0, int col1) {
  if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int phys = i ^ ((lane >> 2) & 1);
    st_shared_v4(es.buf + (uint32_t)(lane * 32 + phys * 16), v0[i]);
    st_shared_v4(es.buf + (uint32_t)kStageC + (uint32_t)(lane * 32 + phys * 16), v1[i]);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(tm)),
                 "r"(es.buf), "r"(col0), "r"(es.row0)
                 : "memory");
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(tm)),
                 "r"(es.buf + (uint32_t)kStageC), "r"(col1), "r"(es.row0)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
}

// Stage-and-store with the residual already in the staging buffer: this lane's
// row is read from shared memory, added to v, and the sum stored in place.
__device__ __forceinline__ void res_stage_store(const CUtensorMap* tmC, EpiStore& es, float* v, int lane, int col) {
  const uint32_t b = es.buf + (uint32_t)es.sb * (uint32_t)kStageC;
  const bool ok = mbar_wait_bounded(&es.rbar[es.sb], (es.rpar >> es.sb) & 1u, es.abort_flag);
  es.rpar ^= 1u << es.sb;
  if (!ok && lane == 0) {  // the result is not valid; the error word says so
    if (!*es.abort_flag) vla_record_error(VLA_DERR_GEMM_EPILOGUE_TIMEOUT);
    *es.abort_flag = 1;
  }
  uint4 pk[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t a = b + (uint32_t)(lane * 64 + ((i ^ ((lane >> 1) & 3)) * 16));
    uint4 r;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
    float rf[8];
    unpack_bf16x8(r, rf);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[8 * i + e] += rf[e];
    pk[i] = pack_bf16x8(v + 8 * i);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) st_shared_v4(b + (uint32_t)(lane * 64 + ((i ^ ((lane >> 1) & 3)) * 16)), pk[i]);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) tma_store_2d(tmC, b, col, es.row0);
  es.sb ^= 1;
}

// All of this warp's TMA stores have completed (issued by lane 0).
__device__ __forceinline__ void stage_drain(int lane) {
  if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  __syncwarp();
}

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BUDGET = kSmemLimit - 1024 - kBarrierBytes - kEpiStoreBytes;
  static constexpr int STAGES = (BUDGET / STAGE_BYTES) > 8 ? 8 : (BUDGET / STAGE_BYTES);
  static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + kEpiStoreBytes + kBarrierBytes + 1024;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "UMMA N (multiple of 32 for the epilogue chunks)");
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

__device__ __forceinline__ long long res_row(const DevEpi& ep, int m) {
  return ep.res_row_mod > 0 ? (long long)(m % ep.res_row_mod) : (long long)m;
}

// Residual (bf16) and bias values of one 32-column chunk, fetched ahead of use.
struct Chunk32 {
  uint4 r[4];
  uint4 b[4];
};

// N is a multiple of 16, so a chunk is either 32 columns wide or the 16-column
// tail of the row; nothing at or beyond column N is read or written.
__device__ __forceinline__ int chunk_vecs(const DevEpi& ep, int n) { return (n + 32 <= ep.N) ? 4 : 2; }

__device__ __forceinline__ void prefetch32(const DevEpi& ep, int m, int n, bool row_ok, Chunk32& c) {
  const int nv = chunk_vecs(ep, n);
#pragma unroll
  for (int i = 0; i < 4; ++i) c.r[i] = c.b[i] = make_uint4(0u, 0u, 0u, 0u);
  if (ep.residual != nullptr && row_ok && !ep.tma_r) {
    const uint4* rp = reinterpret_cast<const uint4*>(ep.residual + res_row(ep, m) * ep.ldr + n);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i < nv) c.r[i] = rp[i];
  }
  if (ep.bias != nullptr) {
    const uint4* bp = reinterpret_cast<const uint4*>(ep.bias + n);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i < nv) c.b[i] = __ldg(bp + i);
  }
}

// Finish the chunk [n, n+32) (or its 16-column tail) of row m held in v[] (fp32, alpha applied).
// With ep.tma_c every lane takes part (rows at or past M are clipped by the
// tensor store); otherwise rows past M return early.
__device__ __forceinline__ void finish32(const DevEpi& ep, int m, int n, long long orow, float* v, bool row_ok,
                                         const Chunk32& c, const CUtensorMap* tmC, EpiStore& es, int lane) {
  if (ep.bias != nullptr) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float b[8];
      unpack_bf16x8(c.b[i], b);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[8 * i + e] += b[e];
    }
  }
  if (ep.act == VLA_ACT_GELU_TANH) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = gelu_tanh_f(v[i]);
  }
  if (ep.tma_c) {  // never Euler: the residual follows bias / GELU directly
    if (ep.tma_r) {
      res_stage_store(tmC, es, v, lane, n);
      return;
    }
    if (ep.residual != nullptr) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float r[8];
        unpack_bf16x8(c.r[i], r);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[8 * i + e] += r[e];
      }
    }
    uint4 pk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pk[i] = pack_bf16x8(v + 8 * i);
    stage_store<4>(tmC, es, pk, lane, n);
    return;
  }
  if (!row_ok) return;
  const int nv = chunk_vecs(ep, n);
  if (ep.act == VLA_ACT_EULER) {
    float* xp = ep.euler_x + (long long)m * ep.ldx + n;
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      if (i >= 8 * nv) break;
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
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float r[8];
      unpack_bf16x8(c.r[i], r);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[8 * i + e] += r[e];
    }
  }
  uint4* cp = reinterpret_cast<uint4*>(ep.C + orow * ep.ldc + n);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (i < nv) cp[i] = pack_bf16x8(v + 8 * i);
}

// Partial accumulators of other CTAs added to this CTA's TMEM values right after
// each TMEM load (split-K, gemm_splitk.cuh); the plain kernels use NoPartial,
// which compiles to nothing.
struct NoPartial {
  __device__ __forceinline__ void add16(int, float*) const {}
};

// RoPE epilogue of row m over the 64-wide heads of a BN-wide tile: rotate pairs
// (d, d+32), d < 32.  The pairs split into two halves (d < 16, d >= 16); with an
// even number of warps per lane quarter each warp owns one half of every head it
// visits, so it loads that half's 16 cos + 16 sin of row m's position once per
// tile and reuses them for all heads (every thread reads its own table row, so
// each table load touches 32 cache lines: reloading it per head made the RoPE
// GEMMs bound by L1 wavefronts).
template <int BN, class PS = NoPartial>
__device__ __forceinline__ void rope_tile(const DevEpi& ep, uint32_t taddr, int m, int n0, long long orow,
                                          bool row_ok, int part, int nparts, const CUtensorMap* tmC, EpiStore& es,
                                          int lane, const PS& ps = PS()) {
  const bool split = (nparts & 1) == 0;
  const int hq0 = split ? (part & 1) : 0;
  const int hq1 = split ? (part & 1) : 1;
  const int h0 = split ? (part >> 1) : part;
  const int hstep = split ? (nparts >> 1) : nparts;
  const float* cs = ep.rope_cs + (long long)(m % ep.rope_seq) * 64;
#pragma unroll 1
  for (int hq = hq0; hq <= hq1; ++hq) {
    float cc[16], ss[16];
    bool have_cs = false;
#pragma unroll 1
    for (int h = h0; h < BN / 64; h += hstep) {
      const int n = n0 + 64 * h;
      if (n >= ep.N) break;
      float lo[16], hi[16];
      tmem_ld16x2(taddr + 64 * h + 16 * hq, taddr + 64 * h + 32 + 16 * hq, lo, hi);
      ps.add16(64 * h + 16 * hq, lo);
      ps.add16(64 * h + 32 + 16 * hq, hi);
      if (!row_ok && !ep.tma_c) continue;
      if (ep.alpha != 1.f) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          lo[i] *= ep.alpha;
          hi[i] *= ep.alpha;
        }
      }
      if (ep.bias != nullptr) {  // the same address on every lane: one broadcast load
        float b[8];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(ep.bias + n + 16 * hq) + i), b);
#pragma unroll
          for (int e = 0; e < 8; ++e) lo[8 * i + e] += b[e];
          unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(ep.bias + n + 32 + 16 * hq) + i), b);
#pragma unroll
          for (int e = 0; e < 8; ++e) hi[8 * i + e] += b[e];
        }
      }
      if (n < ep.rope_ncols) {
        if (!have_cs) {
          const float4* c4 = reinterpret_cast<const float4*>(cs + 16 * hq);
          const float4* s4 = reinterpret_cast<const float4*>(cs + 32 + 16 * hq);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 c = __ldg(c4 + i), sn = __ldg(s4 + i);
            cc[4 * i] = c.x, cc[4 * i + 1] = c.y, cc[4 * i + 2] = c.z, cc[4 * i + 3] = c.w;
            ss[4 * i] = sn.x, ss[4 * i + 1] = sn.y, ss[4 * i + 2] = sn.z, ss[4 * i + 3] = sn.w;
          }
          have_cs = true;
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float a = lo[e], b = hi[e];
          lo[e] = a * cc[e] - b * ss[e];
          hi[e] = b * cc[e] + a * ss[e];
        }
      }
      if (ep.tma_c) {  // (no residual: the host sends RoPE + residual down the direct path)
        const uint4 plo[2] = {pack_bf16x8(lo), pack_bf16x8(lo + 8)};
        const uint4 phi[2] = {pack_bf16x8(hi), pack_bf16x8(hi + 8)};
        stage_store_pair16(tmC, es, plo, phi, lane, n + 16 * hq, n + 32 + 16 * hq);
        continue;
      }
      if (ep.residual != nullptr) {
        const bf16* rp = ep.residual + res_row(ep, m) * ep.ldr + n;
        float r[8];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          unpack_bf16x8(reinterpret_cast<const uint4*>(rp + 16 * hq)[i], r);
#pragma unroll
          for (int e = 0; e < 8; ++e) lo[8 * i + e] += r[e];
          unpack_bf16x8(reinterpret_cast<const uint4*>(rp + 32 + 16 * hq)[i], r);
#pragma unroll
          for (int e = 0; e < 8; ++e) hi[8 * i + e] += r[e];
        }
      }
      bf16* cp = ep.C + orow * ep.ldc + n;
      reinterpret_cast<uint4*>(cp + 16 * hq)[0] = pack_bf16x8(lo);
      reinterpret_cast<uint4*>(cp + 16 * hq)[1] = pack_bf16x8(lo + 8);
      reinterpret_cast<uint4*>(cp + 32 + 16 * hq)[0] = pack_bf16x8(hi);
      reinterpret_cast<uint4*>(cp + 32 + 16 * hq)[1] = pack_bf16x8(hi + 8);
    }
  }
}

// Epilogue of one 128 x BN accumulator tile for one row m; warps that share a
// lane quarter split the column chunks round-robin (part of nparts).
template <int BN, class PS = NoPartial>
__device__ __forceinline__ void epilogue_tile(const DevEpi& ep, uint32_t taddr, int m, int n0, int part,
                                              int nparts, const CUtensorMap* tmC, const CUtensorMap* tmR,
                                              EpiStore& es, int lane, const PS& ps = PS()) {
  const bool row_ok = m < ep.M;
  const long long orow = out_row(ep, m);
  if (ep.act == VLA_ACT_ROPE) {
    rope_tile<BN, PS>(ep, taddr, m, n0, orow, row_ok, part, nparts, tmC, es, lane, ps);
  } else if (ep.act == VLA_ACT_SWIGLU) {
#pragma unroll 1
    for (int c = 32 * part; c < BN; c += 32 * nparts) {
      float g[16], u[16];
      tmem_ld16(taddr + c, g);
      tmem_ld16(taddr + c + 16, u);
      ps.add16(c, g);
      ps.add16(c + 16, u);
      const int n = n0 + c;
      if (n >= ep.N) break;
      if (!row_ok && !ep.tma_c) continue;
      if (ep.alpha != 1.f) {
#pragma unroll
        for (int i = 0; i < 16; ++i) g[i] = silu_f(g[i] * ep.alpha) * (u[i] * ep.alpha);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) g[i] = silu_f(g[i]) * u[i];
      }
      const int nc = n >> 1;
      if (ep.residual != nullptr && row_ok) {
        const uint4* rp = reinterpret_cast<const uint4*>(ep.residual + res_row(ep, m) * ep.ldr + nc);
        float r[16];
        unpack_bf16x8(rp[0], r);
        unpack_bf16x8(rp[1], r + 8);
#pragma unroll
        for (int i = 0; i < 16; ++i) g[i] += r[i];
      }
      if (ep.tma_c) {
        const uint4 pk[2] = {pack_bf16x8(g), pack_bf16x8(g + 8)};
        stage_store<2>(tmC, es, pk, lane, nc);
        continue;
      }
      uint4* cp = reinterpret_cast<uint4*>(ep.C + orow * ep.ldc + nc);
      cp[0] = pack_bf16x8(g);
      cp[1] = pack_bf16x8(g + 8);
    }
  } else {
    // 32-column chunks; the next chunk's residual / bias loads are issued before
    // this chunk's stores so their latency overlaps (C may alias the residual).
    const int step = 32 * nparts;
    int c = 32 * part;
    Chunk32 cur, nxt;
    // residual rows of this warp's 32 output rows (blocks of 32 never straddle
    // the res_row_mod period: the host only sets tma_r when it divides by 32)
    const int rrow = (int)res_row(ep, es.row0);
    if (c < BN && n0 + c < ep.N) {
      prefetch32(ep, m, n0 + c, row_ok, cur);
      if (ep.tma_r) res_load(tmR, es, es.sb, n0 + c, rrow, 1, lane);
    }
#pragma unroll 1
    for (; c < BN; c += step) {
      const int n = n0 + c;
      if (n >= ep.N) break;
      float v[32];
      tmem_ld16(taddr + c, v);
      tmem_ld16(taddr + c + 16, v + 16);
      ps.add16(c, v);
      ps.add16(c + 16, v + 16);
      const bool more = c + step < BN && n + step < ep.N;
      if (more) {
        prefetch32(ep, m, n + step, row_ok, nxt);
        if (ep.tma_r) res_load(tmR, es, es.sb ^ 1, n + step, rrow, 0, lane);
      }
      if (ep.alpha != 1.f) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= ep.alpha;
      }
      finish32(ep, m, n, orow, v, row_ok, cur, tmC, es, lane);
      if (more) cur = nxt;
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR, DevEpi ep,
                        int M, int N, int K) {
  using Cf = Cfg<BN>;
  constexpr int STAGES = Cf::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + STAGES * Cf::A_BYTES;
  uint8_t* sC = sB + STAGES * Cf::B_BYTES;  // output staging (1024-byte aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(sC + kEpiStoreBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* rbar = tempty + 2;  // [kEpiWarps][2]: residual chunk landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 2 * kEpiWarps);
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
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&rbar[i], 1);
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (ep.tma_c) tma_prefetch_desc(&tmC);
    if (ep.tma_r) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cf::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // Weights do not depend on the previous kernel: the producer stages the B
  // tiles of its first tile's first k-blocks before waiting for that kernel
  // (their stages are armed for the full A + B bytes; A follows after the wait).
  int prefetched = 0;
  const uint32_t stage_tx = (uint32_t)((ep.a_rows > 0 ? ep.a_rows : BM) * BK * 2 + Cf::B_BYTES);
  if (warp == 0 && lane == 0 && ep.b_static && (int)blockIdx.x < num_tiles) {
    int mb, nb;
    tile_coords(blockIdx.x, num_m, num_n, mb, nb);
    for (; prefetched < STAGES && prefetched < num_kb; ++prefetched) {
      mbar_arrive_expect_tx(&full[prefetched], stage_tx);
      tma_load_2d(sB + prefetched * Cf::B_BYTES, &tmB, &full[prefetched], prefetched * BK, nb * BN);
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");

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
          if (it < prefetched) {  // stage armed and its B tile in flight since the prologue
            tma_load_2d(sA + s * Cf::A_BYTES, &tmA, &full[s], kb * BK, mb * BM);
            ++it;
            continue;
          }
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], stage_tx);
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
      const int issued = it > prefetched ? it : prefetched;
      const int first = issued > STAGES ? issued - STAGES : 0;
      for (int j = first; j < issued; ++j)
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
    EpiStore es{smem_u32(sC) + (uint32_t)((warp - 2) * 2 * kStageC), 0, 0, rbar + 2 * (warp - 2), 0u, abort_flag};
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
      es.row0 = mb * BM + q * 32;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(as * BN);
      epilogue_tile<BN>(ep, taddr, m, nb * BN, part, kEpiWarps / 4, &tmC, &tmR, es, lane);
      tc_fence_before();
      mbar_arrive(&tempty[as]);
      ++tc;
    }
    if (ep.tma_c) stage_drain(lane);
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
