// Pipelined short-sequence attention on the tensor cores (tcgen05 + TMA): the
// text prefix (113 keys, causal), the action expert's self-attention (50 keys,
// causal) and its cross-attention to the prefix (113 keys, key padding).
//
// Work item = one (sequence, kv head): the G = Hq / Hkv query heads that share
// the kv head are loaded as one stacked tile by a single 4-D TMA copy (tensor
// dims: 64 head elements, Hq heads, Lq queries, batch; box 64 x G x Lq x 1), so
// stacked row s is query s / G of head kvh * G + s % G; K and V of the kv head
// arrive by 4-D TMA copies of NK rows (rows past Lk are zero-filled by the
// TMA unit).  The item's R = G * Lq rows form T = ceil(R / 128) M-tiles.
//
// One persistent CTA per SM, warp-specialised, every hand-off an mbarrier:
//   warp 0  TMA producer: item k into smem stage k % stages (2-4 stages);
//   warp 1  S issuer (one thread): per M-tile u, S = Q K^T (128 x NK x 64)
//           into TMEM slot u % 4 (128 columns each);
//   warp 3  P.V issuer (one thread): O = P V (A = P from TMEM, V MN-major
//           from smem) into the slot's columns 64..127 once P is written;
//   warps 4..  NG softmax warpgroups (NG = 4, or 2) taking M-tiles in turn
//           (group g: tiles g, g + NG, ..., so with 4 groups two of them share
//           the full first tiles of 150-row items): thread r owns
//           row r, reads S, masks keys past kv_len / above the causal diagonal,
//           writes P = 2^(s * scale - m) as bf16 pairs over the S columns it
//           has read, keeps the fp32 row sum; then reads O, divides, and writes
//           the output row into the item's (finished) Q tile in smem;
//   warp 2  TMA store of the item's R output rows (same 4-D box as Q), then
//           releases the stage to the producer.
// So copies of items k+1.., the MMAs of tile u+1 and the softmax of tile u
// overlap instead of running as one dependent chain per item.
//
// Semantics are those of the other attention kernels: fp32 scores and
// softmax, exp2 with the scale folded in, P rounded to bf16 for P.V, causal
// masking key > query index, kv_len[b] limiting the keys of sequence b, rows
// without a visible key give 0.
#pragma once
#include "attention_short.cuh"
#include "common.cuh"

namespace vla {
namespace attn_pipe {

constexpr int HD = 64;
constexpr int MT = 128;
// threads of a CTA with NG softmax warpgroups (warps 0-3: producer, S issuer,
// store, P.V issuer)
__host__ __device__ constexpr int threads_for(int NG) { return 128 + 128 * NG; }
constexpr int kSlots = 4;
constexpr uint32_t SLOT_COLS = 128;
constexpr uint32_t O_OFF = 64;
constexpr uint32_t TMEM_COLS = kSlots * SLOT_COLS;  // 512: one CTA per SM
constexpr int kMaxStages = 4;
constexpr int kMaxTiles = 4;  // R = G * Lq <= 512 stacked rows per item
constexpr int TILE_BYTES = MT * HD * 2;

struct Params {
  int Lq, Lk, G, Hkv, batch, causal;
  int T;             // M-tiles per item
  int stages;        // smem stages
  uint32_t q_tx;     // bytes of one item's Q copy (R * 128)
  uint32_t q_region; // R * 128 rounded up to 1024 (K and V tiles follow)
  uint32_t stage_bytes;
  const int* kv_len;
  float scale_log2;
};

struct Bars {
  uint64_t full[kMaxStages], empty[kMaxStages], staged[kMaxStages];
  uint64_t s_full[kSlots], p_full[kSlots], o_full[kSlots], slot_free[kSlots];
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Bars) <= 1024, "barrier block");

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_4d(const void* tmap, uint32_t src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

__device__ __forceinline__ void fail(volatile int* abort_flag) {
  *abort_flag = 1;
  vla_record_error(VLA_DERR_ATTN_TIMEOUT);
}

// 32 lanes x 16 consecutive 32-bit TMEM columns from registers, then wait
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

template <int NK, int NG>
__global__ void __launch_bounds__(threads_for(NG), 1)
    attn_pipe_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars& bb = *reinterpret_cast<Bars*>(base);
  const uint32_t stage0 = smem_u32(base + 1024);
  // The Q copy fills R rows; the last M-tile's MMA also reads rows past R (up to
  // T * 128), which lie in this stage's K / V tiles or padding: garbage query
  // rows whose outputs are never stored.  stage_bytes >= T * 16 KB keeps those
  // reads inside the stage.
  const uint32_t q_region = p.q_region;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.batch * p.Hkv;
  const int my_items = (int)blockIdx.x < n_items ? (n_items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int my_tiles = my_items * p.T;
  volatile int* abort_flag = &bb.abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&bb.full[s], 1);
      mbar_init(&bb.empty[s], 1);
      mbar_init(&bb.staged[s], (uint32_t)(MT * p.T));
    }
    for (int j = 0; j < kSlots; ++j) {
      mbar_init(&bb.s_full[j], 1);
      mbar_init(&bb.p_full[j], MT);
      mbar_init(&bb.o_full[j], 1);
      mbar_init(&bb.slot_free[j], MT);
    }
    bb.abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&bb.tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bb.tmem_base;
  pdl_prologue();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      int issued = 0;
      bool ok = true;
      for (int k = 0; k < my_items; ++k) {
        const int it = (int)blockIdx.x + k * (int)gridDim.x;
        const int b = it / p.Hkv, kvh = it % p.Hkv;
        const int s = k % p.stages;
        if (!mbar_wait_bounded(&bb.empty[s], ((uint32_t)(k / p.stages) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t st = stage0 + (uint32_t)s * p.stage_bytes;
        mbar_arrive_expect_tx(&bb.full[s], p.q_tx + 2u * NK * 128u);
        tma_load_4d(st, &tq, &bb.full[s], 0, kvh * p.G, 0, b);
        tma_load_4d(st + q_region, &tk, &bb.full[s], 0, kvh, 0, b);
        tma_load_4d(st + q_region + NK * 128, &tv, &bb.full[s], 0, kvh, 0, b);
        ++issued;
      }
      if (!ok) fail(abort_flag);
      if (*abort_flag) {
        // let this CTA's copies in flight land before the CTA exits (bounded)
        for (int k = issued - 1; k >= 0 && k >= issued - p.stages; --k)
          mbar_wait_bounded(&bb.full[k % p.stages], (uint32_t)(k / p.stages) & 1u, nullptr, 2000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------- S issuer ----------------
    // S(u) = Q K^T of every M-tile in order: the first tile of an item waits
    // for its copies, every tile for its TMEM slot (freed once the softmax
    // warps have read out O of tile u - kSlots).  The P.V products have their
    // own issuing thread (warp 3): one thread issuing both took 300-600 cycles
    // per four-MMA group plus its polling and set the kernel's pace.
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(MT, NK);
      bool ok = true;
      int t = 0, s = 0, slot = 0;
      uint32_t full_par = 0, free_par = 1;  // parities of full[s] and slot_free[slot]
      for (int u = 0; u < my_tiles; ++u) {
        if ((t == 0 && !mbar_wait_bounded(&bb.full[s], full_par, abort_flag)) ||
            !mbar_wait_bounded(&bb.slot_free[slot], free_par, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t st = stage0 + (uint32_t)s * p.stage_bytes;
        const uint64_t qd = make_sw128_desc(st + (uint32_t)t * TILE_BYTES), kd = make_sw128_desc(st + q_region);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          tc_mma_bf16(tmem + (uint32_t)slot * SLOT_COLS, qd + 2 * kk, kd + 2 * kk, idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(&bb.s_full[slot]);
        if (++slot == kSlots) slot = 0, free_par ^= 1u;
        if (++t == p.T) {
          t = 0;
          if (++s == p.stages) s = 0, full_par ^= 1u;
        }
      }
      if (!ok) fail(abort_flag);
    }
  } else if (warp == 3) {
    // ---------------- P.V issuer ----------------
    // O(w) = P V of every M-tile in order, once the softmax warps have written
    // P(w) into the slot (the item's copies have landed: its S was issued after
    // them; the wait on full[s] only makes that explicit and passes at once).
    if (lane == 0) {
      constexpr uint32_t idesc_pv = make_idesc_bf16(MT, HD) | (1u << 16);  // B (V) MN-major
      bool ok = true;
      int t = 0, s = 0, slot = 0;
      uint32_t full_par = 0, p_par = 0;
      for (int w = 0; w < my_tiles; ++w) {
        if ((t == 0 && !mbar_wait_bounded(&bb.full[s], full_par, abort_flag)) ||
            !mbar_wait_bounded(&bb.p_full[slot], p_par, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sv = stage0 + (uint32_t)s * p.stage_bytes + q_region + NK * 128;
        const uint32_t sc = tmem + (uint32_t)slot * SLOT_COLS;
#pragma unroll
        for (int kk = 0; kk < NK / 16; ++kk)
          attn_sq::mma_ts(sc + O_OFF, sc + (uint32_t)kk * 8u, attn_sq::mn_desc(sv + (uint32_t)kk * 2048u), idesc_pv,
                          kk > 0 ? 1u : 0u);
        tc_commit(&bb.o_full[slot]);
        if (++slot == kSlots) slot = 0, p_par ^= 1u;
        if (++t == p.T) {
          t = 0;
          if (++s == p.stages) s = 0, full_par ^= 1u;
        }
      }
      if (!ok) fail(abort_flag);
    }
  } else if (warp == 2) {
    // ---------------- output stores ----------------
    if (lane == 0) {
      bool ok = true;
      for (int k = 0; k < my_items; ++k) {
        const int s = k % p.stages;
        if (!mbar_wait_bounded(&bb.staged[s], (uint32_t)(k / p.stages) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        const int it = (int)blockIdx.x + k * (int)gridDim.x;
        const int b = it / p.Hkv, kvh = it % p.Hkv;
        tma_store_4d(&to, stage0 + (uint32_t)s * p.stage_bytes, 0, kvh * p.G, 0, b);
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // the stage may be refilled
        mbar_arrive(&bb.empty[s]);
      }
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
      if (!ok) fail(abort_flag);
    }
  } else if (warp >= 4) {
    // ---------------- softmax + output rows ----------------
    const int wg = (warp - 4) >> 2, quarter = warp & 3;  // M-tiles u = wg, wg + NG, ...
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int R = p.G * p.Lq;
    bool ok = true;
    for (int u = wg; u < my_tiles; u += NG) {
      const int k = u / p.T, t = u % p.T, s = k % p.stages;
      const int it = (int)blockIdx.x + k * (int)gridDim.x;
      const int b = it / p.Hkv;
      const int slot = u % kSlots;
      const uint32_t par = (uint32_t)(u / kSlots) & 1u;
      const uint32_t sc = tmem + lane_base + (uint32_t)slot * SLOT_COLS;
      const int srow = t * MT + r;
      const bool live = t * MT + quarter * 32 < R;  // warp-uniform: some row of this warp is real
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bb.s_full[slot], par, abort_flag));
      if (!ok) break;
      tc_fence_after();
      float l = 0.f;
      if (live) {
        int lk = p.Lk;
        if (p.kv_len != nullptr) lk = max(0, min(lk, __ldg(p.kv_len + b)));
        int kend = lk;
        if (p.causal) kend = min(kend, srow / p.G + 1);
        float m = -INFINITY;
#pragma unroll
        for (int h = 0; h < NK / 32; ++h) {
          float v[32];
          tmem_ld32(sc + 32 * h, v);
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (32 * h + c < kend) m = fmaxf(m, v[c]);
        }
        const float mb = m == -INFINITY ? 0.f : m * p.scale_log2;
        // P of keys 32h..32h+31 goes to columns 16h..16h+15, all of them read
        // already (this chunk's own load included)
#pragma unroll
        for (int h = 0; h < NK / 32; ++h) {
          uint32_t pk[16];
          float v[32];
          tmem_ld32(sc + 32 * h, v);
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const int key = 32 * h + c;
            const float e0 = key < kend ? attn_sq::ex2f(fmaf(v[c], p.scale_log2, -mb)) : 0.f;
            const float e1 = key + 1 < kend ? attn_sq::ex2f(fmaf(v[c + 1], p.scale_log2, -mb)) : 0.f;
            l += e0 + e1;
            pk[c >> 1] = pack_bf16x2(e0, e1);
          }
          tmem_st16u(sc + 16 * h, pk);
        }
      }
      tc_fence_before();
      mbar_arrive(&bb.p_full[slot]);
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bb.o_full[slot], par, abort_flag));
      if (!ok) break;
      tc_fence_after();
      // O in 32-column halves (16-column pieces with four softmax groups, for
      // their 96-register budget); the output row replaces query row srow of
      // the item's Q tile (S of this tile has completed), in the tile's
      // 128-byte swizzle
      constexpr int OC = NG == 4 ? 16 : 32;
      const bool store_row = live && srow < R;
      const uint32_t row_addr = stage0 + (uint32_t)s * p.stage_bytes + (uint32_t)srow * 128u;
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int piece = 0; piece < HD / OC; ++piece) {
        float o[OC];
        if (live) {
          if constexpr (OC == 16)
            tmem_ld16(sc + O_OFF + (uint32_t)(OC * piece), o);
          else
            tmem_ld32(sc + O_OFF + (uint32_t)(OC * piece), o);
        }
        if (piece == HD / OC - 1) {
          tc_fence_before();
          mbar_arrive(&bb.slot_free[slot]);
        }
        if (store_row) {
#pragma unroll
          for (int j = 0; j < OC / 8; ++j) {
            const int c8 = (OC / 8) * piece + j;
            float t8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) t8[i] = o[8 * j + i] * inv;
            const uint4 w4 = pack_bf16x8(t8);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row_addr +
                                                                          (uint32_t)((c8 ^ (srow & 7)) << 4)),
                         "r"(w4.x), "r"(w4.y), "r"(w4.z), "r"(w4.w)
                         : "memory");
          }
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the TMA store
      mbar_arrive(&bb.staged[s]);
    }
    if (!ok) fail(abort_flag);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace attn_pipe
}  // namespace vla
