// Host launcher of the tcgen05 GEMM: argument validation, tile-width choice,
// tensor maps, persistent grid sizing (one CTA per SM).
#pragma once
#include "gemm.cuh"
#include "gemm2.cuh"
#include "gemm_splitk.cuh"
#include "gemm_skinny.cuh"
#include "host_common.cuh"

namespace vla {
namespace gemm {

// Estimated relative cost of a tile width: waves of 128 x BN tiles over the
// SMs, each tile costing (BN + 48) column-units (48 ~ fixed A-tile and
// epilogue overhead per tile).
static int choose_bn(int64_t M, int64_t N, int act, int num_sms) {
  const int cands[8] = {256, 224, 192, 160, 128, 96, 64, 32};
  int best = 0;
  double best_cost = 1e300;
  for (int bn : cands) {
    if (act == VLA_ACT_ROPE && bn % 64 != 0) continue;
    const int64_t tiles = ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
    const int64_t waves = (tiles + num_sms - 1) / num_sms;
    const double cost = (double)waves * (bn + 48);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

// Largest number of co-resident 2-CTA clusters of the pair kernel<BN, KPS> (GPC
// boundaries can leave SMs without a partner), cached per device and width.
template <int BN, int KPS>
static int max_pair_clusters() {
  static int cached[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (cached[dev] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cfg2<BN, KPS>::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_bf16_tc2_kernel<BN, KPS>, &cfg) != cudaSuccess || n <= 0)
      n = device_info().num_sms / 2;
    cached[dev] = n;
  }
  return cached[dev];
}

template <int BN, int KPS>
static int launch_bn2_k(const CUtensorMap& ta, const void* A, int64_t lda, const void* B, int64_t ldb,
                        const CUtensorMap& tc, const CUtensorMap& tr, const DevEpi& ep, int64_t M, int64_t N,
                        int64_t K, cudaStream_t st) {
  using Cf = Cfg2<BN, KPS>;
  CUtensorMap tb, ta3, tb3;
  int rc = make_tmap_bf16_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK, BN / 2);
  if (rc) return rc;
  if (KPS > 1) {
    rc = make_tmap_bf16_kslab(&ta3, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BM, KPS);
    if (!rc) rc = make_tmap_bf16_kslab(&tb3, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BN / 2, KPS);
    if (rc) return rc;
  } else {
    ta3 = ta;
    tb3 = tb;
  }
  static thread_local int attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    VLA_CUDA_TRY(cudaFuncSetAttribute(gemm_bf16_tc2_kernel<BN, KPS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      Cf::SMEM_BYTES));
    VLA_CUDA_TRY(
        cudaFuncSetAttribute(gemm_bf16_tc2_kernel<BN, KPS>, cudaFuncAttributeNonPortableClusterSizeAllowed, 0));
    attr_dev_mask |= 1 << (dev & 31);
  }
  const int64_t tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN);
  const int clusters = max_pair_clusters<BN, KPS>();
  const int grid = 2 * (int)(tiles < clusters ? tiles : clusters);
  prof_begin(st);
  launch_k_cluster(gemm_bf16_tc2_kernel<BN, KPS>, 2, dim3(grid), dim3(kThreads), Cf::SMEM_BYTES, st, ta, tb, ta3, tb3,
                   tc, tr, ep, (int)M, (int)N, (int)K);
  {
    const double out_cols = ep.act == VLA_ACT_SWIGLU ? N / 2 : N;
    double bytes = 2.0 * ((double)M * K + (double)N * K + (double)M * out_cols);
    if (ep.residual) bytes += 2.0 * M * out_cols;
    if (ep.act == VLA_ACT_EULER) bytes += 8.0 * M * N;
    prof_end(st, VLA_KIND_GEMM, 2.0 * M * N * K, bytes, M, N, K, BN, 2);
  }
  return launch_status("gemm_bf16_tc2");
}

// k-blocks per stage of the pair kernel: 2 (one k-slab box per operand fills
// a stage; measured +6 to +14 % on the 720- to 960-wide GEMMs of the step, equal
// on the rest, and 4 no better); VLA_GEMM_PAIR_KPS=1|2|4 overrides (A/B).
static int pair_kps(int64_t K) {
  static const int env = [] {
    const char* v = getenv("VLA_GEMM_PAIR_KPS");
    const int k = v ? atoi(v) : 2;
    return (k == 2 || k == 4) ? k : 1;
  }();
  return K / BK >= env ? env : 1;
}

template <int BN>
static int launch_bn2(const CUtensorMap& ta, const void* A, int64_t lda, const void* B, int64_t ldb,
                      const CUtensorMap& tc, const CUtensorMap& tr, const DevEpi& ep, int64_t M, int64_t N, int64_t K,
                      cudaStream_t st) {
  const int kps = pair_kps(K);
  if constexpr (Cfg2<BN, 4>::STAGES >= 2) {
    if (kps == 4) return launch_bn2_k<BN, 4>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
  }
  if (kps >= 2) return launch_bn2_k<BN, 2>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
  return launch_bn2_k<BN, 1>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
}

// One-CTA tile or CTA pair (gemm2.cuh).  The pair halves each SM's B staging
// traffic and doubles the MMA's M; inside the full C4 step (B = 256) it measured
// faster on B200 for every GEMM shape of the step (+3-25 % per shape).  With two
// k-blocks per pair stage it also wins on the expert's 3200-row GEMMs of the
// B = 64 step (chunk +1.5 %); small M (the single-observation blocks, below 2048
// rows) stays on one CTA per tile.
static int choose_ctas(int64_t M, int bn) {
  return (M >= 16 * BM && bn >= 64) ? 2 : 1;
}

// Tile width of a CTA-pair launch.  With two k-blocks per stage (pair_kps) a
// tile's main loop costs about its width (the MMA's pace) plus a fixed share
// (the copies' and barriers' per-stage costs, the epilogue tail); a launch
// costs its waves of 256 x BN tiles over the pairs.  Measured at M = 12800
// (graph-timed TFLOP/s, widths 256 / 192 / 160 / 128): N = 720 K = 960
// 793 / 853 / 728 / 660, N = 1600 K = 720 973 / 890 / 924 / 805, which
// waves x (BN + 96) ranks correctly; equal costs keep the wider tile.
static int choose_bn_pair(int64_t M, int64_t N, int act, int num_sms) {
  const int cands[5] = {256, 224, 192, 160, 128};
  const int64_t pairs = num_sms / 2 > 0 ? num_sms / 2 : 1;
  int best = 0;
  int64_t best_cost = 0;
  for (int bn : cands) {
    if (act == VLA_ACT_ROPE && bn % 64 != 0) continue;
    const int64_t tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + bn - 1) / bn);
    const int64_t waves = (tiles + pairs - 1) / pairs;
    const int64_t cost = waves * (bn + 96);
    if (best == 0 || cost < best_cost) {
      best = bn;
      best_cost = cost;
    }
  }
  return best;
}

template <int BN>
static int launch_bn(const CUtensorMap& ta, const void* B, int64_t ldb, const CUtensorMap& tc, const CUtensorMap& tr,
                     const DevEpi& ep,
                     int64_t M, int64_t N, int64_t K, cudaStream_t st) {
  using Cf = Cfg<BN>;
  CUtensorMap tb;
  int rc = make_tmap_bf16_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK, BN);
  if (rc) return rc;
  static thread_local int attr_dev_mask = 0;  // per-thread, per-device: attribute set once
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    VLA_CUDA_TRY(cudaFuncSetAttribute(gemm_bf16_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      Cf::SMEM_BYTES));
    attr_dev_mask |= 1 << (dev & 31);
  }
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int sms = device_info().num_sms;
  const int grid = (int)(tiles < sms ? tiles : sms);
  prof_begin(st);
  launch_k(gemm_bf16_tc_kernel<BN>, dim3(grid), dim3(kThreads), Cf::SMEM_BYTES, st, ta, tb, tc, tr, ep, (int)M, (int)N,
           (int)K);
  {
    const double out_cols = ep.act == VLA_ACT_SWIGLU ? N / 2 : N;
    double bytes = 2.0 * ((double)M * K + (double)N * K + (double)M * out_cols);
    if (ep.residual) bytes += 2.0 * M * out_cols;
    if (ep.act == VLA_ACT_EULER) bytes += 8.0 * M * N;
    prof_end(st, VLA_KIND_GEMM, 2.0 * M * N * K, bytes, M, N, K, BN, 1);
  }
  return launch_status("gemm_bf16_tc");
}

// Skinny launch (M <= 128, gemm_skinny.cuh): ta is the two-dimensional A map
// with AR-row boxes; the k-slab maps of A and B are made here.
template <int BN, int AR, int KPS = kSkinnyKps>
static int launch_skinny(const CUtensorMap& ta, const void* A, int64_t lda, const void* B, int64_t ldb,
                         const CUtensorMap& tc, const CUtensorMap& tr, const DevEpi& ep, int64_t M, int64_t N, int64_t K,
                         cudaStream_t st) {
  using Cf = CfgK<BN, AR, KPS>;
  CUtensorMap tb, ta3, tb3;
  int rc = make_tmap_bf16_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK, BN);
  if (!rc) rc = make_tmap_bf16_kslab(&ta3, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, AR, KPS);
  if (!rc) rc = make_tmap_bf16_kslab(&tb3, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BN, KPS);
  if (rc) return rc;
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int sms = device_info().num_sms;
  const int grid = (int)(tiles < sms ? tiles : sms);
  // two MMA-issuing threads (DUAL) for 64-row copies at widths up to 128, one
  // tile per CTA and at least two units of k-blocks; VLA_GEMM_SKINNY_DUAL=0
  // turns it off (A/B)
  static const bool dual_on = [] {
    const char* v = getenv("VLA_GEMM_SKINNY_DUAL");
    return v == nullptr || atoi(v) != 0;
  }();
  const int64_t units = ((K + BK - 1) / BK + KPS - 1) / KPS;
  constexpr bool kDualShape = AR == kSkinnyRows && BN <= 128;
  const bool dual = kDualShape && dual_on && units >= 2 && tiles <= sms;
  auto kern = dual ? gemm_bf16_skinny_kernel<BN, AR, KPS, kDualShape> : gemm_bf16_skinny_kernel<BN, AR, KPS, false>;
  static thread_local int attr_dev_mask[2] = {0, 0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask[dual] & (1 << (dev & 31)))) {
    VLA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM_BYTES));
    attr_dev_mask[dual] |= 1 << (dev & 31);
  }
  prof_begin(st);
  launch_k(kern, dim3(grid), dim3(kThreads), Cf::SMEM_BYTES, st, ta, tb, ta3, tb3, tc, tr, ep, (int)M, (int)N, (int)K);
  {
    const double out_cols = ep.act == VLA_ACT_SWIGLU ? N / 2 : N;
    double bytes = 2.0 * ((double)M * K + (double)N * K + (double)M * out_cols);
    if (ep.residual) bytes += 2.0 * M * out_cols;
    if (ep.act == VLA_ACT_EULER) bytes += 8.0 * M * N;
    prof_end(st, VLA_KIND_GEMM, 2.0 * M * N * K, bytes, M, N, K, BN, 1);
  }
  return launch_status("gemm_bf16_skinny");
}

// One-CTA launches of more than one row tile whose tiles fit one wave, at tile
// widths up to 128 (three or more stages of two k-blocks), go through the unit
// kernel (measured: B = 8 chunk 685 -> 701 chunks/s; at B = 64, where the
// expert's 3200-row GEMMs take 256-wide tiles with two such stages, it lost
// 1.5-3 % and is not used).  VLA_GEMM_UNIT2=0 turns it off (A/B).
static bool use_unit2(int64_t M, int64_t N, int64_t K, int bn) {
  static const bool on = [] {
    const char* v = getenv("VLA_GEMM_UNIT2");
    return v == nullptr || atoi(v) != 0;
  }();
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
  return on && bn <= 128 && K / BK >= 2 && tiles <= device_info().num_sms;
}

// The skinny kernel serves one row tile (M <= 64 with 64-row copies at tile
// widths 32 / 64 / 128, M <= 128 with 128-row copies at 32 / 64, where two
// stages still fit) with at least one whole stage of k-blocks;
// VLA_GEMM_SKINNY=0 turns it off (A/B).
static bool use_skinny(int64_t M, int64_t K, int bn) {
  static const bool on = [] {
    const char* v = getenv("VLA_GEMM_SKINNY");
    return v == nullptr || atoi(v) != 0;
  }();
  if (!on || K / BK < kSkinnyKps) return false;
  if (M <= kSkinnyRows) return bn == 32 || bn == 64 || bn == 128;
  return M <= BM && (bn == 32 || bn == 64);
}

// Largest number of co-resident clusters of S split-K CTAs (kernel<BN>), cached.
template <int BN>
static int max_splitk_clusters(int S) {
  static int cached[64][kMaxSplit + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (cached[dev][S] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S * (device_info().num_sms / S));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = CfgS<BN>::smem_bytes(S - 1);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_bf16_splitk_kernel<BN>, &cfg) != cudaSuccess || n <= 0)
      n = device_info().num_sms / S;
    cached[dev][S] = n;
  }
  return cached[dev][S];
}

template <int BN>
static int launch_splitk(const CUtensorMap& ta, const void* B, int64_t ldb, const CUtensorMap& tc,
                         const CUtensorMap& tr, const DevEpi& ep, int64_t M, int64_t N, int64_t K, int S,
                         cudaStream_t st) {
  using Cf = CfgS<BN>;
  CUtensorMap tb;
  int rc = make_tmap_bf16_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK, BN);
  if (rc) return rc;
  const int smem = Cf::smem_bytes(S - 1);
  const int stages = Cf::stages_for(S - 1);
  VLA_CHECK_ARG(stages >= 2, "gemm split-K: %d partial slots leave no room for the stage ring", S - 1);
  static thread_local int attr_smem[32] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_smem[dev & 31] < smem) {
    VLA_CUDA_TRY(cudaFuncSetAttribute(gemm_bf16_splitk_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_smem[dev & 31] = smem;
  }
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int clusters = max_splitk_clusters<BN>(S);
  const int grid = S * (int)(tiles < clusters ? tiles : clusters);
  prof_begin(st);
  launch_k_cluster(gemm_bf16_splitk_kernel<BN>, S, dim3(grid), dim3(kThreads), smem, st, ta, tb, tc, tr, ep, (int)M,
                   (int)N, (int)K, S, stages);
  {
    const double out_cols = ep.act == VLA_ACT_SWIGLU ? N / 2 : N;
    double bytes = 2.0 * ((double)M * K + (double)N * K + (double)M * out_cols);
    if (ep.residual) bytes += 2.0 * M * out_cols;
    if (ep.act == VLA_ACT_EULER) bytes += 8.0 * M * N;
    prof_end(st, VLA_KIND_GEMM, 2.0 * M * N * K, bytes, M, N, K, BN, -S);
  }
  return launch_status("gemm_bf16_splitk");
}

// K split for a one-CTA tiling with few tiles: enough clusters of S CTAs to
// cover the SMs, each CTA keeping at least two k-blocks (0 = no split).
// Largest split whose partial slots leave room for a two-stage ring at width bn.
static int max_split(int bn) {
  auto fits = [&](int S) {
    switch (bn) {
      case 32: return CfgS<32>::stages_for(S - 1) >= 2;
      case 64: return CfgS<64>::stages_for(S - 1) >= 2;
      case 128: return CfgS<128>::stages_for(S - 1) >= 2;
      default: return false;
    }
  };
  int S = kMaxSplit;
  while (S >= 2 && !fits(S)) --S;
  return S;
}

static int choose_split(int64_t M, int64_t N, int64_t K, int bn, int num_sms) {
  if (bn != 32 && bn != 64 && bn != 128) return 0;
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
  const int64_t kb = (K + BK - 1) / BK;
  if (2 * tiles > num_sms || kb < 4) return 0;
  int64_t S = num_sms / tiles;
  if (S > max_split(bn)) S = max_split(bn);
  if (S > kb / 2) S = kb / 2;
  return S >= 2 ? (int)S : 0;
}

// Everything of a GEMM launch but the tile width: argument checks, the device
// epilogue description and the A / C / residual tensor maps.
struct GemmPlan {
  DevEpi ep;
  int act;
  CUtensorMap ta, tc, tr;
};

static int plan_gemm(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M, int64_t N,
                     int64_t K, const vla_epilogue* e, GemmPlan& plan) {
  VLA_CHECK_ARG(A && B && C, "gemm: null operand");
  VLA_CHECK_ARG(M >= 0 && N > 0 && K > 0, "gemm: bad shape M=%lld N=%lld K=%lld", (long long)M, (long long)N,
                (long long)K);
  VLA_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm: shape exceeds int32");
  VLA_CHECK_ARG(N % 16 == 0, "gemm: N=%lld must be a multiple of 16", (long long)N);
  VLA_CHECK_ARG(lda >= K && ldb >= K, "gemm: lda/ldb smaller than K");
  VLA_CHECK_ALIGN(lda % 8 == 0 && ldb % 8 == 0 && ldc % 8 == 0, "gemm: lda/ldb/ldc must be multiples of 8 elements");
  VLA_CHECK_ALIGN(aligned16(A) && aligned16(B) && aligned16(C), "gemm: A/B/C must be 16-byte aligned");
  if (M == 0) return VLA_OK;  // nothing to launch; the plan stays unfilled

  DevEpi& ep = plan.ep;
  ep = DevEpi{};
  ep.C = reinterpret_cast<bf16*>(C);
  ep.ldc = ldc;
  ep.alpha = 1.f;
  ep.M = (int)M;
  ep.N = (int)N;
  int& act = plan.act;
  act = VLA_ACT_NONE;
  if (e != nullptr) {
    act = e->act;
    ep.bias = reinterpret_cast<const bf16*>(e->bias);
    ep.residual = reinterpret_cast<const bf16*>(e->residual);
    ep.ldr = e->ldr;
    ep.res_row_mod = e->res_row_mod;
    ep.alpha = e->alpha == 0.f ? 1.f : e->alpha;
    ep.rope_cs = e->rope_cs;
    ep.rope_seq = e->rope_seq;
    ep.rope_ncols = e->rope_ncols;
    ep.out_grp = e->out_grp;
    ep.out_grp_stride = e->out_grp_stride;
    ep.euler_x = e->euler_x;
    ep.ldx = e->ldx;
    ep.euler_dt = e->euler_dt;
    ep.b_static = e->b_static != 0;
  }
  ep.act = act;
  VLA_CHECK_ARG(act >= VLA_ACT_NONE && act <= VLA_ACT_EULER, "gemm: unknown act %d", act);
  const int64_t out_cols = act == VLA_ACT_SWIGLU ? N / 2 : N;
  VLA_CHECK_ARG(ldc >= out_cols, "gemm: ldc=%lld < output columns %lld", (long long)ldc, (long long)out_cols);
  if (ep.residual) {
    VLA_CHECK_ARG(ep.ldr >= out_cols, "gemm: ldr smaller than output columns");
    VLA_CHECK_ALIGN(ep.ldr % 8 == 0 && aligned16(ep.residual), "gemm: residual must be 16-byte aligned, ldr %% 8 == 0");
  }
  if (ep.bias) VLA_CHECK_ALIGN(aligned16(ep.bias), "gemm: bias must be 16-byte aligned");
  if (act == VLA_ACT_SWIGLU) {
    VLA_CHECK_ARG(N % 32 == 0, "gemm: SwiGLU needs N %% 32 == 0");
    VLA_CHECK_ARG(ep.bias == nullptr, "gemm: SwiGLU epilogue takes no bias");
  }
  if (act == VLA_ACT_ROPE) {
    VLA_CHECK_ARG(ep.rope_cs && ep.rope_seq > 0, "gemm: RoPE needs a cos/sin table and rope_seq > 0");
    VLA_CHECK_ARG(ep.rope_ncols % 64 == 0 && ep.rope_ncols <= N, "gemm: rope_ncols must be a multiple of 64 <= N");
    VLA_CHECK_ARG(N % 64 == 0, "gemm: RoPE needs N %% 64 == 0");
  }
  if (act == VLA_ACT_EULER) {
    VLA_CHECK_ARG(ep.euler_x != nullptr && ep.ldx >= N, "gemm: Euler needs an fp32 state with ldx >= N");
    VLA_CHECK_ALIGN(aligned16(ep.euler_x) && ep.ldx % 4 == 0, "gemm: Euler state must be 16-byte aligned");
  }

  CUtensorMap& ta = plan.ta;
  int rc = make_tmap_bf16_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, BM);
  if (rc) return rc;
  // Output through shared memory + TMA stores for the plain / bias / GELU /
  // residual / SwiGLU / RoPE epilogues (row scatter and Euler store directly).
  // Box: 32 rows x 32 columns (64-byte swizzle), or 16 columns (32-byte
  // swizzle); out-of-range rows and columns are clipped.
  CUtensorMap& tc = plan.tc;
  memset(&tc, 0, sizeof(tc));
  ep.tma_c = (act == VLA_ACT_NONE || act == VLA_ACT_GELU_TANH || act == VLA_ACT_SWIGLU ||
              (act == VLA_ACT_ROPE && ep.residual == nullptr)) &&
             ep.out_grp == 0;
  if (ep.tma_c) {
    // 16-column boxes for SwiGLU's halved output and for RoPE's half-head segments
    const bool sw = act == VLA_ACT_SWIGLU || act == VLA_ACT_ROPE;
    rc = make_tmap_bf16_2d(&tc, C, (uint64_t)out_cols, (uint64_t)M, (uint64_t)ldc, sw ? 16u : 32u, 32u,
                           sw ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
  }
  // The residual through the same staging buffers (32 x 32 chunks, 64-byte
  // swizzle) when each 32-row block maps to 32 consecutive residual rows.
  CUtensorMap& tr = plan.tr;
  memset(&tr, 0, sizeof(tr));
  ep.tma_r = ep.tma_c && ep.residual != nullptr && act != VLA_ACT_SWIGLU &&
             (ep.res_row_mod == 0 || ep.res_row_mod % 32 == 0);
  if (ep.tma_r) {
    const uint64_t rows = ep.res_row_mod > 0 ? (uint64_t)ep.res_row_mod : (uint64_t)M;
    rc = make_tmap_bf16_2d(&tr, ep.residual, (uint64_t)out_cols, rows, (uint64_t)ep.ldr, 32u, 32u,
                           CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
  }
  return VLA_OK;
}

static int run(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M, int64_t N,
               int64_t K, const vla_epilogue* e, cudaStream_t st, int force_bn = 0, int force_ctas = 0,
               int force_split = -1) {
  GemmPlan plan;
  int rc = plan_gemm(A, lda, B, ldb, C, ldc, M, N, K, e, plan);
  if (rc) return rc;
  if (M == 0) return VLA_OK;
  const DevEpi& ep = plan.ep;
  const int act = plan.act;
  const CUtensorMap& ta = plan.ta;
  const CUtensorMap& tc = plan.tc;
  const CUtensorMap& tr = plan.tr;
  int bn = force_bn ? force_bn : choose_bn(M, N, act, device_info().num_sms);
  // VLA_GEMM_CTAS=1|2 overrides the automatic one-CTA / pair choice (A/B measurement)
  static const int env_ctas = [] {
    const char* v = getenv("VLA_GEMM_CTAS");
    return v ? atoi(v) : 0;
  }();
  const int ctas = force_ctas                          ? force_ctas
                   : (env_ctas == 1 || env_ctas == 2) ? env_ctas
                                                      : choose_ctas(M, bn);
  if (ctas == 1) {
    // explicit splits come from vla_gemm_bf16_split
    static const int env_split = [] {
      const char* v = getenv("VLA_GEMM_SPLITK");
      return v ? atoi(v) : -1;
    }();
    // The automatic choice does not split: inside a CUDA graph at one observation
    // the clustered launch measured slower than the plain one on every expert
    // shape (M = 50: 720 x 2048 12.0 -> 15.5 us, 720 x 960 7.2 -> 14.2 us,
    // 1600 x 720 7.5 -> 14.6 us; the whole B = 1 chunk 10.0 -> 13.4 ms), the
    // per-launch cost of these tiny GEMMs being fixed overhead, not the K loop.
    // VLA_GEMM_SPLITK=1 enables choose_split for measurements.
    int split = force_split >= 0 ? force_split
                : env_split == 1 ? choose_split(M, N, K, bn, device_info().num_sms)
                                 : 0;
    if (split > kMaxSplit || (split >= 2 && (K + BK - 1) / BK < split))
      return set_error(VLA_E_INVALID, "gemm: split %d needs 2..%d and at most one part per k-block", split, kMaxSplit);
    if (split >= 2) {
      switch (bn) {
        case 32: return launch_splitk<32>(ta, B, ldb, tc, tr, ep, M, N, K, split, st);
        case 64: return launch_splitk<64>(ta, B, ldb, tc, tr, ep, M, N, K, split, st);
        case 128: return launch_splitk<128>(ta, B, ldb, tc, tr, ep, M, N, K, split, st);
        default: return set_error(VLA_E_UNSUPPORTED, "gemm: split-K tile width %d not built", bn);
      }
    }
  }
  if (ctas == 2 && !force_bn) bn = choose_bn_pair(M, N, act, device_info().num_sms);
  if (ctas == 2 && bn < 64) return run(A, lda, B, ldb, C, ldc, M, N, K, e, st, 64, 2);
  if (ctas == 2) {
    switch (bn) {
      case 256: return launch_bn2<256>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 224: return launch_bn2<224>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 192: return launch_bn2<192>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 160: return launch_bn2<160>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 128: return launch_bn2<128>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 96: return launch_bn2<96>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 64: return launch_bn2<64>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      default: return set_error(VLA_E_UNSUPPORTED, "gemm: pair tile width %d not built", bn);
    }
  }
  if (M <= 64) {
    // one M-tile of at most 64 real rows: copy 64-row A boxes (half the A bytes
    // of every k-block, which dominate a skinny GEMM's loads)
    rc = make_tmap_bf16_2d(&plan.ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, 64);
    if (rc) return rc;
    plan.ep.a_rows = 64;
    if (use_skinny(M, K, bn)) {
      switch (bn) {
        case 32: return launch_skinny<32, 64>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
        case 64: return launch_skinny<64, 64>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
        case 128: return launch_skinny<128, 64>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
        default: break;
      }
    }
  } else if (use_skinny(M, K, bn)) {
    if (bn == 32) return launch_skinny<32, 128>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
    if (bn == 64) return launch_skinny<64, 128>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
  } else if (use_unit2(M, N, K, bn)) {
    switch (bn) {
      case 256: return launch_skinny<256, 128, 2>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 224: return launch_skinny<224, 128, 2>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 192: return launch_skinny<192, 128, 2>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 160: return launch_skinny<160, 128, 2>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 128: return launch_skinny<128, 128, 2>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 96: return launch_skinny<96, 128, 2>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 64: return launch_skinny<64, 128, 2>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      case 32: return launch_skinny<32, 128, 2>(ta, A, lda, B, ldb, tc, tr, ep, M, N, K, st);
      default: break;
    }
  }
  switch (bn) {
    case 256: return launch_bn<256>(ta, B, ldb, tc, tr, ep, M, N, K, st);
    case 224: return launch_bn<224>(ta, B, ldb, tc, tr, ep, M, N, K, st);
    case 192: return launch_bn<192>(ta, B, ldb, tc, tr, ep, M, N, K, st);
    case 160: return launch_bn<160>(ta, B, ldb, tc, tr, ep, M, N, K, st);
    case 128: return launch_bn<128>(ta, B, ldb, tc, tr, ep, M, N, K, st);
    case 96: return launch_bn<96>(ta, B, ldb, tc, tr, ep, M, N, K, st);
    case 64: return launch_bn<64>(ta, B, ldb, tc, tr, ep, M, N, K, st);
    case 32: return launch_bn<32>(ta, B, ldb, tc, tr, ep, M, N, K, st);
    default: return set_error(VLA_E_UNSUPPORTED, "gemm: tile width %d not built", bn);
  }
}

}  // namespace gemm
}  // namespace vla
