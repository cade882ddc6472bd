// Block builders: compose the GEMM / norm / attention kernels into the
// reference's transformer layers.  All launches go to one stream; scratch
// lives in a caller-provided workspace (no allocation here).
#pragma once
#include "attention.cuh"
#include "attention_pipe.cuh"
#include "attention_short.cuh"
#include "attention_tc.cuh"
#include "elementwise.cuh"
#include "gemm_host.cuh"
#include "layer_fused.cuh"
#include "norm.cuh"

namespace vla {
namespace blocks {

static inline size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

static inline int grid_for(long long work, int threads) {
  const int sms = device_info().num_sms;
  long long blocks = (work + threads - 1) / threads;
  const long long cap = (long long)sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

// static_params: g / b are weights that no earlier kernel of the stream writes
// (the layers' own norms), fetched before the launch-overlap wait.
static int rownorm(int mode, const void* x, int64_t ldx, const void* g, const void* b, void* y, int64_t ldy, int64_t M,
                   int64_t N, float eps, cudaStream_t st, bool static_params = false) {
  VLA_CHECK_ARG(x && g && y && (mode == 0 || b), "norm: null pointer");
  VLA_CHECK_ARG(M >= 0 && N > 0 && N % 8 == 0, "norm: N=%lld must be a positive multiple of 8", (long long)N);
  VLA_CHECK_ALIGN(ldx % 8 == 0 && ldy % 8 == 0 && aligned16(x) && aligned16(y) && aligned16(g) && (!b || aligned16(b)),
                  "norm: 16-byte alignment");
  if (M == 0) return VLA_OK;
  // a resident grid (8 CTAs of 8 warps per SM) walking the rows: 3-5 % faster
  // than one short-lived CTA per 8 rows (SigLIP LayerNorm 151 -> 144 us)
  const int64_t blocks = (M + norm::kWarps - 1) / norm::kWarps;
  const int64_t cap = 8ll * device_info().num_sms;
  const int grid = (int)(blocks < cap ? blocks : cap);
  const bf16* bb = mode == 0 ? nullptr : (const bf16*)b;
  // early weight loads only for grids of at most one row per warp: the extra
  // registers cost residency on the big row counts (B = 256 step -1.3 %), while
  // one observation's norms gain the load latency (B = 1 chunk +3.9 %)
  static_params = static_params && blocks <= cap;
  auto kern = mode == 0 ? (static_params ? norm::rownorm_kernel<0, true> : norm::rownorm_kernel<0, false>)
                        : (static_params ? norm::rownorm_kernel<1, true> : norm::rownorm_kernel<1, false>);
  prof_begin(st);
  launch_k(kern, dim3(grid), dim3(norm::kWarps * 32), 0, st, (const bf16*)x, ldx, (const bf16*)g, bb, (bf16*)y, ldy,
           (int)M, (int)N, eps);
  prof_end(st, VLA_KIND_NORM, 0.0, 4.0 * (double)M * N);
  return launch_status("rownorm");
}

// tcgen05 attention: persistent CTAs over (query tile, head, sequence) items
static int attention_tc(const attn::Params& p, int batch, cudaStream_t st) {
  VLA_CHECK_ARG(!p.causal, "attention (tcgen05): causal masking is not supported");
  VLA_CHECK_ARG(p.q_batch % p.q_row == 0 && p.k_batch % p.k_row == 0 && p.v_batch % p.v_row == 0 &&
                    p.k_batch / p.k_row == p.v_batch / p.v_row,
                "attention (tcgen05): sequence strides must be whole rows, equal for K and V");
  const long long q_rows = p.q_batch / p.q_row, k_rows = p.k_batch / p.k_row;
  const long long total_q = (batch - 1) * q_rows + p.Lq, total_k = (batch - 1) * k_rows + p.Lk;
  VLA_CHECK_ARG(total_q < (1ll << 31) && total_k < (1ll << 31), "attention (tcgen05): too many rows");
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_bf16_2d(&tq, p.q, (uint64_t)p.Hq * 64, (uint64_t)total_q, (uint64_t)p.q_row, 64, 128);
  if (rc) return rc;
  rc = make_tmap_bf16_2d(&tk, p.k, (uint64_t)p.Hkv * 64, (uint64_t)(total_k > 0 ? total_k : 1), (uint64_t)p.k_row,
                         64, 128);
  if (rc) return rc;
  rc = make_tmap_bf16_2d(&tv, p.v, (uint64_t)p.Hkv * 64, (uint64_t)(total_k > 0 ? total_k : 1), (uint64_t)p.v_row,
                         64, 128);
  if (rc) return rc;
  attn_tc::Params tp{};
  tp.Lq = p.Lq;
  tp.Lk = p.Lk;
  tp.Hq = p.Hq;
  tp.Hkv = p.Hkv;
  tp.batch = batch;
  tp.n_qt = (p.Lq + attn_tc::ITEM_ROWS - 1) / attn_tc::ITEM_ROWS;
  tp.q_rows_per_seq = q_rows;
  tp.k_rows_per_seq = k_rows;
  tp.o = p.o;
  tp.o_row = p.o_row;
  tp.o_batch = p.o_batch;
  tp.kv_len = p.kv_len;
  tp.scale_log2 = p.scale_log2;
  const int smem = (int)sizeof(attn_tc::Smem) + 1024;
  // key pairs (of every 8) whose exponentials run on the FMA pipe:
  // VLA_ATTN_POLY8 = 0, 2 or 3
  static const int poly8 = [] {
    const char* v = getenv("VLA_ATTN_POLY8");
    const int n = v != nullptr ? atoi(v) : 2;
    return n == 0 || n == 3 ? n : 2;
  }();
  // P.V products issued by warp 3 for both groups (default) or by each
  // group's S issuer (VLA_ATTN_PV_WARP=0)
  static const bool pv_warp = [] {
    const char* v = getenv("VLA_ATTN_PV_WARP");
    return !(v != nullptr && atoi(v) == 0);
  }();
  auto kern = pv_warp ? (poly8 == 0   ? attn_tc::flash_attn_tc_kernel<0, true>
                         : poly8 == 3 ? attn_tc::flash_attn_tc_kernel<3, true>
                                      : attn_tc::flash_attn_tc_kernel<2, true>)
                      : (poly8 == 0   ? attn_tc::flash_attn_tc_kernel<0, false>
                         : poly8 == 3 ? attn_tc::flash_attn_tc_kernel<3, false>
                                      : attn_tc::flash_attn_tc_kernel<2, false>);
  static thread_local int attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    VLA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cudaFuncAttributes fa{};
    VLA_CUDA_TRY(cudaFuncGetAttributes(&fa, kern));
    // the in-kernel register split (setmaxnreg) hands out exactly the launch's
    // registers: it is only sound at the register count it was sized for
    if (fa.numRegs != attn_tc::kLaunchRegs || fa.maxThreadsPerBlock < attn_tc::kThreads)
      return set_error(VLA_E_CUDA,
                       "flash_attn_tc: built with %d registers/thread (%d threads per block); the register split "
                       "needs exactly %d for %d threads",
                       fa.numRegs, fa.maxThreadsPerBlock, attn_tc::kLaunchRegs, attn_tc::kThreads);
    attr_dev_mask |= 1 << (dev & 31);
  }
  const long long items = (long long)tp.n_qt * p.Hq * batch;
  VLA_CHECK_ARG(items < (1ll << 31), "attention (tcgen05): too many work items");
  const int sms = device_info().num_sms;
  const int grid = (int)(items < sms ? items : sms);
  prof_begin(st);
  launch_k(kern, dim3(grid), dim3(attn_tc::kThreads), smem, st, tq, tk, tv, tp);
  prof_end(st, VLA_KIND_ATTENTION, 4.0 * batch * p.Hq * (double)p.Lq * p.Lk * 64,
           2.0 * batch * ((double)p.Lq * p.Hq * 64 * 2 + (double)p.Lk * p.Hkv * 64 * 2));
  return launch_status("flash_attn_tc");
}

// short-sequence tcgen05 attention: persistent CTAs over (sequence, kv head,
// 128 stacked query rows) items, 4 per SM
static int attention_short(const attn::Params& p, int batch, cudaStream_t st) {
  VLA_CHECK_ARG(p.Lk <= 128, "attention (tcgen05 short): Lk=%d exceeds 128", p.Lk);
  attn_sq::Params sp{};
  sp.q = p.q, sp.k = p.k, sp.v = p.v, sp.o = p.o;
  sp.q_row = p.q_row, sp.k_row = p.k_row, sp.v_row = p.v_row, sp.o_row = p.o_row;
  sp.q_batch = p.q_batch, sp.k_batch = p.k_batch, sp.v_batch = p.v_batch, sp.o_batch = p.o_batch;
  sp.Lq = p.Lq, sp.Lk = p.Lk, sp.Hq = p.Hq, sp.Hkv = p.Hkv, sp.G = p.Hq / p.Hkv;
  sp.n_mt = (int)(((long long)sp.G * p.Lq + attn_sq::MT - 1) / attn_sq::MT);
  sp.batch = batch, sp.causal = p.causal, sp.kv_len = p.kv_len, sp.scale_log2 = p.scale_log2;
  const long long items = (long long)batch * p.Hkv * sp.n_mt;
  const int smem = (int)sizeof(attn_sq::Smem) + 1024;
  const bool n64 = p.Lk <= 64;
  auto kern = n64 ? attn_sq::attn_short_kernel<64> : attn_sq::attn_short_kernel<128>;
  static thread_local int attr_dev_mask[2] = {0, 0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask[n64] & (1 << (dev & 31)))) {
    VLA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_dev_mask[n64] |= 1 << (dev & 31);
  }
  VLA_CHECK_ARG(items < (1ll << 31), "attention (tcgen05 short): too many work items");
  const long long cap = 4ll * device_info().num_sms;
  const int grid = (int)(items < cap ? items : cap);
  prof_begin(st);
  launch_k(kern, dim3(grid), dim3(attn_sq::kThreads), smem, st, sp);
  prof_end(st, VLA_KIND_ATTENTION, 4.0 * batch * p.Hq * (double)p.Lq * p.Lk * 64,
           2.0 * batch * ((double)p.Lq * p.Hq * 64 * 2 + (double)p.Lk * p.Hkv * 64 * 2));
  return launch_status("attn_short");
}

// 4-D bf16 tensor map of one attention operand viewed as (64 head elements,
// heads, rows, sequences) with strides (128 B, row stride, sequence stride);
// box = 64 x box_heads x box_rows x 1, 128-byte swizzle, zero fill outside.
static int make_tmap_heads_4d(CUtensorMap* m, const void* ptr, int heads, int rows, int batch, long long row_stride,
                              long long batch_stride, int box_heads, int box_rows) {
  auto enc = tmap_encoder();
  if (enc == nullptr) return set_error(VLA_E_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  // a single sequence may come with a zero sequence stride; any legal stride
  // serves, the coordinate is always 0
  const long long bstride = batch > 1 ? batch_stride : row_stride * rows;
  cuuint64_t dims[4] = {64, (cuuint64_t)heads, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[3] = {128, (cuuint64_t)row_stride * 2, (cuuint64_t)bstride * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_heads, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(VLA_E_CUDA, "cuTensorMapEncodeTiled (4-D) failed (%d): heads=%d rows=%d batch=%d ld=%lld bs=%lld",
                     (int)r, heads, rows, batch, row_stride, batch_stride);
  return VLA_OK;
}

// Whether the pipelined short-sequence kernel takes this problem.
static bool pipe_fits(const attn::Params& p, int batch) {
  const int G = p.Hq / p.Hkv;
  return p.Lk >= 1 && p.Lk <= 128 && p.Lq <= 256 && G <= 256 &&
         (long long)G * p.Lq <= attn_pipe::kMaxTiles * attn_pipe::MT &&
         (batch == 1 || (p.q_batch > 0 && p.k_batch > 0 && p.v_batch > 0 && p.o_batch > 0)) &&
         (long long)batch * p.Hkv < (1ll << 31);
}

// pipelined short-sequence tcgen05 attention: one persistent warp-specialised
// CTA per SM over (sequence, kv head) items, TMA in and out
static int attention_pipe(const attn::Params& p, int batch, cudaStream_t st) {
  VLA_CHECK_ARG(pipe_fits(p, batch), "attention (pipelined tcgen05): Lk=%d Lq=%d G=%d outside the kernel's range",
                p.Lk, p.Lq, p.Hq / p.Hkv);
  const int G = p.Hq / p.Hkv;
  const int NK = p.Lk <= 64 ? 64 : 128;
  attn_pipe::Params pp{};
  pp.Lq = p.Lq, pp.Lk = p.Lk, pp.G = G, pp.Hkv = p.Hkv, pp.batch = batch, pp.causal = p.causal;
  pp.T = (G * p.Lq + attn_pipe::MT - 1) / attn_pipe::MT;
  pp.q_tx = (uint32_t)(G * p.Lq * 128);
  pp.q_region = (uint32_t)((G * p.Lq * 128 + 1023) / 1024 * 1024);
  pp.stage_bytes = pp.q_region + 2u * NK * 128u;
  if (pp.stage_bytes < (uint32_t)(pp.T * attn_pipe::TILE_BYTES)) pp.stage_bytes = (uint32_t)(pp.T * attn_pipe::TILE_BYTES);
  pp.kv_len = p.kv_len;
  pp.scale_log2 = p.scale_log2;
  const int smem_cap = device_info().max_smem_optin > 0 ? device_info().max_smem_optin : 232448;
  const int avail = smem_cap - 2048;
  pp.stages = avail / (int)pp.stage_bytes;
  if (pp.stages > attn_pipe::kMaxStages) pp.stages = attn_pipe::kMaxStages;
  VLA_CHECK_ARG(pp.stages >= 1, "attention (pipelined tcgen05): stage of %u bytes does not fit", pp.stage_bytes);
  const int smem = 2048 + pp.stages * (int)pp.stage_bytes;
  CUtensorMap tq, tk, tv, to;
  int rc = make_tmap_heads_4d(&tq, p.q, p.Hq, p.Lq, batch, p.q_row, p.q_batch, G, p.Lq);
  if (!rc) rc = make_tmap_heads_4d(&tk, p.k, p.Hkv, p.Lk, batch, p.k_row, p.k_batch, 1, NK);
  if (!rc) rc = make_tmap_heads_4d(&tv, p.v, p.Hkv, p.Lk, batch, p.v_row, p.v_batch, 1, NK);
  if (!rc) rc = make_tmap_heads_4d(&to, p.o, p.Hq, p.Lq, batch, p.o_row, p.o_batch, G, p.Lq);
  if (rc) return rc;
  // softmax warpgroups: 4 (two of them share the full M-tiles of a
  // 150-row item) unless VLA_ATTN_PIPE_GROUPS=2
  static const int groups = [] {
    const char* v = getenv("VLA_ATTN_PIPE_GROUPS");
    return (v != nullptr && atoi(v) == 2) ? 2 : 4;
  }();
  auto kern = NK == 64 ? (groups == 4 ? attn_pipe::attn_pipe_kernel<64, 4> : attn_pipe::attn_pipe_kernel<64, 2>)
                       : (groups == 4 ? attn_pipe::attn_pipe_kernel<128, 4> : attn_pipe::attn_pipe_kernel<128, 2>);
  static thread_local int attr_smem[2][2][32] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int& cur = attr_smem[groups == 4][NK == 64][dev & 31];
  if (cur < smem) {
    VLA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cur = smem;
  }
  const long long items = (long long)batch * p.Hkv;
  const int sms = device_info().num_sms;
  const int grid = (int)(items < sms ? items : sms);
  prof_begin(st);
  launch_k(kern, dim3(grid), dim3(attn_pipe::threads_for(groups)), smem, st, tq, tk, tv, to, pp);
  prof_end(st, VLA_KIND_ATTENTION, 4.0 * batch * p.Hq * (double)p.Lq * p.Lk * 64,
           2.0 * batch * ((double)p.Lq * p.Hq * 64 * 2 + (double)p.Lk * p.Hkv * 64 * 2));
  return launch_status("attn_pipe");
}

static int attention(const attn::Params& p, int batch, cudaStream_t st, int impl = VLA_ATTN_AUTO) {
  VLA_CHECK_ARG(p.q && p.k && p.v && p.o, "attention: null pointer");
  VLA_CHECK_ARG(batch >= 0 && p.Lq >= 0 && p.Lk >= 0 && p.Hq > 0 && p.Hkv > 0 && p.Hq % p.Hkv == 0,
                "attention: bad shape");
  VLA_CHECK_ARG(p.q_row > 0 && p.k_row > 0 && p.v_row > 0 && p.o_row > 0, "attention: row strides must be positive");
  VLA_CHECK_ALIGN(aligned16(p.q) && aligned16(p.k) && aligned16(p.v) && aligned16(p.o) && p.q_row % 8 == 0 &&
                      p.k_row % 8 == 0 && p.v_row % 8 == 0 && p.o_row % 8 == 0 && p.q_batch % 8 == 0 &&
                      p.k_batch % 8 == 0 && p.v_batch % 8 == 0 && p.o_batch % 8 == 0,
                  "attention: 16-byte alignment of pointers and strides");
  if (batch == 0 || p.Lq == 0) return VLA_OK;
  if (impl == VLA_ATTN_TCGEN05 || (impl == VLA_ATTN_AUTO && !p.causal && p.Lk >= 256 &&
                                   p.q_batch % p.q_row == 0 && p.k_batch % p.k_row == 0 &&
                                   p.v_batch % p.v_row == 0 && p.k_batch / p.k_row == p.v_batch / p.v_row))
    return attention_tc(p, batch, st);
  // short sequences: the tcgen05 kernel stacks the query heads of a kv head into
  // 128-row tiles, the mma.sync kernel pads each head to 64-row tiles; take the
  // tcgen05 kernel unless its padding is larger (text prefix 3 x 113 rows: 88 %
  // either way, tcgen05 13 % faster; expert 3 x 50 rows: 59 % vs 78 %, mma.sync
  // 5-10 % faster)
  if (impl == VLA_ATTN_TCGEN05_SHORT) return attention_short(p, batch, st);
  // short sequences (text prefix, action expert): the pipelined kernel, 30-45 %
  // faster than the one-chain-per-CTA kernels on all three shapes
  // With few items (batch x kv heads at most half the SMs: one or a few
  // observations) the per-item chain (copy, S, softmax, P.V, store) of the
  // pipelined kernel is the launch's latency, and the mma.sync kernel, whose CTAs
  // each take one 64-query tile of one head, finishes sooner (graph-timed, 15 / 5
  // heads: B = 1 expert self 5.0 -> 2.8 us, cross 6.1 -> 3.7, text 8.6 -> 4.1;
  // B = 8 5.2 -> 4.3, 6.3 -> 6.2, 8.9 -> 7.5).
  const bool few_items = (long long)batch * p.Hkv * 2 <= device_info().num_sms;
  if (impl == VLA_ATTN_TCGEN05_PIPE || (impl == VLA_ATTN_AUTO && !few_items && pipe_fits(p, batch)))
    return attention_pipe(p, batch, st);
  if (impl == VLA_ATTN_AUTO && !few_items && p.Lk <= 128) {
    const long long g_rows = (long long)(p.Hq / p.Hkv) * p.Lq;
    const long long pad_short = ((g_rows + 127) / 128) * 128;
    const long long pad_mma = (long long)(p.Hq / p.Hkv) * (((long long)p.Lq + 63) / 64) * 64;
    if (pad_short <= pad_mma) return attention_short(p, batch, st);
  }
  dim3 grid((p.Lq + attn::BQ - 1) / attn::BQ, p.Hq, batch);
  prof_begin(st);
  launch_k(attn::flash_attn_kernel, dim3(grid), dim3(attn::kThreads), 0, st, p);
  {
    const double lk = (double)p.Lk;
    const double flops = 4.0 * batch * p.Hq * (double)p.Lq * lk * attn::HD;
    const double bytes = 2.0 * batch * ((double)p.Lq * p.Hq * attn::HD * 2 + lk * p.Hkv * attn::HD * 2);
    prof_end(st, VLA_KIND_ATTENTION, flops, bytes);
  }
  return launch_status("flash_attn");
}

// ----------------------------------------------------------------------------
// Llama-style layer (text decoder block / action-expert block)
// ----------------------------------------------------------------------------
struct LlamaWs {
  bf16 *h, *qkv, *attn, *mlp;
  unsigned int* counter;
};

// Layer calls take rows = batch * seq below 2^31 (the GEMM's M limit); checking
// it before any size arithmetic keeps the workspace products far from int64
// overflow (rows * width * 2 < 2^31 * 2^32).
static constexpr int64_t kMaxLayerRows = (1ll << 31) - 1;

static size_t llama_ws_bytes(const vla_llama_layer* w, int64_t rows, bool need_qkv) {
  if (rows < 0 || rows > kMaxLayerRows || w->hidden < 0 || w->ffn < 0 || w->heads < 0 || w->kv_heads < 0)
    return SIZE_MAX;
  const int64_t q = (int64_t)w->heads * w->head_dim, kv = (int64_t)w->kv_heads * w->head_dim;
  size_t s = align_up(rows * w->hidden * 2) + align_up(rows * q * 2) + align_up(rows * w->ffn * 2);
  if (need_qkv) s += align_up(rows * (q + 2 * kv) * 2);
  return s + 256;  // the fused layer kernel's grid-barrier counter
}

static LlamaWs carve(const vla_llama_layer* w, int64_t rows, void* ws, bool need_qkv) {
  const int64_t q = (int64_t)w->heads * w->head_dim;
  uint8_t* p = (uint8_t*)ws;
  LlamaWs r{};
  r.h = (bf16*)p;
  p += align_up(rows * w->hidden * 2);
  r.attn = (bf16*)p;
  p += align_up(rows * q * 2);
  r.mlp = (bf16*)p;
  p += align_up(rows * w->ffn * 2);
  if (need_qkv) {
    r.qkv = (bf16*)p;
    p += align_up(rows * (q + 2 * (int64_t)w->kv_heads * w->head_dim) * 2);
  }
  r.counter = (unsigned int*)p;
  return r;
}

static int check_llama(const vla_llama_layer* w) {
  VLA_CHECK_ARG(w != nullptr, "llama layer: null weights");
  VLA_CHECK_ARG(w->norm1 && w->w_qkv && w->w_o && w->norm2 && w->w_gu && w->w_down, "llama layer: null weight");
  VLA_CHECK_ARG(w->head_dim == 64, "llama layer: head_dim must be 64");
  VLA_CHECK_ARG(w->hidden % 16 == 0 && w->ffn % 16 == 0 && w->heads % w->kv_heads == 0,
                "llama layer: hidden/ffn must be multiples of 16");
  return VLA_OK;
}

// MLP half shared by self and cross layers: x += down(silu(gate(rms(x))) * up(rms(x)))
static int llama_mlp(const vla_llama_layer* w, bf16* x, int64_t rows, const LlamaWs& ws, cudaStream_t st) {
  const int64_t H = w->hidden, F = w->ffn;
  int rc = rownorm(0, x, H, w->norm2, nullptr, ws.h, H, rows, H, w->eps, st, true);
  if (rc) return rc;
  vla_epilogue e{};
  e.b_static = 1;
  e.act = VLA_ACT_SWIGLU;
  rc = gemm::run(ws.h, H, w->w_gu, H, ws.mlp, F, rows, 2 * F, H, &e, st);
  if (rc) return rc;
  vla_epilogue r{};
  r.b_static = 1;
  r.residual = x;
  r.ldr = H;
  return gemm::run(ws.mlp, F, w->w_down, F, x, H, rows, H, F, &r, st);
}

// The whole layer as one cooperative launch (layer_fused.cuh) for small row
// counts.  Off by default: at one observation it measured slower than the
// seven launches it replaces (expert layer ~66 vs ~50 us in the graph; B = 1
// chunk 10.4 vs 8.0 ms for the expert), the phases' own latency, not the
// launches, being the cost.
static constexpr int64_t kFusedLayerRows = 512;

static std::atomic<int> g_fused_layers{0};  // vla_set_fused_layers()

static bool use_fused_layer(const vla_llama_layer* w, int64_t rows, int kv_seq) {
  return g_fused_layers.load(std::memory_order_relaxed) != 0 && rows <= kFusedLayerRows && kv_seq >= 1 && kv_seq <= 128 && w->hidden <= 1024 &&
         w->hidden % 8 == 0 && w->heads % w->kv_heads == 0;
}

static int llama_fused(const vla_llama_layer* w, bf16* x, int batch, int seq, const float* rope_cs, bf16* qkv,
                       const bf16* k, const bf16* v, int64_t ldkv, int kv_seq, const int* kv_len, const LlamaWs& b,
                       bool cross, cudaStream_t st) {
  const int64_t rows = (int64_t)batch * seq, H = w->hidden, F = w->ffn;
  const int64_t Q = (int64_t)w->heads * 64, KV = (int64_t)w->kv_heads * 64;
  const int64_t NQ = cross ? Q : Q + 2 * KV;
  lfused::Params P;
  memset(&P, 0, sizeof(P));
  gemm::GemmPlan pq, po, pg, pd;
  vla_epilogue e{};
  e.b_static = 1;
  e.act = VLA_ACT_ROPE;
  e.rope_cs = rope_cs;
  e.rope_seq = seq;
  e.rope_ncols = (int)(cross ? Q : Q + KV);
  int rc = gemm::plan_gemm(b.h, H, w->w_qkv, H, qkv, NQ, rows, NQ, H, &e, pq);
  vla_epilogue r{};
  r.b_static = 1;
  r.residual = x;
  r.ldr = H;
  if (!rc) rc = gemm::plan_gemm(b.attn, Q, w->w_o, Q, x, H, rows, H, Q, &r, po);
  vla_epilogue g{};
  g.b_static = 1;
  g.act = VLA_ACT_SWIGLU;
  if (!rc) rc = gemm::plan_gemm(b.h, H, w->w_gu, H, b.mlp, F, rows, 2 * F, H, &g, pg);
  if (!rc) rc = gemm::plan_gemm(b.mlp, F, w->w_down, F, x, H, rows, H, F, &r, pd);
  if (!rc) rc = make_tmap_bf16_2d(&P.b_qkv, w->w_qkv, (uint64_t)H, (uint64_t)NQ, (uint64_t)H, gemm::BK, 64);
  if (!rc) rc = make_tmap_bf16_2d(&P.b_o, w->w_o, (uint64_t)Q, (uint64_t)H, (uint64_t)Q, gemm::BK, 32);
  if (!rc) rc = make_tmap_bf16_2d(&P.b_gu, w->w_gu, (uint64_t)H, (uint64_t)(2 * F), (uint64_t)H, gemm::BK, 32);
  if (!rc) rc = make_tmap_bf16_2d(&P.b_down, w->w_down, (uint64_t)F, (uint64_t)H, (uint64_t)F, gemm::BK, 32);
  if (rc) return rc;
  P.a_h = pq.ta;
  P.a_attn = po.ta;
  P.a_mlp = pd.ta;
  P.c_qkv = pq.tc;
  P.c_x = po.tc;
  P.r_x = po.tr;
  P.c_mlp = pg.tc;
  P.g_qkv = {pq.ep, (int)rows, (int)NQ, (int)H};
  P.g_o = {po.ep, (int)rows, (int)H, (int)Q};
  P.g_gu = {pg.ep, (int)rows, (int)(2 * F), (int)H};
  P.g_down = {pd.ep, (int)rows, (int)H, (int)F};
  P.norm1 = (const bf16*)w->norm1;
  P.norm2 = (const bf16*)w->norm2;
  P.x = x;
  P.h = b.h;
  P.rows = (int)rows;
  P.H = (int)H;
  P.eps = w->eps;
  attn_sq::Params& a = P.att;
  a.q = qkv;
  a.k = cross ? k : qkv + Q;
  a.v = cross ? v : qkv + Q + KV;
  a.o = b.attn;
  a.q_row = NQ;
  a.q_batch = (long long)seq * NQ;
  a.k_row = a.v_row = cross ? ldkv : NQ;
  a.k_batch = a.v_batch = cross ? (long long)kv_seq * ldkv : (long long)seq * NQ;
  a.o_row = Q;
  a.o_batch = (long long)seq * Q;
  a.Lq = seq;
  a.Lk = kv_seq;
  a.Hq = w->heads;
  a.Hkv = w->kv_heads;
  a.G = w->heads / w->kv_heads;
  a.n_mt = (a.G * seq + attn_sq::MT - 1) / attn_sq::MT;
  a.batch = batch;
  a.causal = cross ? 0 : 1;
  a.kv_len = cross ? kv_len : nullptr;
  a.scale_log2 = 0.125f * 1.4426950408889634f;
  P.barrier = b.counter;
  VLA_CUDA_TRY(cudaMemsetAsync(b.counter, 0, sizeof(unsigned int), st));
  auto kern = kv_seq <= 64 ? lfused::llama_layer_fused_kernel<64> : lfused::llama_layer_fused_kernel<128>;
  static thread_local int attr_dev_mask[2] = {0, 0};
  const int which = kv_seq <= 64 ? 0 : 1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask[which] & (1 << (dev & 31)))) {
    VLA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lfused::SMEM_BYTES));
    int per_sm = 0;
    VLA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, gemm::kThreads, lfused::SMEM_BYTES));
    if (per_sm < 1) return set_error(VLA_E_CUDA, "fused layer: no resident CTA per SM");
    attr_dev_mask[which] |= 1 << (dev & 31);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(device_info().num_sms);
  cfg.blockDim = dim3(gemm::kThreads);
  cfg.dynamicSmemBytes = lfused::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  prof_begin(st);
  cudaLaunchKernelEx(&cfg, kern, P);
  prof_end(st, VLA_KIND_GEMM,
           2.0 * rows * ((double)NQ * H + (double)H * Q + 2.0 * F * H + (double)H * F) +
               4.0 * batch * w->heads * (double)seq * kv_seq * 64,
           2.0 * ((double)NQ * H + (double)H * Q + 2.0 * F * H + (double)H * F));
  return launch_status("llama_layer_fused");
}

static int llama_self(const vla_llama_layer* w, void* xv, int batch, int seq, const float* rope_cs, void* qkv_out,
                      void* ws, size_t ws_bytes, cudaStream_t st) {
  int rc = check_llama(w);
  if (rc) return rc;
  VLA_CHECK_ARG(xv && rope_cs && batch >= 0 && seq > 0, "llama self: bad arguments");
  const int64_t rows = (int64_t)batch * seq;
  VLA_CHECK_ARG(rows <= kMaxLayerRows, "llama self: batch * seq = %lld rows, above 2^31 - 1", (long long)rows);
  const bool own_qkv = qkv_out == nullptr;
  VLA_CHECK_ARG(ws != nullptr || rows == 0, "llama self: null workspace");
  if (ws_bytes < llama_ws_bytes(w, rows, own_qkv))
    return set_error(VLA_E_WORKSPACE, "llama self: workspace %zu < %zu", ws_bytes, llama_ws_bytes(w, rows, own_qkv));
  VLA_CHECK_ALIGN(aligned16(ws) && aligned16(xv) && (own_qkv || aligned16(qkv_out)), "llama self: alignment");
  if (rows == 0) return VLA_OK;
  LlamaWs b = carve(w, rows, ws, own_qkv);
  bf16* x = (bf16*)xv;
  bf16* qkv = own_qkv ? b.qkv : (bf16*)qkv_out;
  const int64_t H = w->hidden, Q = (int64_t)w->heads * 64, KV = (int64_t)w->kv_heads * 64, NQKV = Q + 2 * KV;
  if (use_fused_layer(w, rows, seq))
    return llama_fused(w, x, batch, seq, rope_cs, qkv, nullptr, nullptr, 0, seq, nullptr, b, false, st);

  rc = rownorm(0, x, H, w->norm1, nullptr, b.h, H, rows, H, w->eps, st, true);
  if (rc) return rc;
  vla_epilogue e{};
  e.b_static = 1;
  e.act = VLA_ACT_ROPE;
  e.rope_cs = rope_cs;
  e.rope_seq = seq;
  e.rope_ncols = (int)(Q + KV);
  rc = gemm::run(b.h, H, w->w_qkv, H, qkv, NQKV, rows, NQKV, H, &e, st);
  if (rc) return rc;
  attn::Params p{};
  p.q = qkv;
  p.k = qkv + Q;
  p.v = qkv + Q + KV;
  p.o = b.attn;
  p.q_row = p.k_row = p.v_row = NQKV;
  p.q_batch = p.k_batch = p.v_batch = (long long)seq * NQKV;
  p.o_row = Q;
  p.o_batch = (long long)seq * Q;
  p.Lq = p.Lk = seq;
  p.Hq = w->heads;
  p.Hkv = w->kv_heads;
  p.causal = 1;
  p.scale_log2 = 0.125f * 1.4426950408889634f;
  rc = attention(p, batch, st);
  if (rc) return rc;
  vla_epilogue r{};
  r.b_static = 1;
  r.residual = x;
  r.ldr = H;
  rc = gemm::run(b.attn, Q, w->w_o, Q, x, H, rows, H, Q, &r, st);
  if (rc) return rc;
  return llama_mlp(w, x, rows, b, st);
}

static int llama_cross(const vla_llama_layer* w, void* xv, int batch, int seq, const float* rope_cs, const void* k,
                       const void* v, int64_t ldkv, int kv_seq, const int* kv_len, void* ws, size_t ws_bytes,
                       cudaStream_t st) {
  int rc = check_llama(w);
  if (rc) return rc;
  VLA_CHECK_ARG(xv && rope_cs && k && v && batch >= 0 && seq > 0 && kv_seq >= 0, "llama cross: bad arguments");
  const int64_t rows = (int64_t)batch * seq;
  VLA_CHECK_ARG(rows <= kMaxLayerRows, "llama cross: batch * seq = %lld rows, above 2^31 - 1", (long long)rows);
  const int64_t H = w->hidden, Q = (int64_t)w->heads * 64;
  VLA_CHECK_ARG(ldkv >= (int64_t)w->kv_heads * 64, "llama cross: ldkv too small");
  if (ws_bytes < llama_ws_bytes(w, rows, true))
    return set_error(VLA_E_WORKSPACE, "llama cross: workspace %zu < %zu", ws_bytes, llama_ws_bytes(w, rows, true));
  VLA_CHECK_ALIGN(aligned16(ws) && aligned16(xv), "llama cross: alignment");
  if (rows == 0) return VLA_OK;
  LlamaWs b = carve(w, rows, ws, true);
  bf16* x = (bf16*)xv;
  bf16* q = b.qkv;  // [rows, Q]
  if (use_fused_layer(w, rows, kv_seq))
    return llama_fused(w, x, batch, seq, rope_cs, q, (const bf16*)k, (const bf16*)v, ldkv, kv_seq, kv_len, b, true,
                       st);

  rc = rownorm(0, x, H, w->norm1, nullptr, b.h, H, rows, H, w->eps, st, true);
  if (rc) return rc;
  vla_epilogue e{};
  e.b_static = 1;
  e.act = VLA_ACT_ROPE;
  e.rope_cs = rope_cs;
  e.rope_seq = seq;
  e.rope_ncols = (int)Q;
  rc = gemm::run(b.h, H, w->w_qkv, H, q, Q, rows, Q, H, &e, st);
  if (rc) return rc;
  attn::Params p{};
  p.q = q;
  p.k = (const bf16*)k;
  p.v = (const bf16*)v;
  p.o = b.attn;
  p.q_row = Q;
  p.q_batch = (long long)seq * Q;
  p.k_row = p.v_row = ldkv;
  p.k_batch = p.v_batch = (long long)kv_seq * ldkv;
  p.o_row = Q;
  p.o_batch = (long long)seq * Q;
  p.Lq = seq;
  p.Lk = kv_seq;
  p.Hq = w->heads;
  p.Hkv = w->kv_heads;
  p.causal = 0;
  p.kv_len = kv_len;
  p.scale_log2 = 0.125f * 1.4426950408889634f;
  rc = attention(p, batch, st);
  if (rc) return rc;
  vla_epilogue r{};
  r.b_static = 1;
  r.residual = x;
  r.ldr = H;
  rc = gemm::run(b.attn, Q, w->w_o, Q, x, H, rows, H, Q, &r, st);
  if (rc) return rc;
  return llama_mlp(w, x, rows, b, st);
}

// ----------------------------------------------------------------------------
// SigLIP encoder layer
// ----------------------------------------------------------------------------
static size_t vision_ws_bytes(const vla_vision_layer* w, int64_t rows) {
  if (rows < 0 || rows > kMaxLayerRows || w->hidden < 0 || w->ffn < 0) return SIZE_MAX;
  const int64_t H = w->hidden;
  return align_up(rows * H * 2) + align_up(rows * 3 * H * 2) + align_up(rows * H * 2) + align_up(rows * w->ffn * 2);
}

static int vision_layer(const vla_vision_layer* w, void* xv, int batch, int seq, void* ws, size_t ws_bytes,
                        cudaStream_t st) {
  VLA_CHECK_ARG(w && xv, "vision layer: null argument");
  VLA_CHECK_ARG(w->ln1_g && w->ln1_b && w->w_qkv && w->b_qkv && w->w_o && w->b_o && w->ln2_g && w->ln2_b &&
                    w->w_fc1 && w->b_fc1 && w->w_fc2 && w->b_fc2,
                "vision layer: null weight");
  VLA_CHECK_ARG(w->head_dim == 64 && w->heads * 64 == w->hidden, "vision layer: heads * 64 must equal hidden");
  VLA_CHECK_ARG(batch >= 0 && seq > 0, "vision layer: bad batch / seq");
  const int64_t rows = (int64_t)batch * seq, H = w->hidden, F = w->ffn;
  VLA_CHECK_ARG(rows <= kMaxLayerRows, "vision layer: batch * seq = %lld rows, above 2^31 - 1", (long long)rows);
  if (ws_bytes < vision_ws_bytes(w, rows))
    return set_error(VLA_E_WORKSPACE, "vision layer: workspace %zu < %zu", ws_bytes, vision_ws_bytes(w, rows));
  VLA_CHECK_ALIGN(aligned16(ws) && aligned16(xv), "vision layer: alignment");
  if (rows == 0) return VLA_OK;
  uint8_t* p8 = (uint8_t*)ws;
  bf16* h = (bf16*)p8;
  p8 += align_up(rows * H * 2);
  bf16* qkv = (bf16*)p8;
  p8 += align_up(rows * 3 * H * 2);
  bf16* at = (bf16*)p8;
  p8 += align_up(rows * H * 2);
  bf16* mlp = (bf16*)p8;
  bf16* x = (bf16*)xv;

  int rc = rownorm(1, x, H, w->ln1_g, w->ln1_b, h, H, rows, H, w->eps, st, true);
  if (rc) return rc;
  vla_epilogue e{};
  e.b_static = 1;
  e.bias = w->b_qkv;
  rc = gemm::run(h, H, w->w_qkv, H, qkv, 3 * H, rows, 3 * H, H, &e, st);
  if (rc) return rc;
  attn::Params p{};
  p.q = qkv;
  p.k = qkv + H;
  p.v = qkv + 2 * H;
  p.o = at;
  p.q_row = p.k_row = p.v_row = 3 * H;
  p.q_batch = p.k_batch = p.v_batch = (long long)seq * 3 * H;
  p.o_row = H;
  p.o_batch = (long long)seq * H;
  p.Lq = p.Lk = seq;
  p.Hq = p.Hkv = w->heads;
  p.causal = 0;
  p.scale_log2 = 0.125f * 1.4426950408889634f;
  rc = attention(p, batch, st);
  if (rc) return rc;
  vla_epilogue r{};
  r.b_static = 1;
  r.bias = w->b_o;
  r.residual = x;
  r.ldr = H;
  rc = gemm::run(at, H, w->w_o, H, x, H, rows, H, H, &r, st);
  if (rc) return rc;
  rc = rownorm(1, x, H, w->ln2_g, w->ln2_b, h, H, rows, H, w->eps, st, true);
  if (rc) return rc;
  vla_epilogue g{};
  g.b_static = 1;
  g.bias = w->b_fc1;
  g.act = VLA_ACT_GELU_TANH;
  rc = gemm::run(h, H, w->w_fc1, H, mlp, F, rows, F, H, &g, st);
  if (rc) return rc;
  vla_epilogue d{};
  d.b_static = 1;
  d.bias = w->b_fc2;
  d.residual = x;
  d.ldr = H;
  return gemm::run(mlp, F, w->w_fc2, F, x, H, rows, H, F, &d, st);
}

}  // namespace blocks
}  // namespace vla
