// libvla_b200.so — single translation unit holding every sm_100a kernel of
// the SmolVLA hot path and the extern "C" entry points declared in
// include/vla_b200.h.  One TU keeps the device error word in one place.
#include <cmath>
#include <vector>

#include "blocks.cuh"
#include "render.cuh"
#include "gemm_host.cuh"
#include "host_common.cuh"

using namespace vla;

// Scratch of vla_llama_self_layer_bf16_noalloc: one fixed array in device
// memory, present on every device that loads this library.  Host code may
// not use the symbol itself as a device address; it looks the address up
// once per device (noalloc_scratch below).
static __device__ __align__(256) unsigned char g_noalloc_scratch[VLA_NOALLOC_SCRATCH_BYTES];

static void* noalloc_scratch(int* rc) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    *rc = set_error(VLA_E_CUDA, "noalloc: cudaGetDevice failed");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *rc = set_error(VLA_E_CUDA, "noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                      cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = p;
  }
  *rc = VLA_OK;
  return addr[dev];
}

// One thread waits on a fresh mbarrier that nothing arrives on; the bounded
// wait gives up after limit_ns and records the test code.
__global__ void expired_wait_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  mbar_fence_init();
  if (!mbar_wait_bounded(&bar, 0u, nullptr, limit_ns)) vla_record_error(VLA_DERR_TEST_TIMEOUT);
}

// y = 2^x by the FMA-pipe exponential of the SigLIP attention's softmax
// (attn_tc::ex2_poly2), one pair of elements per thread.
__global__ void exp2_fma_kernel(const float* x, float* y, long long n) {
  const long long i = 2 * ((long long)blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float x1 = i + 1 < n ? x[i + 1] : 0.f;
  float e0, e1;
  attn_tc::ex2_poly2(x[i], x1, e0, e1);
  y[i] = e0;
  if (i + 1 < n) y[i + 1] = e1;
}

extern "C" {

const char* vla_last_error(void) { return t_last_error; }

int vla_test_expired_wait(int32_t limit_us, vla_stream_t stream) {
  VLA_CHECK_ARG(limit_us >= 1 && limit_us <= 1000000, "test_expired_wait: limit_us must be in [1, 1e6]");
  expired_wait_kernel<<<1, 32, 0, as_stream(stream)>>>((uint64_t)limit_us * 1000ull);
  return launch_status("test_expired_wait");
}

int vla_test_exp2_fma(const float* x, float* y, int64_t n, vla_stream_t stream) {
  VLA_CHECK_ARG(x != nullptr && y != nullptr, "test_exp2_fma: null pointer");
  VLA_CHECK_ARG(n >= 0 && n <= (1ll << 30), "test_exp2_fma: n must be in [0, 2^30]");
  if (n == 0) return VLA_OK;
  const long long pairs = (n + 1) / 2;
  exp2_fma_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, as_stream(stream)>>>(x, y, n);
  return launch_status("test_exp2_fma");
}

int vla_version(void) { return 100; }

int vla_sync_check(void) {
  VLA_CUDA_TRY(cudaDeviceSynchronize());
  unsigned int code = 0, zero = 0;
  VLA_CUDA_TRY(cudaMemcpyFromSymbol(&code, g_vla_device_error, sizeof(code)));
  if (code != 0) {
    VLA_CUDA_TRY(cudaMemcpyToSymbol(g_vla_device_error, &zero, sizeof(zero)));
    return set_error(VLA_E_DEVICE_TIMEOUT, "device wait limit expired (code 0x%x)", code);
  }
  return VLA_OK;
}

int vla_peek_device_error(unsigned int* code) {
  VLA_CHECK_ARG(code != nullptr, "null code");
  VLA_CUDA_TRY(cudaMemcpyFromSymbol(code, g_vla_device_error, sizeof(*code)));
  return VLA_OK;
}

uint64_t vla_launch_count(void) { return g_launch_count.load(); }

int vla_set_fused_layers(int32_t enable) { return blocks::g_fused_layers.exchange(enable ? 1 : 0); }

int vla_set_launch_overlap(int32_t enable) {
  const int old = g_launch_overlap.exchange(enable ? 1 : 0);
  return old;
}

int vla_profile_start(int32_t capacity) {
  VLA_CHECK_ARG(capacity > 0, "profile_start: capacity must be positive");
  VLA_CHECK_ARG(!g_prof.on, "profile_start: profiler already running");
  for (auto e : g_prof.pool) cudaEventDestroy(e);
  g_prof.pool.assign(2 * (size_t)capacity, nullptr);
  for (auto& e : g_prof.pool) VLA_CUDA_TRY(cudaEventCreate(&e));
  g_prof.recs.clear();
  g_prof.recs.reserve(capacity);
  g_prof.next = 0;
  g_prof.pending = nullptr;
  g_prof.on = true;
  return VLA_OK;
}

int vla_profile_stop(vla_profile_record* out, int32_t capacity, int32_t* count) {
  VLA_CHECK_ARG(g_prof.on, "profile_stop: profiler not running");
  g_prof.on = false;
  int n = 0;
  for (const ProfRec& r : g_prof.recs) {
    VLA_CUDA_TRY(cudaEventSynchronize(r.b));
    if (out != nullptr && n < capacity) {
      float ms = 0.f;
      VLA_CUDA_TRY(cudaEventElapsedTime(&ms, r.a, r.b));
      out[n].kind = r.kind;
      out[n].ms = ms;
      out[n].flops = r.flops;
      out[n].bytes = r.bytes;
      out[n].m = r.m;
      out[n].n = r.n;
      out[n].k = r.k;
      out[n].tile_n = r.tile_n;
      out[n].ctas = r.ctas;
    }
    ++n;
  }
  if (count) *count = n;
  for (auto e : g_prof.pool) cudaEventDestroy(e);
  g_prof.pool.clear();
  g_prof.recs.clear();
  return VLA_OK;
}

int vla_abi_sizes(int64_t* out, int32_t n) {
  const int64_t sz[5] = {(int64_t)sizeof(vla_epilogue), (int64_t)sizeof(vla_attention_args),
                         (int64_t)sizeof(vla_llama_layer), (int64_t)sizeof(vla_vision_layer),
                         (int64_t)sizeof(vla_profile_record)};
  for (int i = 0; i < n && i < 5; ++i) out[i] = sz[i];
  return 5;
}

int vla_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M, int64_t N,
                  int64_t K, const vla_epilogue* epi, vla_stream_t stream) {
  return gemm::run(A, lda, B, ldb, C, ldc, M, N, K, epi, as_stream(stream));
}

int vla_gemm_bf16_tiled(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                        int64_t N, int64_t K, const vla_epilogue* epi, int tile_n, vla_stream_t stream) {
  VLA_CHECK_ARG(tile_n >= 32 && tile_n <= 256 && tile_n % 32 == 0, "tile_n must be a multiple of 32 in [32, 256]");
  return gemm::run(A, lda, B, ldb, C, ldc, M, N, K, epi, as_stream(stream), tile_n);
}

int vla_gemm_bf16_ex(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                     int64_t N, int64_t K, const vla_epilogue* epi, int32_t tile_n, int32_t ctas, vla_stream_t stream) {
  VLA_CHECK_ARG(tile_n == 0 || (tile_n >= 32 && tile_n <= 256 && tile_n % 32 == 0),
                "tile_n must be 0 or a multiple of 32 in [32, 256]");
  VLA_CHECK_ARG(ctas >= 0 && ctas <= 2, "ctas must be 0 (auto), 1 or 2");
  VLA_CHECK_ARG(ctas != 2 || tile_n == 0 || tile_n >= 64, "a CTA pair needs tile_n >= 64");
  return gemm::run(A, lda, B, ldb, C, ldc, M, N, K, epi, as_stream(stream), tile_n, ctas);
}

int vla_gemm_bf16_split(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                        int64_t N, int64_t K, const vla_epilogue* epi, int32_t tile_n, int32_t splits,
                        vla_stream_t stream) {
  VLA_CHECK_ARG(splits == 0 || splits == 1 || (splits >= 2 && splits <= 8), "gemm: splits must be 0, 1 or 2..8");
  VLA_CHECK_ARG(tile_n == 0 || tile_n == 32 || tile_n == 64 || tile_n == 128,
                "gemm split-K: tile_n must be 0, 32, 64 or 128");
  return gemm::run(A, lda, B, ldb, C, ldc, M, N, K, epi, as_stream(stream), tile_n, 1,
                   splits == 0 ? -1 : splits == 1 ? 0 : splits);
}

int vla_rms_norm_bf16(const void* x, int64_t ldx, const void* g, void* y, int64_t ldy, int64_t M, int64_t N, float eps,
                      vla_stream_t stream) {
  return blocks::rownorm(0, x, ldx, g, nullptr, y, ldy, M, N, eps, as_stream(stream));
}

int vla_layer_norm_bf16(const void* x, int64_t ldx, const void* g, const void* b, void* y, int64_t ldy, int64_t M,
                        int64_t N, float eps, vla_stream_t stream) {
  return blocks::rownorm(1, x, ldx, g, b, y, ldy, M, N, eps, as_stream(stream));
}

int vla_rope_bf16(void* x, int64_t ld, int64_t M, int32_t ncols, int32_t seq, const float* cs, vla_stream_t stream) {
  VLA_CHECK_ARG(x && cs && M >= 0 && seq > 0 && ncols > 0 && ncols % 64 == 0 && ld >= ncols, "rope: bad arguments");
  VLA_CHECK_ALIGN(aligned16(x) && ld % 8 == 0, "rope: alignment");
  if (M == 0) return VLA_OK;
  const long long work = M * (ncols / 64) * 4;
  prof_begin(as_stream(stream));
  launch_k(ew::rope_kernel, dim3(blocks::grid_for(work, 256)), dim3(256), 0, as_stream(stream), (bf16*)x, ld, M, ncols, seq, cs);
  prof_end(as_stream(stream), VLA_KIND_ROPE, 0.0, 4.0 * (double)M * ncols);
  return launch_status("rope");
}

int vla_rope_table(float* cs, int32_t seq, int32_t head_dim, double theta) {
  VLA_CHECK_ARG(cs && seq > 0 && head_dim > 0 && head_dim % 2 == 0, "rope_table: bad arguments");
  const int half = head_dim / 2;
  for (int k = 0; k < half; ++k) {
    const float expo = (2.0f / (float)head_dim) * (float)k;
    const float ts = (float)std::pow(theta, (double)expo);
    for (int pos = 0; pos < seq; ++pos) {
      const float rad = (float)pos / ts;
      cs[(size_t)pos * head_dim + k] = (float)std::cos((double)rad);
      cs[(size_t)pos * head_dim + half + k] = (float)std::sin((double)rad);
    }
  }
  return VLA_OK;
}

int vla_softmax_bf16(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M, int64_t N, float scale,
                     int32_t causal_row_start, vla_stream_t stream) {
  VLA_CHECK_ARG(x && y && M >= 0 && N > 0 && ldx >= N && ldy >= N, "softmax: bad arguments");
  if (M == 0) return VLA_OK;
  const int wpb = 8;
  prof_begin(as_stream(stream));
  launch_k(ew::softmax_kernel, dim3((int)((M + wpb - 1) / wpb)), dim3(wpb * 32), 0, as_stream(stream), 
      (const bf16*)x, ldx, (bf16*)y, ldy, (int)M, (int)N, scale, causal_row_start);
  prof_end(as_stream(stream), VLA_KIND_SOFTMAX, 0.0, 4.0 * (double)M * N);
  return launch_status("softmax");
}

int vla_elementwise_bf16(int32_t op, const void* x, int64_t ldx, const void* y2, int64_t ldy2, void* out, int64_t ldo,
                         int64_t M, int64_t N, vla_stream_t stream) {
  VLA_CHECK_ARG(op >= 0 && op <= 3, "elementwise: unknown op %d", op);
  VLA_CHECK_ARG(x && out && (op < 2 || y2) && M >= 0 && N > 0 && N % 8 == 0, "elementwise: bad arguments");
  VLA_CHECK_ALIGN(aligned16(x) && aligned16(out) && (op < 2 || aligned16(y2)) && ldx % 8 == 0 && ldo % 8 == 0 &&
                      (op < 2 || ldy2 % 8 == 0),
                  "elementwise: alignment");
  if (M == 0) return VLA_OK;
  prof_begin(as_stream(stream));
  launch_k(ew::act_kernel, dim3(blocks::grid_for(M * (N / 8), 256)), dim3(256), 0, as_stream(stream), 
      (const bf16*)x, ldx, (const bf16*)y2, ldy2, (bf16*)out, ldo, M, (int)N, op);
  prof_end(as_stream(stream), VLA_KIND_ELEMENTWISE, 0.0, (op >= 2 ? 6.0 : 4.0) * (double)M * N);
  return launch_status("elementwise");
}

int vla_attention_bf16(const vla_attention_args* a, vla_stream_t stream) {
  VLA_CHECK_ARG(a != nullptr, "attention: null args");
  VLA_CHECK_ARG(a->head_dim == 64, "attention: head_dim must be 64");
  VLA_CHECK_ARG(std::fabs(a->scale - 0.125f) < 1e-7f, "attention: scale must be 1/sqrt(64)");
  attn::Params p{};
  p.q = (const bf16*)a->q;
  p.k = (const bf16*)a->k;
  p.v = (const bf16*)a->v;
  p.o = (bf16*)a->o;
  p.q_row = a->q_row;
  p.k_row = a->k_row;
  p.v_row = a->v_row;
  p.o_row = a->o_row;
  p.q_batch = a->q_batch;
  p.k_batch = a->k_batch;
  p.v_batch = a->v_batch;
  p.o_batch = a->o_batch;
  p.Lq = a->Lq;
  p.Lk = a->Lk;
  p.Hq = a->Hq;
  p.Hkv = a->Hkv;
  p.causal = a->causal;
  p.kv_len = a->kv_len;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  VLA_CHECK_ARG(a->impl >= VLA_ATTN_AUTO && a->impl <= VLA_ATTN_TCGEN05_PIPE, "attention: unknown impl %d", a->impl);
  return blocks::attention(p, a->batch, as_stream(stream), a->impl);
}

int vla_pixel_shuffle_bf16(const void* in, void* out, int32_t B, int32_t grid, int32_t scale, int32_t C,
                           vla_stream_t stream) {
  VLA_CHECK_ARG(in && out && B >= 0 && grid > 0 && scale > 0 && grid % scale == 0 && C > 0 && C % 8 == 0,
                "pixel_shuffle: bad arguments");
  VLA_CHECK_ALIGN(aligned16(in) && aligned16(out), "pixel_shuffle: alignment");
  if (B == 0) return VLA_OK;
  const long long work = (long long)B * grid * grid * (C / 8);
  prof_begin(as_stream(stream));
  // 32-bit vector counter while it cannot overflow (with the grid stride added)
  auto ps_kern = work < (1ll << 30) ? ew::pixel_shuffle_kernel<int> : ew::pixel_shuffle_kernel<long long>;
  launch_k(ps_kern, dim3(blocks::grid_for(work, 256)), dim3(256), 0, as_stream(stream), (const bf16*)in, (bf16*)out, B,
           grid, scale, C);
  prof_end(as_stream(stream), VLA_KIND_LAYOUT, 0.0, 4.0 * (double)B * grid * grid * C);
  return launch_status("pixel_shuffle");
}

int vla_camera_preprocess_u8(const uint8_t* frames, int32_t B, int32_t H, int32_t W, int32_t S, int32_t p,
                             int32_t mode, void* out, vla_stream_t stream) {
  VLA_CHECK_ARG(frames && out && B >= 0 && H > 0 && W > 0 && S > 0 && S % 8 == 0 && (mode == 0 || mode == 1),
                "camera_preprocess: bad arguments (S must be a positive multiple of 8, mode 0 or 1)");
  VLA_CHECK_ARG(mode == 0 || (p > 0 && p % 8 == 0 && S % p == 0),
                "camera_preprocess: patch mode needs p a multiple of 8 dividing S");
  VLA_CHECK_ALIGN(aligned16(out), "camera_preprocess: output alignment");
  if (B == 0) return VLA_OK;
  const long long work = (long long)B * 3 * S * (S / 8);
  prof_begin(as_stream(stream));
  auto kern = work < (1ll << 30) ? ew::camera_preprocess_kernel<int> : ew::camera_preprocess_kernel<long long>;
  launch_k(kern, dim3(blocks::grid_for(work, 256)), dim3(256), 0, as_stream(stream), frames, (bf16*)out, B, H, W, S,
           p, mode, (float)H / (float)S, (float)W / (float)S);
  prof_end(as_stream(stream), VLA_KIND_LAYOUT, 0.0, (double)B * H * W * 3 + 2.0 * B * 3 * S * S);
  return launch_status("camera_preprocess");
}

int vla_pusht_render_u8(const float* scene, int32_t n, int32_t S, uint8_t* frames, vla_stream_t stream) {
  VLA_CHECK_ARG(scene && frames && n >= 0 && S > 0, "pusht_render: bad arguments");
  if (n == 0) return VLA_OK;
  const long long work = (long long)n * S * S;
  prof_begin(as_stream(stream));
  launch_k(render::pusht_render_kernel, dim3(blocks::grid_for(work, 256)), dim3(256), 0, as_stream(stream), scene, n,
           S, frames);
  prof_end(as_stream(stream), VLA_KIND_LAYOUT, 0.0, 3.0 * (double)work);
  return launch_status("pusht_render");
}

int vla_patch_im2col_bf16(const void* img, void* out, int32_t B, int32_t Cin, int32_t H, int32_t W, int32_t p,
                          vla_stream_t stream) {
  VLA_CHECK_ARG(img && out && B >= 0 && Cin > 0 && p > 0 && H % p == 0 && W % p == 0 && p % 8 == 0,
                "im2col: bad arguments (patch must be a multiple of 8, H and W multiples of patch)");
  VLA_CHECK_ALIGN(aligned16(img) && aligned16(out), "im2col: alignment");
  if (B == 0) return VLA_OK;
  const long long work = (long long)B * (H / p) * (W / p) * (Cin * p * p / 8);
  prof_begin(as_stream(stream));
  auto ic_kern = work < (1ll << 30) ? ew::im2col_kernel<int> : ew::im2col_kernel<long long>;
  launch_k(ic_kern, dim3(blocks::grid_for(work, 256)), dim3(256), 0, as_stream(stream), (const bf16*)img, (bf16*)out, B,
           Cin, H, W, p);
  prof_end(as_stream(stream), VLA_KIND_LAYOUT, 0.0, 4.0 * (double)B * Cin * H * W);
  return launch_status("im2col");
}

int vla_embed_bf16(const int32_t* ids, const void* table, int32_t vocab, int32_t H, int32_t B, int32_t T, float scale,
                   void* out, int64_t ldo, int32_t rows_per_seq, int32_t row_offset, vla_stream_t stream) {
  VLA_CHECK_ARG(ids && table && out && vocab > 0 && H > 0 && H % 8 == 0 && B >= 0 && T >= 0 && ldo >= H &&
                    row_offset >= 0 && row_offset + T <= rows_per_seq,
                "embed: bad arguments");
  VLA_CHECK_ALIGN(aligned16(table) && aligned16(out) && ldo % 8 == 0, "embed: alignment");
  if (B == 0 || T == 0) return VLA_OK;
  const long long work = (long long)B * T * (H / 8);
  prof_begin(as_stream(stream));
  launch_k(ew::embed_kernel, dim3(blocks::grid_for(work, 256)), dim3(256), 0, as_stream(stream), 
      ids, (const bf16*)table, vocab, H, B, T, scale, (bf16*)out, ldo, rows_per_seq, row_offset);
  prof_end(as_stream(stream), VLA_KIND_LAYOUT, 0.0, 4.0 * (double)B * T * H);
  return launch_status("embed");
}

int vla_f32_to_bf16(const float* x, int64_t ldx, void* y, int64_t ldy, int64_t M, int64_t N, vla_stream_t stream) {
  VLA_CHECK_ARG(x && y && M >= 0 && N > 0 && ldx >= N && ldy >= N, "f32_to_bf16: bad arguments");
  if (M == 0) return VLA_OK;
  prof_begin(as_stream(stream));
  launch_k(ew::f32_to_bf16_kernel, dim3(blocks::grid_for(M * N, 256)), dim3(256), 0, as_stream(stream), x, ldx, (bf16*)y, ldy, M,
                                                                                      (int)N);
  prof_end(as_stream(stream), VLA_KIND_LAYOUT, 0.0, 6.0 * (double)M * N);
  return launch_status("f32_to_bf16");
}

size_t vla_llama_layer_workspace(const vla_llama_layer* w, int64_t rows, int32_t with_qkv) {
  if (w == nullptr || rows < 0) return 0;
  return blocks::llama_ws_bytes(w, rows, with_qkv != 0);
}

int vla_llama_self_layer_bf16(const vla_llama_layer* w, void* x, int32_t batch, int32_t seq, const float* rope_cs,
                              void* qkv_out, void* workspace, size_t workspace_bytes, vla_stream_t stream) {
  return blocks::llama_self(w, x, batch, seq, rope_cs, qkv_out, workspace, workspace_bytes, as_stream(stream));
}

int vla_llama_cross_layer_bf16(const vla_llama_layer* w, void* x, int32_t batch, int32_t seq, const float* rope_cs,
                               const void* k, const void* v, int64_t ldkv, int32_t kv_seq, const int32_t* kv_len,
                               void* workspace, size_t workspace_bytes, vla_stream_t stream) {
  return blocks::llama_cross(w, x, batch, seq, rope_cs, k, v, ldkv, kv_seq, kv_len, workspace, workspace_bytes,
                             as_stream(stream));
}

size_t vla_noalloc_scratch_bytes(void) { return VLA_NOALLOC_SCRATCH_BYTES; }

int vla_llama_self_layer_bf16_noalloc(const vla_llama_layer* w, void* x, int32_t batch, int32_t seq,
                                      const float* rope_cs, void* qkv_out, vla_stream_t stream) {
  VLA_CHECK_ARG(w != nullptr && batch >= 0 && seq > 0, "noalloc llama self: bad arguments");
  const int64_t rows = (int64_t)batch * seq;
  VLA_CHECK_ARG(rows <= blocks::kMaxLayerRows, "noalloc llama self: batch * seq = %lld rows, above 2^31 - 1",
                (long long)rows);
  const size_t need = blocks::llama_ws_bytes(w, rows, qkv_out == nullptr);
  if (need > VLA_NOALLOC_SCRATCH_BYTES)
    return set_error(VLA_E_WORKSPACE,
                     "noalloc llama self: %lld rows need %zu bytes of scratch, above the fixed %u-byte static array; "
                     "use vla_llama_self_layer_bf16 with a caller workspace",
                     (long long)rows, need, (unsigned)VLA_NOALLOC_SCRATCH_BYTES);
  int rc = VLA_OK;
  void* scratch = noalloc_scratch(&rc);
  if (scratch == nullptr) return rc;
  return blocks::llama_self(w, x, batch, seq, rope_cs, qkv_out, scratch, VLA_NOALLOC_SCRATCH_BYTES,
                            as_stream(stream));
}

size_t vla_vision_layer_workspace(const vla_vision_layer* w, int64_t rows) {
  if (w == nullptr || rows < 0) return 0;
  return blocks::vision_ws_bytes(w, rows);
}

int vla_vision_layer_bf16(const vla_vision_layer* w, void* x, int32_t batch, int32_t seq, void* workspace,
                          size_t workspace_bytes, vla_stream_t stream) {
  return blocks::vision_layer(w, x, batch, seq, workspace, workspace_bytes, as_stream(stream));
}

}  // extern "C"
