/*
 * vla_b200.h — C ABI of libvla_b200.so, the sm_100a (B200) implementation of
 * the SmolVLA bf16 inference hot path.
 *
 * Each entry point replaces one kernel module (or one host-side block
 * builder) of the reference xl434/vla-to-npu, cited per function as
 * reference-file:line.  In the reference every kernel is an Allo
 * `ExternalModule(top=..., impl_path=...)` with a fixed-shape signature
 * `extern "C" void top(bfloat16 in[R][C], ..., bfloat16 out[R][C])`, called
 * as `mod(np_in..., np_out)` with caller-owned buffers and no status.  Here:
 *
 *   - every pointer is a DEVICE pointer (CUDA global memory) owned by the
 *     caller; bf16 tensors are row-major with an explicit row stride in
 *     elements (ld*); shapes are runtime arguments, not compile-time;
 *   - every call is asynchronous on the given CUDA stream (NULL = legacy
 *     default stream) and returns 0 on success or a negative VLA_E* code;
 *     vla_last_error() returns a thread-local message for the last failure;
 *   - kernels never trap or spin forever: a bounded wait that expires sets a
 *     device error word that vla_sync_check() reports (VLA_E_DEVICE_TIMEOUT);
 *   - weights of linear layers are passed K-major, i.e. as W^T with shape
 *     [out_features, in_features] (torch nn.Linear layout).  The reference
 *     stores them [in, out] (`params["Wq"] = W.T`,
 *     vla/text_encoder_bf16.py:602); the host wrappers transpose once.
 */
#ifndef VLA_B200_H
#define VLA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* vla_stream_t; /* a cudaStream_t */

enum {
  VLA_OK = 0,
  VLA_E_INVALID = -1,      /* bad shape / stride / null pointer */
  VLA_E_ALIGN = -2,        /* pointer or stride violates the 16-byte TMA rule */
  VLA_E_CUDA = -3,         /* a CUDA runtime / driver call failed */
  VLA_E_UNSUPPORTED = -4,  /* valid request this build does not implement */
  VLA_E_DEVICE_TIMEOUT = -5, /* a kernel's bounded wait expired (see vla_sync_check) */
  VLA_E_WORKSPACE = -6     /* workspace too small */
};

/* Activation / epilogue kinds of vla_gemm_bf16. */
enum {
  VLA_ACT_NONE = 0,
  VLA_ACT_GELU_TANH = 1, /* 0.5 x (1 + tanh(0.79788456 (x + 0.044715 x^3))) */
  VLA_ACT_SWIGLU = 2,    /* B rows interleaved in 16-row blocks [gate16 | up16]; C[:, j] = silu(g) * u, C has N/2 cols */
  VLA_ACT_ROPE = 3,      /* rotate columns [0, rope_ncols) in 64-wide heads (half-split RoPE) */
  VLA_ACT_EULER = 4      /* fp32 state x[m, n] += euler_dt * acc; C = bf16(x) */
};

/*
 * Fused GEMM epilogue.  For output element (m, n):
 *   v = alpha * acc(m, n) + bias[n]
 *   v = act(v)                    (GELU / SwiGLU pair / RoPE rotation / Euler update)
 *   v = v + residual[r(m), n]     r(m) = m % res_row_mod if res_row_mod > 0 else m
 *   C[o(m), n] = bf16(v)          o(m) = (m / out_grp) * out_grp_stride + m % out_grp if out_grp > 0 else m
 * A zero-initialised struct (alpha = 0 is read as 1) gives the plain product.
 */
typedef struct vla_epilogue {
  const void* bias;      /* bf16 [N] or NULL */
  const void* residual;  /* bf16, row stride ldr, or NULL (may alias C for in-place residual adds) */
  int64_t ldr;
  int32_t res_row_mod;
  int32_t act;           /* VLA_ACT_* */
  float alpha;
  int32_t rope_seq;      /* RoPE position of row m = m % rope_seq */
  const float* rope_cs;  /* fp32 table [positions][64]: cos(pos*f_k) k<32, then sin(pos*f_k) */
  int32_t rope_ncols;    /* columns [0, rope_ncols) are rotated, multiple of 64 */
  int32_t out_grp;
  int64_t out_grp_stride;
  float* euler_x;        /* fp32 [M, ldx] Euler state (VLA_ACT_EULER) */
  int64_t ldx;
  float euler_dt;
  /* 1 when no work earlier in the stream writes B (model weights): a one-CTA
   * launch may then fetch its first B tiles while the previous kernel drains. */
  int32_t b_static;
  int32_t reserved[3];
} vla_epilogue;

/* ---------------------------------------------------------------------- */
/* Library status                                                          */
/* ---------------------------------------------------------------------- */
const char* vla_last_error(void);
int vla_version(void);
/* Synchronises the current device, then reads and clears the device error
 * word.  Returns VLA_OK, VLA_E_DEVICE_TIMEOUT or VLA_E_CUDA. */
int vla_sync_check(void);
/* Device error word without clearing (0 = none). */
int vla_peek_device_error(unsigned int* code);
/* Exercises the device error channel without a fault: launches one block whose
 * thread waits on an mbarrier that nothing ever completes, with a time limit of
 * limit_us microseconds (1 .. 1000000); the wait runs out, the kernel records
 * the test code 0x1FF in the device error word and returns.  A following
 * vla_sync_check() then reports VLA_E_DEVICE_TIMEOUT.  No counterpart in the
 * reference (its NPU calls have no error channel). */
int vla_test_expired_wait(int32_t limit_us, vla_stream_t stream);
/* Evaluates y[i] = 2^x[i] (n fp32 device values) with the FMA-pipe
 * exponential that the SigLIP attention kernel uses for a quarter of its
 * softmax keys (Cody-Waite split, cubic minimax fit of 2^f on [0, 1)), so its
 * error bound can be tested against exact powers of two.  Inputs below -126
 * give values below 2^-126.  No counterpart in the reference (its AIE softmax
 * takes exp from a lookup table). */
int vla_test_exp2_fma(const float* x, float* y, int64_t n, vla_stream_t stream);
/* sizeof of the ABI structs, in the order vla_epilogue, vla_attention_args,
 * vla_llama_layer, vla_vision_layer, vla_profile_record, written to out[0..n);
 * returns the count. */
int vla_abi_sizes(int64_t* out, int32_t n);
/* Number of kernel launches this library has issued in this process (all
 * devices, all threads); a graph replay re-runs captured launches without
 * counting them again. */
uint64_t vla_launch_count(void);
/* Launch overlap between consecutive kernels of this library on one stream
 * (programmatic dependent launch: a kernel may be scheduled while its
 * predecessor drains and waits for the predecessor's results before its first
 * global-memory access).  On by default; 0 disables it.  Returns the previous
 * setting.  No counterpart in the reference (its NPU calls are synchronous). */
int vla_set_launch_overlap(int32_t enable);
/* Single-launch layers: a vla_llama_self_layer_bf16 / vla_llama_cross_layer_bf16
 * call of at most 512 rows (batch * seq) with at most 128 keys runs the whole
 * layer (two RMSNorms, four GEMMs, attention) as ONE cooperative kernel, one CTA
 * per SM, its phases separated by grid-wide barriers, instead of seven
 * dependent launches.  Results are bit-identical to the seven-launch path.
 * Off by default: measured at one observation it is slower (an expert layer
 * ~66 us against ~50 us inside a CUDA graph: each phase's TMA / MMA / store
 * latency plus a grid barrier costs more than the launch it saves).  1 enables
 * it, 0 disables; returns the previous setting.  No counterpart in the
 * reference (its layers are sequences of NPU calls). */
int vla_set_fused_layers(int32_t enable);

/* Launch profiler (measurement only; no counterpart in the reference, whose
 * timing is the XRT host's "NPU execution time" print, gemm/v1_test_tiled_gemm.py:81-96).
 * Between vla_profile_start and vla_profile_stop every launch of this library
 * on this thread is bracketed by CUDA events; stop synchronises and returns one
 * record per launch: its kind, device time and algorithmic FLOPs / bytes.
 * Not for use during CUDA-graph capture. */
enum {
  VLA_KIND_GEMM = 0,
  VLA_KIND_ATTENTION = 1,
  VLA_KIND_NORM = 2,
  VLA_KIND_ROPE = 3,
  VLA_KIND_SOFTMAX = 4,
  VLA_KIND_ELEMENTWISE = 5,
  VLA_KIND_LAYOUT = 6
};
typedef struct vla_profile_record {
  int32_t kind;
  float ms;
  double flops;
  double bytes;
  int64_t m, n, k;  /* GEMM problem shape (0 for other kinds) */
  int32_t tile_n;   /* GEMM: output tile width BN */
  int32_t ctas;     /* GEMM: CTAs per output tile (1, or 2 for a cta_group::2 pair) */
} vla_profile_record;
int vla_profile_start(int32_t capacity);
int vla_profile_stop(vla_profile_record* out, int32_t capacity, int32_t* count);

/* ---------------------------------------------------------------------- */
/* Per-op kernels (the reference's ExternalModule tops)                    */
/* ---------------------------------------------------------------------- */

/* C[M, N] = epilogue(A[M, K] . B[N, K]^T), bf16 in, fp32 accumulate in
 * tensor memory (tcgen05), bf16 out.
 * Replaces Allo `GEMM(M, N, K, Pm, Pn, Pk, bf16, bf16)` (library module;
 * local copy cc/gemm.py:44-77; call sites vla/text_encoder_bf16.py:175-224,
 * vla/vision_block_bf16.py:135-169, vla/action_expert_bf16.py:247-321) and the
 * host K-chunk accumulation loops (vla/text_encoder_bf16.py:583-590).
 * Constraints: K >= 1; N % 16 == 0; lda, ldb, ldc multiples of 8; A, B, C
 * 16-byte aligned.  For VLA_ACT_SWIGLU N % 32 == 0 and C has N/2 columns. */
int vla_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M, int64_t N,
                  int64_t K, const vla_epilogue* epi, vla_stream_t stream);

/* Same GEMM with the N tile width forced (a multiple of 32 in [32, 256]) instead of chosen
 * by the launcher's wave-count heuristic; used by tests and tile sweeps. */
int vla_gemm_bf16_tiled(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                        int64_t N, int64_t K, const vla_epilogue* epi, int32_t tile_n, vla_stream_t stream);


/* The GEMM with its schedule chosen by the caller: tile_n = N tile width
 * (multiple of 32 in [32, 256], 0 = automatic) and ctas = 1 (one CTA per
 * 128 x tile_n tile), 2 (a two-CTA cluster per 256 x tile_n tile, tile_n >= 64:
 * each CTA stages its own A rows and half of the B tile, the pair's MMAs are
 * issued by one CTA as tcgen05.mma.cta_group::2) or 0 (automatic). */
int vla_gemm_bf16_ex(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                     int64_t N, int64_t K, const vla_epilogue* epi, int32_t tile_n, int32_t ctas, vla_stream_t stream);

/* The GEMM on one-CTA tiles with the K extent split over a cluster of
 * `splits` CTAs (2..8) per output tile: each CTA multiplies its contiguous
 * share of the k-blocks, the partial fp32 tiles are summed in the leading
 * CTA's shared memory (distributed shared memory, no global scratch) and the
 * leader runs the fused epilogue.  It puts more SMs on the weight stream of
 * outputs with few tiles, but at one observation (M = 50) the clustered launch
 * measured slower than the plain one, so vla_gemm_bf16 never splits by itself.
 * splits 2..8 (at most 5 CTAs at tile_n 64, 2 at 128; at most one CTA per
 * k-block), 1 = no split, 0 = the launcher's choice (no split); tile_n 0 / 32
 * / 64 / 128. */
int vla_gemm_bf16_split(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                        int64_t N, int64_t K, const vla_epilogue* epi, int32_t tile_n, int32_t splits,
                        vla_stream_t stream);

/* Row normalisation over bf16 rows of width N (N % 8 == 0), fp32 statistics.
 * RMSNorm:  y = x * rsqrt(mean(x^2) + eps) * g
 *   replaces rms_norm_960_bf16 (cc/bf16/rms_norm_960_bf16.cc:60-62) and
 *   rms_norm_bf16 (cc/bf16_old/rms_norm_bf16.cc:16-64) with their tiling loop
 *   `rmsnorm` (vla/text_encoder_bf16.py:398-404).
 * LayerNorm: y = (x - mean) * rsqrt(var + eps) * g + b
 *   replaces layer_norm_bf16 + the bias-add region (cc/bf16_old/layer_norm_bf16.cc:16-70,
 *   vla/vision_block_bf16.py:89-127) and `layernorm` (vla/vision_block_bf16.py:272-280).
 * y may alias x. */
int vla_rms_norm_bf16(const void* x, int64_t ldx, const void* g, void* y, int64_t ldy, int64_t M, int64_t N, float eps,
                      vla_stream_t stream);
int vla_layer_norm_bf16(const void* x, int64_t ldx, const void* g, const void* b, void* y, int64_t ldy, int64_t M,
                        int64_t N, float eps, vla_stream_t stream);

/* In-place half-split RoPE on x [M, ld]: columns [0, ncols) are 64-wide heads,
 * row m has position m % seq; cs = fp32 [seq][64] (cos | sin) table (see
 * vla_rope_table).  Replaces rope_apply_packed (vla/text_encoder_bf16.py:422-475)
 * and the AIE RoPE/sin/cos kernels (cc/float/rope_vec_ops.cc:8-95,
 * cc/float/sine.cc:117, cc/float/cosine.cc:116). */
int vla_rope_bf16(void* x, int64_t ld, int64_t M, int32_t ncols, int32_t seq, const float* cs, vla_stream_t stream);

/* Host helper: fill cs[seq][head_dim] with cos(pos / ts_k) | sin(pos / ts_k),
 * ts_k = theta^(2k / head_dim), fp32 radians (vla/text_encoder_bf16.py:80-96). */
int vla_rope_table(float* cs_host, int32_t seq, int32_t head_dim, double theta);

/* Row softmax of x [M, N] (scores * scale), fp32 math, bf16 out.
 * causal_row_start < 0: unmasked — softmax_bf16_32_128 (cc/bf16_old/v2_softmax_bf16.cc:627-645),
 *   softmax_float32_seq1024 (cc/float/v1_softmax_float.cc:117-179);
 * causal_row_start >= 0: row r masks columns > causal_row_start + r, masked
 *   entries are written as 0 — masked_softmax_128_bf16(scores, row_start, out)
 *   (cc/bf16/masked_softmax_128_bf16.cc:251-398). */
int vla_softmax_bf16(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M, int64_t N, float scale,
                     int32_t causal_row_start, vla_stream_t stream);

/* Elementwise activations on [M, N] bf16, N % 8 == 0.
 * VLA_EW_GELU_TANH : gelu_bf16 (cc/bf16_old/gelu_bf16.cc:83-102)
 * VLA_EW_SILU      : silu_{128,160,256}_bf16 (cc/bf16/silu_160_bf16.cc:29-127)
 * VLA_EW_SILU_MUL  : silu(x) * y2 (vla/text_encoder_bf16.py:547-581)
 * VLA_EW_ADD       : x + y2 (cc/bf16_old/add_64_64_bf16.cc:12-49) */
enum { VLA_EW_GELU_TANH = 0, VLA_EW_SILU = 1, VLA_EW_SILU_MUL = 2, VLA_EW_ADD = 3 };
int vla_elementwise_bf16(int32_t op, const void* x, int64_t ldx, const void* y2, int64_t ldy2, void* out, int64_t ldo,
                         int64_t M, int64_t N, vla_stream_t stream);

/* Flash attention, head_dim 64: O = softmax(Q K^T * scale + mask) V per head.
 * Replaces the per-head score GEMM + softmax + P.V loops of the reference
 * blocks (vla/text_encoder_bf16.py:502-526, vla/vision_block_bf16.py:325-367,
 * vla/action_expert_bf16.py:690-713, 765-787).  Q rows are [seq, Hq*64] per
 * sequence (sequence b starts at q + b*q_batch), K/V [seq_k, Hkv*64]; query
 * head h reads KV head h*Hkv/Hq.  mask: causal (key > query masked) and/or
 * kv_len[b] (keys >= kv_len[b] masked).  Only scale == 1/8 (1/sqrt(64)) is
 * supported. */
typedef struct vla_attention_args {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t q_row, k_row, v_row, o_row;
  int64_t q_batch, k_batch, v_batch, o_batch;
  int32_t batch, Lq, Lk, Hq, Hkv, head_dim;
  int32_t causal;
  const int32_t* kv_len; /* device int32 [batch] or NULL */
  float scale;
  int32_t impl;          /* VLA_ATTN_AUTO, _MMA_SYNC, _TCGEN05 or _TCGEN05_SHORT */
} vla_attention_args;
/* Attention kernels: AUTO picks the tcgen05 kernel (persistent, 128-row query
 * tiles, TMEM accumulators) for non-causal attention with Lk >= 256, the
 * pipelined short-sequence tcgen05 kernel (TCGEN05_PIPE below) for Lk <= 128,
 * causal or not, when its shape limits hold, and the mma.sync kernel (64-row
 * tiles) otherwise.  TCGEN05_SHORT (all keys of a sequence in one tile, the
 * query heads of a kv head stacked into 128-row tiles, one item per CTA at a
 * time) is selectable explicitly.  TCGEN05 supports
 * non-causal attention only and needs q_batch / k_batch / v_batch to be whole
 * multiples of the row strides; TCGEN05_SHORT needs Lk <= 128.
 * TCGEN05_PIPE is the pipelined short-sequence kernel (one warp-specialised
 * CTA per SM, TMA loads and stores, per (sequence, kv head) items in flight
 * while earlier items compute): 1 <= Lk <= 128, Lq <= 256,
 * (Hq / Hkv) * Lq <= 512, and nonzero sequence strides when batch > 1. */
enum {
  VLA_ATTN_AUTO = 0,
  VLA_ATTN_MMA_SYNC = 1,
  VLA_ATTN_TCGEN05 = 2,
  VLA_ATTN_TCGEN05_SHORT = 3,
  VLA_ATTN_TCGEN05_PIPE = 4
};
int vla_attention_bf16(const vla_attention_args* a, vla_stream_t stream);

/* Pixel shuffle: in [B, grid*grid, C] -> out [B, (grid/s)^2, s*s*C] with
 * out[b, (h/s)*(grid/s) + w/s, (h%s)*s*C + (w%s)*C + c] = in[b, h*grid + w, c]
 * (con_ref, vla/vla.py:434-436; copy regions of fused_op, vla/connector_bf16.py:97-111). */
int vla_pixel_shuffle_bf16(const void* in, void* out, int32_t B, int32_t grid, int32_t scale, int32_t C,
                           vla_stream_t stream);

/* Patch im2col for a stride == kernel conv: img [B, Cin, H, W] bf16 ->
 * A [B*(H/p)*(W/p), Cin*p*p] (column = cin*p*p + ky*p + kx), the A operand of
 * the patch-embedding GEMM that replaces conv_bf16 (cc/bf16_old/conv_bf16.cc:12-55)
 * and its 14,592-call host loop (vla/preprocessing_bf16.py:86-103). */
int vla_patch_im2col_bf16(const void* img, void* out, int32_t B, int32_t Cin, int32_t H, int32_t W, int32_t p,
                          vla_stream_t stream);

/* Camera frames to model input: frames uint8 [B, H, W, 3] (row-major HWC, any
 * H and W), bilinear resize to S x S with half-pixel centres and no
 * antialiasing (torch F.interpolate(mode="bilinear", align_corners=False)),
 * scaled to [-1, 1] as v * 2/255 - 1, bf16 out:
 *   mode 0: out = image [B, 3, S, S] (NCHW, the input of vla_patch_im2col_bf16);
 *   mode 1: out = the patch-embedding GEMM's A operand [B * (S/p)^2, 3 p p]
 *           (column cin*p*p + ky*p + kx), i.e. resize + normalisation + im2col in
 *           one pass; p a multiple of 8 dividing S.
 * S must be a multiple of 8.  The reference feeds images that are already
 * 512 x 512 floats (preprocessing_block, vla/preprocessing_bf16.py:105-109;
 * vla/vla.py:318); this is the input side that turns camera frames into them,
 * so hosts ship 1 byte per pixel channel instead of 2. */
int vla_camera_preprocess_u8(const uint8_t* frames, int32_t B, int32_t H, int32_t W, int32_t S, int32_t p,
                             int32_t mode, void* out, vla_stream_t stream);

/* Camera of the closed-loop PushT demo (the reference renders it with
 * matplotlib, simulation/pusht_env.py:196-264): scene fp32 [n, 8] = end effector
 * x, y; block x, y, theta; target x, y, theta (512 x 512 workspace, y up) ->
 * frames uint8 [n, S, S, 3]: background, target T outline, block T, end
 * effector disc. */
int vla_pusht_render_u8(const float* scene, int32_t n, int32_t S, uint8_t* frames, vla_stream_t stream);

/* Token embedding gather: out[b*rows_per_seq + row_offset + t, :] =
 * table[ids[b*T + t], :] * scale (create_text_emb, vla/vla.py:169-174). */
int vla_embed_bf16(const int32_t* ids, const void* table, int32_t vocab, int32_t H, int32_t B, int32_t T, float scale,
                   void* out, int64_t ldo, int32_t rows_per_seq, int32_t row_offset, vla_stream_t stream);

/* y[M, N] bf16 = x[M, N] fp32 */
int vla_f32_to_bf16(const float* x, int64_t ldx, void* y, int64_t ldy, int64_t M, int64_t N, vla_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Block builders                                                          */
/* ---------------------------------------------------------------------- */

/* Weights of one Llama-style layer in the library's K-major layout.
 *   self layer : w_qkv = [Wq | Wk | Wv]^T, shape [(heads + 2 kv_heads) * 64, hidden]
 *   cross layer: w_qkv = Wq^T, shape [heads * 64, hidden]
 *   w_o    = Wo^T      [hidden, heads * 64]
 *   w_gu   = gate/up interleaved: rows [32j, 32j+16) = W_gate^T rows [16j, 16j+16),
 *            rows [32j+16, 32j+32) = W_up^T rows [16j, 16j+16); shape [2 ffn, hidden]
 *   w_down = W_down^T  [hidden, ffn]
 *   norm1 / norm2 = RMSNorm gains [hidden] */
typedef struct vla_llama_layer {
  const void* norm1;
  const void* w_qkv;
  const void* w_o;
  const void* norm2;
  const void* w_gu;
  const void* w_down;
  int32_t hidden, heads, kv_heads, head_dim, ffn;
  float eps;
} vla_llama_layer;

/* Workspace bytes for vla_llama_self_layer_bf16 (qkv_out given or not) and
 * vla_llama_cross_layer_bf16 over `rows` = batch * seq rows. */
size_t vla_llama_layer_workspace(const vla_llama_layer* w, int64_t rows, int32_t with_qkv);

/* x [batch*seq, hidden] bf16 updated in place by one causal self-attention
 * layer: RMSNorm -> QKV GEMM with RoPE epilogue -> flash attention -> O GEMM
 * + residual -> RMSNorm -> gate/up GEMM with SwiGLU epilogue -> down GEMM +
 * residual.  qkv_out (optional, [rows, (heads + 2 kv_heads)*64]) receives Q,
 * post-RoPE K and V; the K/V columns are what the action expert's cross
 * layers attend to.
 * Replaces text_encoder_forward (vla/text_encoder_bf16.py:480-595),
 * llama_block_rope (vla/llama_block_rope_bf16.py:519-615) and
 * action_expert_self_forward (vla/action_expert_bf16.py:662-728). */
int vla_llama_self_layer_bf16(const vla_llama_layer* w, void* x, int32_t batch, int32_t seq, const float* rope_cs,
                              void* qkv_out, void* workspace, size_t workspace_bytes, vla_stream_t stream);

/* Cross-attention layer: Q from x (RoPE on Q only), K/V given per sequence
 * ([kv_seq, ldkv] rows, already projected), optional key padding kv_len.
 * Replaces action_expert_cross_forward (vla/action_expert_bf16.py:731-803)
 * and llama_block_rope_cross (vla/llama_block_rope_bf16.py:617-709). */
int vla_llama_cross_layer_bf16(const vla_llama_layer* w, void* x, int32_t batch, int32_t seq, const float* rope_cs,
                               const void* k, const void* v, int64_t ldkv, int32_t kv_seq, const int32_t* kv_len,
                               void* workspace, size_t workspace_bytes, vla_stream_t stream);

/* Allocation-free variant of vla_llama_self_layer_bf16.  It has no
 * counterpart in the reference; it exists for callers that cannot allocate
 * device memory — a real-time control loop that must not call cudaMalloc
 * mid-episode, a host framework or plugin sandbox that owns every device
 * buffer and hands out only inputs and outputs, or an FFI binding with no
 * CUDA allocator of its own.  Such a caller passes x (and optionally
 * qkv_out) as before but no workspace: the layer's scratch lives in one
 * static device array of VLA_NOALLOC_SCRATCH_BYTES inside the library,
 * which every GPU that loads the library holds until the process exits.
 * - A request whose workspace would exceed that size is rejected with
 *   VLA_E_WORKSPACE before any launch (at the 960-wide text-layer shape the
 *   limit is 689 rows = batch * seq, or 936 rows when qkv_out is given).
 *   The call itself allocates nothing.
 * - The first call on each device looks up the array's device address
 *   (cudaGetSymbolAddress) with that device current; make that first call
 *   before any stream capture on the device.  The address is cached for the
 *   life of the process: after cudaDeviceReset on a device this entry point
 *   must not be called on that device again.
 * - All calls share the one array and it keeps the previous call's
 *   contents (nothing in it needs to start at zero).  Two calls whose
 *   kernels overlap on the GPU (different streams, or different host
 *   threads on one device) race on it: serialise them. */
#define VLA_NOALLOC_SCRATCH_BYTES (8u << 20)
size_t vla_noalloc_scratch_bytes(void);
int vla_llama_self_layer_bf16_noalloc(const vla_llama_layer* w, void* x, int32_t batch, int32_t seq,
                                      const float* rope_cs, void* qkv_out, vla_stream_t stream);

/* SigLIP encoder layer weights (K-major): w_qkv = [Wq | Wk | Wv]^T [3 hidden, hidden],
 * b_qkv [3 hidden], w_o [hidden, hidden], w_fc1 [ffn, hidden], w_fc2 [hidden, ffn]. */
typedef struct vla_vision_layer {
  const void* ln1_g;
  const void* ln1_b;
  const void* w_qkv;
  const void* b_qkv;
  const void* w_o;
  const void* b_o;
  const void* ln2_g;
  const void* ln2_b;
  const void* w_fc1;
  const void* b_fc1;
  const void* w_fc2;
  const void* b_fc2;
  int32_t hidden, heads, head_dim, ffn;
  float eps;
} vla_vision_layer;

size_t vla_vision_layer_workspace(const vla_vision_layer* w, int64_t rows);

/* x [batch*seq, hidden] updated in place: LayerNorm -> QKV GEMM + bias ->
 * non-causal flash attention -> O GEMM + bias + residual -> LayerNorm -> fc1
 * GEMM + bias + GELU-tanh -> fc2 GEMM + bias + residual.
 * Replaces vision_block (vla/vision_block_bf16.py:308-420). */
int vla_vision_layer_bf16(const vla_vision_layer* w, void* x, int32_t batch, int32_t seq, void* workspace,
                          size_t workspace_bytes, vla_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* VLA_B200_H */
