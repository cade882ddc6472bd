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
  int32_t reserved[4];
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

#ifdef __cplusplus
}
#endif
#endif /* VLA_B200_H */
