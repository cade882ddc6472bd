// libvla_b200.so — single translation unit holding every sm_100a kernel of
// the SmolVLA hot path and the extern "C" entry points declared in
// include/vla_b200.h.  One TU keeps the device error word in one place.
#include "gemm_host.cuh"
#include "host_common.cuh"

using namespace vla;

extern "C" {

const char* vla_last_error(void) { return t_last_error; }

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

int vla_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M, int64_t N,
                  int64_t K, const vla_epilogue* epi, vla_stream_t stream) {
  return gemm::run(A, lda, B, ldb, C, ldc, M, N, K, epi, as_stream(stream));
}

int vla_gemm_bf16_tiled(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                        int64_t N, int64_t K, const vla_epilogue* epi, int tile_n, vla_stream_t stream) {
  VLA_CHECK_ARG(tile_n == 32 || tile_n == 64 || tile_n == 128 || tile_n == 256, "tile_n must be 32/64/128/256");
  return gemm::run(A, lda, B, ldb, C, ldc, M, N, K, epi, as_stream(stream), tile_n);
}

}  // extern "C"
