// Host-side plumbing shared by every C-ABI entry point: thread-local error
// text, argument checks, device properties, and TMA tensor-map encoding
// through the driver entry point (no link-time dependency on libcuda).
#pragma once
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "vla_b200.h"

namespace vla {

static thread_local char t_last_error[512] = "";

static int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

#define VLA_CHECK_ARG(cond, ...) \
  do {                           \
    if (!(cond)) return ::vla::set_error(VLA_E_INVALID, __VA_ARGS__); \
  } while (0)

#define VLA_CHECK_ALIGN(cond, ...) \
  do {                             \
    if (!(cond)) return ::vla::set_error(VLA_E_ALIGN, __VA_ARGS__); \
  } while (0)

#define VLA_CUDA_TRY(expr)                                                                               \
  do {                                                                                                   \
    cudaError_t _e = (expr);                                                                             \
    if (_e != cudaSuccess) return ::vla::set_error(VLA_E_CUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct DeviceInfo {
  int num_sms = 0;
  int max_smem_optin = 0;
};

static DeviceInfo& device_info() {
  static DeviceInfo info[64];
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  std::call_once(once[dev], [dev]() {
    cudaDeviceGetAttribute(&info[dev].num_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&info[dev].max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (info[dev].num_sms <= 0) info[dev].num_sms = 148;
  });
  return info[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major [outer, inner] matrix with row stride
// ld (elements); box = [box_outer rows, box_inner cols]; 128-byte swizzle.
// Out-of-range boxes are zero-filled by the TMA unit.
static int make_tmap_bf16_2d(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                             uint32_t box_inner, uint32_t box_outer,
                             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto enc = tmap_encoder();
  if (enc == nullptr) return set_error(VLA_E_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(VLA_E_CUDA, "cuTensorMapEncodeTiled failed (%d): inner=%llu outer=%llu ld=%llu box=%ux%u", (int)r,
                     (unsigned long long)inner, (unsigned long long)outer, (unsigned long long)ld, box_inner,
                     box_outer);
  return VLA_OK;
}

// K-slab view of a row-major [outer, inner] bf16 matrix: dimensions (64
// columns, outer rows, inner / 64 whole k-blocks), strides (ld * 2 bytes, 128
// bytes), box (64, box_outer, box_kb), 128-byte swizzle.  One box is box_kb
// consecutive (box_outer x 128-byte) k-block tiles.  Columns past the last
// whole k-block are not covered (the two-dimensional map serves them).
static int make_tmap_bf16_kslab(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                                uint32_t box_outer, uint32_t box_kb) {
  auto enc = tmap_encoder();
  if (enc == nullptr) return set_error(VLA_E_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[3] = {64, outer, inner / 64};
  cuuint64_t strides[2] = {ld * 2, 128};
  cuuint32_t box[3] = {64, box_outer, box_kb};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(VLA_E_CUDA, "cuTensorMapEncodeTiled (k-slab) failed (%d): inner=%llu outer=%llu ld=%llu", (int)r,
                     (unsigned long long)inner, (unsigned long long)outer, (unsigned long long)ld);
  return VLA_OK;
}

// Launch overlap (programmatic dependent launch) for every kernel of this
// library; on by default, switchable with vla_set_launch_overlap().
static std::atomic<int> g_launch_overlap{1};

template <typename... KArgs, typename... Args>
static void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_launch_overlap.load(std::memory_order_relaxed) ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Same, for a kernel launched in clusters of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
static void launch_k_cluster(void (*kernel)(KArgs...), int cluster_x, dim3 grid, dim3 block, size_t smem,
                             cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_launch_overlap.load(std::memory_order_relaxed) ? 2 : 1;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

static inline cudaStream_t as_stream(vla_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of kernels this library has launched in this process.
static std::atomic<unsigned long long> g_launch_count{0};

// ---------------------------------------------------------------------------
// Launch profiler: when enabled (never during graph capture), every launch is
// bracketed by a CUDA event pair and tagged with its kind and algorithmic
// FLOPs / bytes, so a caller can compute per-kernel roofline fractions.
// ---------------------------------------------------------------------------
struct ProfRec {
  int kind;
  double flops, bytes;
  cudaEvent_t a, b;
  int64_t m, n, k;
  int tile_n, ctas;
};
struct Profiler {
  bool on = false;
  std::vector<cudaEvent_t> pool;
  std::vector<ProfRec> recs;
  size_t next = 0;
  cudaEvent_t pending = nullptr;
};
static Profiler g_prof;

static inline void prof_begin(cudaStream_t st) {
  if (!g_prof.on || g_prof.next + 2 > g_prof.pool.size()) return;
  g_prof.pending = g_prof.pool[g_prof.next++];
  cudaEventRecord(g_prof.pending, st);
}
static inline void prof_end(cudaStream_t st, int kind, double flops, double bytes, int64_t m = 0, int64_t n = 0,
                            int64_t k = 0, int tile_n = 0, int ctas = 0) {
  if (!g_prof.on || g_prof.pending == nullptr || g_prof.next + 1 > g_prof.pool.size()) return;
  cudaEvent_t e = g_prof.pool[g_prof.next++];
  cudaEventRecord(e, st);
  g_prof.recs.push_back(ProfRec{kind, flops, bytes, g_prof.pending, e, m, n, k, tile_n, ctas});
  g_prof.pending = nullptr;
}

static int launch_status(const char* what) {
  g_launch_count.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(VLA_E_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return VLA_OK;
}

}  // namespace vla
