// Host-side helpers shared by the translation units of the library.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <utility>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/sdpa_b200.h"
#include "common.cuh"

namespace sdpa_b200 {
namespace host {

inline int dmax_bucket(int64_t d) {
  if (d <= 8) return 8;
  if (d <= 16) return 16;
  if (d <= 32) return 32;
  if (d <= 64) return 64;
  return 128;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Detail of the last SDPA_B200_ECUDA returned on this thread (sdpa_b200_last_error_detail).
inline thread_local char t_err_detail[160] = "";
inline int cuda_failure(const char* what, int code, const char* name) {
  std::snprintf(t_err_detail, sizeof(t_err_detail), "%s: %s (%d)", what, name ? name : "?", code);
  return SDPA_B200_ECUDA;
}
inline int cuda_failure(const char* what, cudaError_t e) {
  return cuda_failure(what, static_cast<int>(e), cudaGetErrorName(e));
}
inline bool map_failure(int code, const char* name) {
  cuda_failure("TMA descriptor", code, name);
  return false;
}

// ---------------------------------------------------------------- TMA maps
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Tensor [B/H, S, H, D] of `esize`-byte elements as a 4-D map over (column,
// head, row, outer batch), box = one 128-byte row segment (64 halves or 32
// floats) x 1 head x `rows` rows x 1; for H = 1 (contiguous [B, S, D]) the 3-D
// map (column, row, batch), box 128 B x `rows` x 1.  128B swizzle by default;
// the shared-memory tile is the same either way.  Columns beyond D and rows
// beyond S read as zero.  Failures record their detail.
inline bool make_map(CUtensorMap* m, CUtensorMapDataType dtype, int esize, const void* base, int64_t B, int64_t H,
                     int64_t S, int64_t D, int rows, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (!fn) return map_failure(0, "cuTensorMapEncodeTiled unavailable");
  if (H < 1 || B % H != 0) return map_failure(static_cast<int>(H), "bad head count");
  const cuuint32_t inner = static_cast<cuuint32_t>(128 / esize);
  const cuuint64_t es = static_cast<cuuint64_t>(esize);
  if (H == 1) {  // contiguous [B, S, D]: the 3-D map (column, row, batch)
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * es, static_cast<cuuint64_t>(S * D) * es};
    cuuint32_t box[3] = {inner, static_cast<cuuint32_t>(rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(m, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS || map_failure(static_cast<int>(r), "cuTensorMapEncodeTiled");
  }
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(S),
                        static_cast<cuuint64_t>(B / H)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(D) * es, static_cast<cuuint64_t>(H * D) * es,
                           static_cast<cuuint64_t>(S * H * D) * es};
  cuuint32_t box[4] = {inner, 1, static_cast<cuuint32_t>(rows), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, dtype, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS || map_failure(static_cast<int>(r), "cuTensorMapEncodeTiled");
}
inline bool make_map_f16(CUtensorMap* m, const void* base, int64_t B, int64_t H, int64_t S, int64_t D, int rows) {
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, B, H, S, D, rows);
}
inline bool make_map_f32(CUtensorMap* m, const void* base, int64_t B, int64_t H, int64_t S, int64_t D, int rows) {
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, B, H, S, D, rows);
}
// fp32 tiles read only as MN-major tf32 operands (32-byte swizzle atoms).
inline bool make_map_f32_mn(CUtensorMap* m, const void* base, int64_t B, int64_t H, int64_t S, int64_t D, int rows) {
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, B, H, S, D, rows, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

// fp32 matrices [B, M, ld] (row length K <= ld, ld a multiple of 4) as the
// 3-D map (column, row, batch), box 32 columns x `rows` rows, 128B swizzle
// (or its 32-byte-atom form for MN-major reads); columns beyond K and rows
// beyond M read as zero.
inline bool make_map_rows_f32(CUtensorMap* m, const float* base, int64_t B, int64_t M, int64_t K, int64_t ld,
                              int rows, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (!fn) return map_failure(0, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 4, static_cast<cuuint64_t>(M * ld) * 4};
  cuuint32_t box[3] = {32, static_cast<cuuint32_t>(rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS || map_failure(static_cast<int>(r), "cuTensorMapEncodeTiled");
}

// Opt a kernel into more than 48 KB of dynamic shared memory, once per device.
template <typename K>
inline cudaError_t ensure_smem(K kernel, size_t bytes, std::atomic<uint64_t>& done_mask) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done_mask.load() & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess) done_mask.fetch_or(bit);
  return e;
}

// SM count of the current device (cached per device ordinal), for persistent grids.
inline int num_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int v = cache[dev & 63].load();
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev & 63].store(v);
  }
  return v;
}

// Launches a tensor-core kernel with programmatic stream serialisation: its
// CTAs may start (and set up barriers and TMEM) while the previous kernel on
// the stream finishes; the kernel waits (griddepcontrol.wait) before touching
// global memory.  SDPA_B200_PDL=0 turns it off (plain stream order).
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("SDPA_B200_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}
template <typename... KArgs, typename... Args>
inline int launch_tc(void (*kern)(KArgs...), int64_t grid, int threads, size_t smem, cudaStream_t st,
                     Args&&... args) {
  if (grid <= 0 || grid > 0x7fffffffLL) return SDPA_B200_EINVAL;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  return e == cudaSuccess ? SDPA_B200_OK : cuda_failure("kernel launch", e);
}

inline int launch_result() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SDPA_B200_OK : cuda_failure("kernel launch", e);
}

}  // namespace host

// Optional events recorded between the backward's launches (diagnostic).
extern thread_local void* const* t_bwd_events;
inline void record_bwd_event(int i, cudaStream_t st) {
  if (t_bwd_events && i < 8 && t_bwd_events[i]) cudaEventRecord(static_cast<cudaEvent_t>(t_bwd_events[i]), st);
}

// Launchers, one per translation unit (launch count added to *launches).
int launch_fwd_tc(const Params& p, cudaStream_t st, int* launches);
int launch_bwd_tc(const Params& p, cudaStream_t st, int* launches);
int launch_fwd_tf32(const Params& p, cudaStream_t st, int* launches);
int launch_bwd_tf32(const Params& p, cudaStream_t st, int* launches);
int launch_fwd_simt_f16(const Params& p, cudaStream_t st, int* launches);
int launch_fwd_simt_f32(const Params& p, cudaStream_t st, int* launches);
int launch_bwd_simt_f16(const Params& p, cudaStream_t st, int* launches);
int launch_bwd_simt_f32(const Params& p, cudaStream_t st, int* launches);
// Reads and clears the status word of each translation unit's kernels.
int status_exchange_fwd_tc(unsigned int* w);
int status_exchange_bwd_tc(unsigned int* w);
int status_exchange_tf32(unsigned int* w);
int status_exchange_simt_fwd_f16(unsigned int* w);
int status_exchange_simt_fwd_f32(unsigned int* w);
int status_exchange_simt_bwd_f16(unsigned int* w);
int status_exchange_simt_bwd_f32(unsigned int* w);

}  // namespace sdpa_b200

// Defines status_exchange_<NAME> for the g_status_word of the including TU.
#define SDPA_B200_STATUS_EXCHANGE(NAME)                                              \
  int sdpa_b200::status_exchange_##NAME(unsigned int* w) {                           \
    unsigned int v = 0, zero = 0;                                                    \
    if (cudaMemcpyFromSymbol(&v, g_status_word, sizeof(v)) != cudaSuccess) return 1; \
    if (cudaMemcpyToSymbol(g_status_word, &zero, sizeof(zero)) != cudaSuccess)      \
      return 1;                                                                      \
    *w |= v;                                                                         \
    return 0;                                                                        \
  }
