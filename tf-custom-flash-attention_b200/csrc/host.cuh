// Host-side helpers shared by the translation units of the library.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
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

// [B, S, D] fp16 tensor, box = 64 columns x `rows` rows x 1 batch, 128B swizzle.
// Columns beyond D and rows beyond S read as zero.
inline bool make_map_f16(CUtensorMap* m, const void* base, int64_t B, int64_t S, int64_t D, int rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D * 2), static_cast<cuuint64_t>(S * D * 2)};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
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

inline int launch_result() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SDPA_B200_OK : SDPA_B200_ECUDA;
}

}  // namespace host

// Optional events recorded between the backward's launches (diagnostic).
extern thread_local void* const* t_bwd_events;
inline void record_bwd_event(int i, cudaStream_t st) {
  if (t_bwd_events) cudaEventRecord(static_cast<cudaEvent_t>(t_bwd_events[i]), st);
}

// Launchers, one per translation unit (launch count added to *launches).
int launch_fwd_tc(const Params& p, cudaStream_t st, int* launches);
int launch_bwd_tc(const Params& p, cudaStream_t st, int* launches);
int launch_fwd_simt_f16(const Params& p, cudaStream_t st, int* launches);
int launch_fwd_simt_f32(const Params& p, cudaStream_t st, int* launches);
int launch_bwd_simt_f16(const Params& p, cudaStream_t st, int* launches);
int launch_bwd_simt_f32(const Params& p, cudaStream_t st, int* launches);
// Reads and clears the status word of each translation unit's kernels.
int status_exchange_fwd_tc(unsigned int* w);
int status_exchange_bwd_tc(unsigned int* w);
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
