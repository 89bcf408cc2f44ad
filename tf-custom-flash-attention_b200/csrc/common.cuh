// Parameters shared by every kernel of the library.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace sdpa_b200 {

constexpr float kEps = 1e-6f;        // sdpa/sdpa_utils.cuh:9
constexpr float kNegInit = -1e9f;    // initial running max, sdpa/sdpa_utils.cuh:11
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct Params {
  // inputs
  const void* q;
  const void* k;
  const void* v;
  const void* o;        // backward: forward output
  const void* d_o;      // backward: gradient of the output
  const float* lse;     // backward: stats of the forward (natural log)
  float* delta;         // backward workspace: rowsum(dO*O) - d_stats, [B*S_q]
  const float* d_stats; // backward: gradient reaching stats (nullptr = none)
  // outputs
  void* out;
  float* stats;
  void* dq;
  void* dk;
  void* dv;
  // shape: B folded batch rows bh = b*H + h; every [.., S, D] tensor except
  // stats/delta is laid out [B/H, S, H, D] (H = 1: contiguous [B, S, D])
  int64_t B, S_q, S_kv;
  int64_t H;
  int D_qk, D_v;
  // semantics
  float scale;          // as given
  float scale_log2;     // scale * log2(e)
  int causal;
  int dropout_on;       // dropout > 1e-6
  float dp_inv;         // 1 / (1 - dropout) (1 when off)
  float dp_keep;        // 1 / dp_inv  ( = 1 - dropout in fp32, as D_i / dp_inverse)
  uint64_t drop_thr;    // dropped iff hi32(state) < drop_thr
  uint64_t rng_base;    // seed + offset
  uint64_t timeout_ns;
  uint32_t one;         // 1: an opaque multiplier for lcg_hi_at
  // fp32 backward with materialised gradients (workspace beyond delta, else
  // null): dS and P~ = dropout-scaled P, both [B, S_q, ld_k]
  float* ws_ds;
  float* ws_p;
  int64_t ld_k;
  int64_t ws_rows;      // batch rows the workspace holds (< B: the backward runs in batch chunks)
  // fp32 forward: tiles per output fold segment, in units of the kernel's own
  // segment (default 2; SDPA_B200_TF32_FOLD, a tuning knob)
  int tf32_fold;
};

// CTA order of the tensor-core kernels over (batch row b, tile t): groups of
// kRasterRows batch rows, tile-major within a group, so that the CTAs resident
// at the same time share batch rows and the operand they all stream (K/V or
// Q/dO of the row) comes from L2 rather than HBM; tile order 0 is the
// heaviest causal tile, so each group still issues heavy tiles first.
#ifndef SDPA_B200_RASTER_ROWS
#define SDPA_B200_RASTER_ROWS 16
#endif
constexpr int kRasterRows = SDPA_B200_RASTER_ROWS;
__device__ __forceinline__ void raster(int64_t idx, int64_t B, int64_t ntiles, int64_t& b, int64_t& t) {
  const int64_t per = kRasterRows * ntiles;
  const int64_t g = idx / per;
  const int64_t rows = B - g * kRasterRows < kRasterRows ? B - g * kRasterRows : kRasterRows;
  const int64_t w = idx - g * per;
  t = w / rows;
  b = g * kRasterRows + (w - t * rows);
}

// Element offset of row s of folded batch row bh in a [B/H, S, H, D] tensor.
__host__ __device__ __forceinline__ int64_t row_offset(int64_t H, int64_t bh, int64_t s, int64_t S, int64_t D) {
  if (H == 1) return (bh * S + s) * D;  // contiguous [B, S, D]: no division
  return ((bh / H) * S + s) * (H * D) + (bh % H) * D;
}
// The same with the layout fixed at compile time (HEADS = false: H is 1).
template <bool HEADS>
__host__ __device__ __forceinline__ int64_t row_offset_t(int64_t H, int64_t bh, int64_t s, int64_t S, int64_t D) {
  return HEADS ? ((bh / H) * S + s) * (H * D) + (bh % H) * D : (bh * S + s) * D;
}

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) {
  return x;
}
template <>
__device__ __forceinline__ float to_f<__half>(__half x) {
  return __half2float(x);
}
template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) {
  return x;
}
template <>
__device__ __forceinline__ __half from_f<__half>(float x) {
  return __float2half_rn(x);
}

}  // namespace sdpa_b200
