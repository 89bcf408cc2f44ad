/*
 * sdpa_b200 -- C ABI of the Blackwell (sm_100a) scaled-dot-product attention
 * forward / backward behind the reference's TensorFlow ops `Sdpa` and
 * `SdpaGrad`.
 *
 * The entry points replace the reference's device-functor seam:
 *   sdpa_b200_fwd  <- functor::FlashAttnFunctor<GPUDevice,T>::operator()
 *                     (sdpa/sdpa.h:11-17, sdpa/sdpa_fwd.cu.cc:176-240),
 *                     called from SdpaFwdOp::Compute (sdpa/sdpa_cpu.cc:84-86)
 *   sdpa_b200_bwd  <- functor::FlashAttnGradFunctor<GPUDevice,T>::operator()
 *                     (sdpa/sdpa.h:19-33, sdpa/sdpa_bwd.cu.cc:347-453),
 *                     called from SdpaBwdOp::Compute (sdpa/sdpa_cpu.cc:188-191)
 *
 * Conventions
 *   - Tensors are dense row-major [B, S, D] (B = batch x heads folded),
 *     device pointers; stats is float32 [B, S_q] in natural-log units:
 *     stats = max_j(scale*q.k_j) + ln(sum_j exp(scale*q.k_j - max) + 1e-6).
 *   - dtype: SDPA_B200_F16 (IEEE half) or SDPA_B200_F32.
 *   - Dropout: element (b,i,j) is dropped iff hi32(LCG(seed + offset +
 *     (b*S_q + i)*S_kv + j)) / 2^32 < dropout, enabled iff dropout > 1e-6
 *     (sdpa/sdpa_utils.cuh:13-19, sdpa/sdpa_fwd.cu.cc:136).  Kept
 *     probabilities are scaled by 1/(1 - dropout).
 *   - causal != 0 masks j > i and requires S_q == S_kv.
 *   - Every call is asynchronous on `stream` (a cudaStream_t; NULL = legacy
 *     default stream), never allocates, frees or synchronises, and is
 *     reentrant.  The caller owns every buffer.
 *   - Return value: SDPA_B200_OK or an error code; sdpa_b200_strerror() gives
 *     text.  Errors never abort the process.
 */
#ifndef SDPA_B200_H_
#define SDPA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum sdpa_b200_dtype { SDPA_B200_F16 = 0, SDPA_B200_F32 = 1 };

enum sdpa_b200_status {
  SDPA_B200_OK = 0,
  SDPA_B200_EINVAL = 1,       /* bad shape, dtype, pointer or argument        */
  SDPA_B200_EUNSUPPORTED = 2, /* max(D_qk, D_v) > 128                          */
  SDPA_B200_ECUDA = 3,        /* a CUDA runtime / launch error                 */
  SDPA_B200_ETIMEOUT = 4,     /* a device-side wait gave up (see status word)  */
  SDPA_B200_EWORKSPACE = 5,   /* workspace missing or too small                */
  SDPA_B200_ESCRATCH = 6      /* problem too large for the built-in scratch    */
};

/* Forward: out [B,S_q,D_v] (dtype), stats [B,S_q] float32.
 * Replaces FlashAttnFunctor<GPUDevice,T> (sdpa/sdpa_fwd.cu.cc:176-240). */
int sdpa_b200_fwd(int dtype, const void* q, const void* k, const void* v, void* out, float* stats, int64_t B,
                  int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout, int causal,
                  uint64_t seed, uint64_t offset, void* stream);

/* Scratch the backward asks for (the caller allocates it; TF: allocate_temp):
 * one float32 per query row (rowsum(dO*O)), which is also the minimum
 * sdpa_b200_bwd accepts; for fp32 (rows of 16-byte multiples) also room for
 * dS and the dropout-scaled P, about 4*B*S_q*S_kv bytes each, which selects
 * the faster GEMM route of the backward.  That part is capped at 4 GiB: past
 * it the query asks for the batch rows that fit, and the backward runs in
 * chunks of that many rows (of as many as any workspace given holds). */
size_t sdpa_b200_bwd_workspace_bytes(int dtype, int64_t B, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v);

/* Backward: dq, dk, dv shaped like q, k, v (dtype), from q, k, v, out, stats
 * and d_out of the forward, no atomics: fp16 runs two kernels, dQ (which
 * also writes rowsum(dO*O) to the workspace) then dK/dV; fp32 runs on the
 * 3xTF32 tensor-core path, with the full workspace as five kernels (rowsum,
 * a score pass writing dS and the dropout-scaled P, then dQ, dK and dV as
 * GEMMs), with the minimum as three recomputing passes (dQ, dK, dV).
 * Replaces FlashAttnGradFunctor<GPUDevice,T> (sdpa/sdpa_bwd.cu.cc:347-453). */
int sdpa_b200_bwd(int dtype, const void* q, const void* k, const void* v, const void* out, const float* stats,
                  const void* d_out, void* dq, void* dk, void* dv, int64_t B, int64_t S_q, int64_t S_kv, int64_t D_qk,
                  int64_t D_v, float scale, float dropout, int causal, uint64_t seed, uint64_t offset,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Backward that also propagates a gradient d_stats [B,S_q] (float32, device)
 * reaching the stats output: stats is the row log-sum-exp, so it adds
 * d_stats_i * p_ij to dS_ij.  No counterpart in the reference (its gradient
 * registration drops it, mha.py:10-21); d_stats = NULL equals sdpa_b200_bwd. */
int sdpa_b200_bwd_dstats(int dtype, const void* q, const void* k, const void* v, const void* out, const float* stats,
                         const float* d_stats, const void* d_out, void* dq, void* dk, void* dv, int64_t B, int64_t S_q,
                         int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout, int causal, uint64_t seed,
                         uint64_t offset, void* workspace, size_t workspace_bytes, void* stream);

/* Head-strided layout for the multi-head layer: q [B,S_q,H,D_qk], k
 * [B,S_kv,H,D_qk], v [B,S_kv,H,D_v], out / d_out [B,S_q,H,D_v] and dq, dk, dv
 * shaped like q, k, v, read and written in place (no transposes); stats,
 * d_stats and the workspace are [B,H,S_q] (workspace bytes as for B*H rows).
 * Results equal sdpa_b200_fwd / _bwd_dstats on the [B*H,S,D] tensors that the
 * reference's MHA builds by transposing (sdpa/mha.py:103-129, heads innermost
 * in the folded batch index, which is also the dropout counter's).  No
 * counterpart in the reference, whose op takes only [B,S,D]. */
int sdpa_b200_fwd_bshd(int dtype, const void* q, const void* k, const void* v, void* out, float* stats, int64_t B,
                       int64_t H, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout,
                       int causal, uint64_t seed, uint64_t offset, void* stream);
int sdpa_b200_bwd_bshd(int dtype, const void* q, const void* k, const void* v, const void* out, const float* stats,
                       const float* d_stats, const void* d_out, void* dq, void* dk, void* dv, int64_t B, int64_t H,
                       int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout, int causal,
                       uint64_t seed, uint64_t offset, void* workspace, size_t workspace_bytes, void* stream);

/* What the last SDPA_B200_ECUDA returned on the calling thread came from (the
 * CUDA error name, or the TMA descriptor encode result); "" before any.
 * Diagnostic, no reference counterpart. */
const char* sdpa_b200_last_error_detail(void);

/* Writes mask[b][i][j] = 1 where (b,i,j) is dropped, from the same device RNG
 * routine the kernels use (diagnostic; no reference counterpart beyond the
 * RNG of sdpa/sdpa_utils.cuh:13-19).  mask is a device uint8 [B,S_q,S_kv]. */
int sdpa_b200_dropout_mask(uint64_t seed, uint64_t offset, int64_t B, int64_t S_q, int64_t S_kv, float dropout,
                           uint8_t* mask, void* stream);

/* Text for a status code. */
const char* sdpa_b200_strerror(int status);

/* Device status word of the current device: bit 0 = a bounded wait timed out
 * inside a kernel.  Synchronises `stream`, reads the word and clears it. */
int sdpa_b200_device_status(unsigned int* word, void* stream);

/* Bound (nanoseconds) of every device-side wait; 0 restores the default (2 s). */
void sdpa_b200_set_wait_timeout_ns(uint64_t ns);

/* Diagnostic: launches one CTA that waits on an mbarrier nothing arrives at,
 * bounded by timeout_ns; the wait gives up and raises bit 0 of the status
 * word.  Used to test timeout handling without faulting the GPU. */
int sdpa_b200_test_wait_timeout(uint64_t timeout_ns, void* stream);

/* Which kernel family serves a shape: 1 = fp16 tcgen05 tensor-core kernels,
 * 2 = fp32 3xTF32 tcgen05 kernels, 0 = SIMT kernels (rows that are not
 * 16-byte multiples, fp16 D_qk < 16, or forced by SDPA_B200_FORCE_SIMT=1).
 * For a backward given the workspace sdpa_b200_bwd_workspace_bytes asks for
 * (with less, the fp32 backward with D_qk > 64 runs on SIMT). */
int sdpa_b200_path(int dtype, int64_t D_qk, int64_t D_v, int backward);

/* Number of kernel launches the last successful fwd/bwd call on this thread made. */
int sdpa_b200_last_launch_count(void);

/* Backward for callers that cannot allocate device memory.
 * No counterpart in the reference.  Same arguments and results as
 * sdpa_b200_bwd, but without a workspace: the per-row scratch
 * (rowsum(dO*O), one float per query row) lives in a fixed array of
 * SDPA_B200_NOALLOC_MAX_ROWS floats (4 MiB) built into the library, which
 * every GPU that loads the library keeps until the process exits.
 *   - Meant for hosts such as a framework's memory-planned executor, a
 *     real-time or embedded runtime, or code running where cudaMalloc is
 *     forbidden or would stall; nothing here calls cudaMalloc, cudaFree or
 *     any allocating routine.
 *   - B * S_q must not exceed SDPA_B200_NOALLOC_MAX_ROWS; larger problems
 *     return SDPA_B200_ESCRATCH and launch nothing.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress with that device current); make that first call
 *     before any stream capture.
 *   - All calls share the one array and it keeps the last call's contents
 *     (every row used is rewritten before it is read, so nothing needs to
 *     start at zero).  Calls whose kernels overlap on the GPU -- different
 *     streams, or different host threads, on the same device -- race on it:
 *     order them on one stream or serialise them. */
#define SDPA_B200_NOALLOC_MAX_ROWS (1 << 20)
int sdpa_b200_bwd_noalloc(int dtype, const void* q, const void* k, const void* v, const void* out,
                          const float* stats, const void* d_out, void* dq, void* dk, void* dv, int64_t B,
                          int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout,
                          int causal, uint64_t seed, uint64_t offset, void* stream);

/* Diagnostic: when events != NULL, the next tensor-core backward calls on
 * this host thread record events[0..n-1] (cudaEvent_t, 4 <= n <= 8) on their
 * stream between their launches, so a caller can time each kernel:
 *   fp16: [0] dQ (+ rowsum D) [1] dK/dV [2], [3] = [2];
 *   fp32 passes: [0] dQ [1] dK [2] dV [3];
 *   fp32 GEMM route: [0] D + score pass [1] dQ GEMM [2] dK GEMM [3] dV GEMM [4]
 *   (with n = 4 the last interval is not recorded).
 * NULL turns it off. */
int sdpa_b200_set_bwd_events(void* const* events, int n);

/* ABI version (major*100 + minor). */
int sdpa_b200_version(void);

#ifdef __cplusplus
}
#endif
#endif /* SDPA_B200_H_ */
