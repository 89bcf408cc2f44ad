// C ABI of the library (declared in include/sdpa_b200.h): argument checks,
// TMA descriptors, kernel selection and launches.  Never allocates, frees or
// synchronises (except sdpa_b200_device_status, which is documented to).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "host.cuh"
#include "ptx.cuh"

using namespace sdpa_b200;
using namespace sdpa_b200::host;

thread_local void* const* sdpa_b200::t_bwd_events = nullptr;

namespace {

constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;
std::atomic<uint64_t> g_timeout_ns{kDefaultTimeoutNs};
thread_local int t_launches = 0;
thread_local void* t_bwd_event_store[8];  // copy of the caller's events

// The TMA descriptors are encoded through the driver API, which needs a
// current context on the calling thread.  A thread that has made no runtime
// call yet (e.g. an autograd worker whose device guard saw the device already
// selected) has none: cudaSetDevice binds the device's primary context.
int bind_context() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaSetDevice(dev);
  return e == cudaSuccess ? SDPA_B200_OK : cuda_failure("binding the device context", e);
}

bool force_simt() {
  const char* e = std::getenv("SDPA_B200_FORCE_SIMT");
  return e && e[0] == '1';
}

// dropped iff hi32(state) < thr  <=>  (float)hi32 / 2^32 < rate, exactly:
// float(u32) is monotone, so the dropped set is a prefix [0, thr).
uint64_t drop_threshold(float rate) {
  uint64_t lo = 0, hi = 1ull << 32;
  while (lo < hi) {
    const uint64_t mid = (lo + hi) / 2;
    const bool drop = static_cast<float>(static_cast<uint32_t>(mid)) / 4294967296.0f < rate;
    if (mid < (1ull << 32) && drop)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

Params make_params(int64_t B, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout,
                   int causal, uint64_t seed, uint64_t offset) {
  Params p;
  std::memset(&p, 0, sizeof(p));
  p.B = B;
  p.H = 1;
  p.S_q = S_q;
  p.S_kv = S_kv;
  p.D_qk = static_cast<int>(D_qk);
  p.D_v = static_cast<int>(D_v);
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  p.causal = causal ? 1 : 0;
  p.dropout_on = dropout > kEps ? 1 : 0;
  p.dp_inv = p.dropout_on ? 1.0f / (1.0f - dropout) : 1.0f;
  p.dp_keep = 1.0f / p.dp_inv;
  p.drop_thr = p.dropout_on ? drop_threshold(dropout) : 0;
  p.rng_base = seed + offset;
  p.one = 1;
  p.timeout_ns = g_timeout_ns.load();
  // 2: |O| error vs the oracle 4.0e-6 / 4.9e-6 / 4.9e-6 of max at S_kv = 4096 /
  // 8192 / 16384 (against 3.8 / 4.2 / 4.9 with 1, 6.3-6.9 with 8), forward +3 %
  static const int fold = [] {
    const char* e = std::getenv("SDPA_B200_TF32_FOLD");
    const int v = e ? std::atoi(e) : 2;
    return v >= 1 && v <= 64 ? v : 2;
  }();
  p.tf32_fold = fold;
  return p;
}

int check_common(int dtype, int64_t B, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, int causal) {
  if (dtype != SDPA_B200_F16 && dtype != SDPA_B200_F32) return SDPA_B200_EINVAL;
  if (B < 0 || S_q < 0 || S_kv < 0 || D_qk < 1 || D_v < 1) return SDPA_B200_EINVAL;
  if (D_qk > 128 || D_v > 128) return SDPA_B200_EUNSUPPORTED;
  if (causal && S_q != S_kv) return SDPA_B200_EINVAL;
  if (B > 0x7fffffffLL || S_q > 0x7fffffffLL || S_kv > 0x7fffffffLL) return SDPA_B200_EINVAL;
  return SDPA_B200_OK;
}

// fp16 scores over fewer than 16 dims stay on the SIMT kernels, which round
// each q*k product to half before summing as the reference does: over so few
// terms that rounding is a visible part of its result (a sweep of random
// shapes found D_qk = 8 on the tensor cores 2.2e-3 of max from the reference).
bool tc_fwd_ok(int dtype, int64_t S_kv, int64_t D_qk, int64_t D_v, const void* q, const void* k, const void* v,
               const void* o) {
  if (force_simt() || dtype != SDPA_B200_F16) return false;
  if (S_kv == 0) return false;  // a TMA map cannot have a zero extent
  if (D_qk % 8 != 0 || D_v % 8 != 0) return false;  // TMA row strides must be 16-byte multiples
  if (D_qk < 16) return false;  // see the comment above
  return aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o);
}

bool tc_bwd_ok(int dtype, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, const void* const* ptrs, int n) {
  if (force_simt() || dtype != SDPA_B200_F16 || S_q == 0 || S_kv == 0) return false;
  if (D_qk % 8 != 0 || D_v % 8 != 0 || D_qk < 16) return false;  // D_qk < 16: see tc_fwd_ok
  for (int i = 0; i < n; ++i)
    if (!aligned16(ptrs[i])) return false;
  return true;
}

// fp32 on the 3xTF32 tensor-core kernels: rows must be 16-byte multiples
// (TMA strides), every pointer 16-byte aligned; the backward serves D_qk <= 64
// (and D_qk = 128 on the GEMM route).
bool tf32_fwd_ok(int dtype, int64_t S_kv, int64_t D_qk, int64_t D_v, const void* q, const void* k, const void* v,
                 const void* o) {
  if (force_simt() || dtype != SDPA_B200_F32 || S_kv == 0) return false;
  if (D_qk % 4 != 0 || D_v % 4 != 0) return false;
  return aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o);
}

// gemm: the workspace admits the GEMM route, which also serves D_qk = 128
// (the recomputing passes need D_qk <= 64).
bool tf32_bwd_ok(int dtype, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, const void* const* ptrs, int n,
                 bool gemm) {
  if (force_simt() || dtype != SDPA_B200_F32 || S_q == 0 || S_kv == 0) return false;
  if (D_qk % 4 != 0 || D_v % 4 != 0) return false;
  if (D_qk > 64 && !gemm) return false;
  for (int i = 0; i < n; ++i)
    if (!aligned16(ptrs[i])) return false;
  return true;
}

// --------------------------------------------------------- diagnostics
__global__ void dropout_mask_kernel(Params p, uint8_t* mask) {
  const int64_t n = p.B * p.S_q * p.S_kv;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < n;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = idx / p.S_kv, j = idx - row * p.S_kv;
    const uint64_t base = p.rng_base + static_cast<uint64_t>(row) * static_cast<uint64_t>(p.S_kv);
    mask[idx] = (p.dropout_on && dropped(lcg_state(base, static_cast<uint64_t>(j)), p.drop_thr)) ? 1 : 0;
  }
}

__global__ void wait_timeout_kernel(uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    WaitCtl ctl;
    ctl.deadline_ns = globaltimer_ns() + timeout_ns;
    ctl.abort_flag = &abort_flag;
    mbar_wait(&bar, 0, ctl);  // nothing arrives: gives up and raises the status bit
  }
  __syncthreads();
}

}  // namespace

extern "C" {

static int fwd_impl(int dtype, const void* q, const void* k, const void* v, void* out, float* stats, int64_t B,
                    int64_t H, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout,
                    int causal, uint64_t seed, uint64_t offset, void* stream) {
  t_launches = 0;
  if (int r = check_common(dtype, B, S_q, S_kv, D_qk, D_v, causal)) return r;
  if (H < 1 || B % H != 0) return SDPA_B200_EINVAL;
  if (B == 0 || S_q == 0) return SDPA_B200_OK;
  if (!out || !stats || (S_kv > 0 && (!q || !k || !v))) return SDPA_B200_EINVAL;
  Params p = make_params(B, S_q, S_kv, D_qk, D_v, scale, dropout, causal, seed, offset);
  p.H = H;
  p.q = q;
  p.k = k;
  p.v = v;
  p.out = out;
  p.stats = stats;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int r = bind_context()) return r;
  if (tc_fwd_ok(dtype, S_kv, D_qk, D_v, q, k, v, out)) return launch_fwd_tc(p, st, &t_launches);
  if (tf32_fwd_ok(dtype, S_kv, D_qk, D_v, q, k, v, out)) return launch_fwd_tf32(p, st, &t_launches);
  return dtype == SDPA_B200_F16 ? launch_fwd_simt_f16(p, st, &t_launches) : launch_fwd_simt_f32(p, st, &t_launches);
}

int sdpa_b200_fwd(int dtype, const void* q, const void* k, const void* v, void* out, float* stats, int64_t B,
                  int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout, int causal,
                  uint64_t seed, uint64_t offset, void* stream) {
  return fwd_impl(dtype, q, k, v, out, stats, B, 1, S_q, S_kv, D_qk, D_v, scale, dropout, causal, seed, offset,
                  stream);
}

static bool bshd_batch(int64_t B, int64_t H) { return B >= 0 && H >= 1 && B <= 0x7fffffffLL / H; }

int sdpa_b200_fwd_bshd(int dtype, const void* q, const void* k, const void* v, void* out, float* stats, int64_t B,
                       int64_t H, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout,
                       int causal, uint64_t seed, uint64_t offset, void* stream) {
  t_launches = 0;
  if (!bshd_batch(B, H)) return SDPA_B200_EINVAL;
  return fwd_impl(dtype, q, k, v, out, stats, B * H, H, S_q, S_kv, D_qk, D_v, scale, dropout, causal, seed, offset,
                  stream);
}

// Workspace of the fp32 backward's GEMM route beyond the delta rows: dS and
// P~, [rows, S_q, ld_k] each (ld_k = S_kv rounded up to 16 bytes).  The
// query asks for all B rows up to a cap that keeps the workspace a small part
// of HBM; past it, for as many rows as fit, and the backward runs in batch
// chunks of that many rows.  Where not even one row fits (or the caller gives
// less than one row's worth) the three recomputing passes run instead.
constexpr size_t kGemmWorkspaceCap = size_t(4) << 30;
static int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }
static size_t delta_bytes(int64_t B, int64_t S_q) {
  return static_cast<size_t>(round_up(B * S_q * static_cast<int64_t>(sizeof(float)), 256));
}
static bool gemm_shape(int dtype, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v) {
  return !force_simt() && dtype == SDPA_B200_F32 && S_q > 0 && S_kv > 0 && D_qk % 4 == 0 && D_v % 4 == 0;
}
// bytes for `rows` batch rows (+ room to align the start to 256 bytes)
static size_t gemm_chunk_bytes(int64_t rows, int64_t S_q, int64_t S_kv) {
  return 2 * static_cast<size_t>(round_up(rows * S_q * round_up(S_kv, 4) * 4, 256)) + 256;
}
// most batch rows (<= B) whose chunk fits in `avail` bytes; 0 if none
static int64_t gemm_rows_fitting(size_t avail, int64_t B, int64_t S_q, int64_t S_kv) {
  const int64_t ld = round_up(S_kv, 4);
  if (avail < 1024 || S_q > static_cast<int64_t>(avail / 8) / ld) return 0;  // not even one row
  const int64_t row_bytes = 8 * S_q * ld;  // dS + P~ of one row
  int64_t rows = static_cast<int64_t>(avail / static_cast<size_t>(row_bytes));
  if (rows > B) rows = B;
  while (rows > 0 && gemm_chunk_bytes(rows, S_q, S_kv) > avail) --rows;
  return rows;
}
static size_t gemm_ws_bytes(int dtype, int64_t B, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v) {
  if (B <= 0 || !gemm_shape(dtype, S_q, S_kv, D_qk, D_v)) return 0;
  const int64_t rows = gemm_rows_fitting(kGemmWorkspaceCap, B, S_q, S_kv);
  return rows > 0 ? gemm_chunk_bytes(rows, S_q, S_kv) : 0;
}

size_t sdpa_b200_bwd_workspace_bytes(int dtype, int64_t B, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v) {
  if (B <= 0 || S_q <= 0) return 0;
  const size_t extra = gemm_ws_bytes(dtype, B, S_q, S_kv, D_qk, D_v);
  return extra ? delta_bytes(B, S_q) + extra : static_cast<size_t>(B) * static_cast<size_t>(S_q) * sizeof(float);
}

static int bwd_impl(int dtype, const void* q, const void* k, const void* v, const void* out, const float* stats,
                    const float* d_stats, const void* d_out, void* dq, void* dk, void* dv, int64_t B, int64_t H,
                    int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout, int causal,
                    uint64_t seed, uint64_t offset, void* workspace, size_t workspace_bytes, void* stream) {
  t_launches = 0;
  if (int r = check_common(dtype, B, S_q, S_kv, D_qk, D_v, causal)) return r;
  if (H < 1 || B % H != 0) return SDPA_B200_EINVAL;
  if (B == 0 || (S_q == 0 && S_kv == 0)) return SDPA_B200_OK;
  // one float per query row is required; the fp32 GEMM route uses more when given
  const size_t need = (B > 0 && S_q > 0) ? static_cast<size_t>(B) * static_cast<size_t>(S_q) * sizeof(float) : 0;
  if (need > 0 && (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 3u)))
    return SDPA_B200_EWORKSPACE;
  if ((S_q > 0 && (!q || !out || !stats || !d_out || !dq)) || (S_kv > 0 && (!k || !v || !dk || !dv)))
    return SDPA_B200_EINVAL;
  Params p = make_params(B, S_q, S_kv, D_qk, D_v, scale, dropout, causal, seed, offset);
  p.H = H;
  p.q = q;
  p.k = k;
  p.v = v;
  p.o = out;
  p.lse = stats;
  p.d_o = d_out;
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.delta = static_cast<float*>(workspace);
  p.d_stats = d_stats;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int r = bind_context()) return r;
  const void* ptrs[] = {q, k, v, out, d_out, dq, dk, dv};
  if (tc_bwd_ok(dtype, S_q, S_kv, D_qk, D_v, ptrs, 8)) return launch_bwd_tc(p, st, &t_launches);
  // GEMM route: the rows of workspace beyond delta (a multiple of H, so a
  // chunk of the [B/H, S, H, D] layout starts at an outer batch row)
  int64_t rows = 0;
  if (gemm_shape(dtype, S_q, S_kv, D_qk, D_v) && workspace_bytes > delta_bytes(B, S_q)) {
    rows = gemm_rows_fitting(workspace_bytes - delta_bytes(B, S_q), B, S_q, S_kv);
    rows -= rows % H;
  }
  const bool gemm = rows > 0;
  if (tf32_bwd_ok(dtype, S_q, S_kv, D_qk, D_v, ptrs, 8, gemm)) {
    if (gemm) {
      const uintptr_t w0 = reinterpret_cast<uintptr_t>(workspace) + delta_bytes(B, S_q);
      uint8_t* w = reinterpret_cast<uint8_t*>((w0 + 255u) & ~uintptr_t(255u));
      p.ld_k = round_up(S_kv, 4);
      p.ws_rows = rows;
      p.ws_ds = reinterpret_cast<float*>(w);
      p.ws_p = reinterpret_cast<float*>(w + round_up(rows * S_q * p.ld_k * 4, 256));
    }
    return launch_bwd_tf32(p, st, &t_launches);
  }
  return dtype == SDPA_B200_F16 ? launch_bwd_simt_f16(p, st, &t_launches) : launch_bwd_simt_f32(p, st, &t_launches);
}

int sdpa_b200_bwd(int dtype, const void* q, const void* k, const void* v, const void* out, const float* stats,
                  const void* d_out, void* dq, void* dk, void* dv, int64_t B, int64_t S_q, int64_t S_kv, int64_t D_qk,
                  int64_t D_v, float scale, float dropout, int causal, uint64_t seed, uint64_t offset,
                  void* workspace, size_t workspace_bytes, void* stream) {
  return bwd_impl(dtype, q, k, v, out, stats, nullptr, d_out, dq, dk, dv, B, 1, S_q, S_kv, D_qk, D_v, scale,
                  dropout, causal, seed, offset, workspace, workspace_bytes, stream);
}

int sdpa_b200_bwd_dstats(int dtype, const void* q, const void* k, const void* v, const void* out, const float* stats,
                         const float* d_stats, const void* d_out, void* dq, void* dk, void* dv, int64_t B, int64_t S_q,
                         int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout, int causal, uint64_t seed,
                         uint64_t offset, void* workspace, size_t workspace_bytes, void* stream) {
  return bwd_impl(dtype, q, k, v, out, stats, d_stats, d_out, dq, dk, dv, B, 1, S_q, S_kv, D_qk, D_v, scale,
                  dropout, causal, seed, offset, workspace, workspace_bytes, stream);
}

int sdpa_b200_bwd_bshd(int dtype, const void* q, const void* k, const void* v, const void* out, const float* stats,
                       const float* d_stats, const void* d_out, void* dq, void* dk, void* dv, int64_t B, int64_t H,
                       int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout, int causal,
                       uint64_t seed, uint64_t offset, void* workspace, size_t workspace_bytes, void* stream) {
  t_launches = 0;
  if (!bshd_batch(B, H)) return SDPA_B200_EINVAL;
  return bwd_impl(dtype, q, k, v, out, stats, d_stats, d_out, dq, dk, dv, B * H, H, S_q, S_kv, D_qk, D_v, scale,
                  dropout, causal, seed, offset, workspace, workspace_bytes, stream);
}

const char* sdpa_b200_last_error_detail(void) { return t_err_detail; }

int sdpa_b200_dropout_mask(uint64_t seed, uint64_t offset, int64_t B, int64_t S_q, int64_t S_kv, float dropout,
                           uint8_t* mask, void* stream) {
  t_launches = 0;
  if (B < 0 || S_q < 0 || S_kv < 0) return SDPA_B200_EINVAL;
  const int64_t n = B * S_q * S_kv;
  if (n == 0) return SDPA_B200_OK;
  if (!mask) return SDPA_B200_EINVAL;
  Params p = make_params(B, S_q, S_kv, 1, 1, 1.0f, dropout, 0, seed, offset);
  const int64_t blocks = (n + 255) / 256 < 148 * 32 ? (n + 255) / 256 : 148 * 32;
  dropout_mask_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(p, mask);
  ++t_launches;
  return launch_result();
}

const char* sdpa_b200_strerror(int status) {
  switch (status) {
    case SDPA_B200_OK: return "ok";
    case SDPA_B200_EINVAL: return "invalid argument";
    case SDPA_B200_EUNSUPPORTED: return "feature size over 128 is not supported";
    case SDPA_B200_ECUDA: return "CUDA error";
    case SDPA_B200_ETIMEOUT: return "a device-side wait timed out";
    case SDPA_B200_EWORKSPACE: return "workspace missing, misaligned or too small";
    case SDPA_B200_ESCRATCH: return "B * S_q exceeds the built-in scratch of sdpa_b200_bwd_noalloc (1048576 rows)";
    default: return "unknown status";
  }
}

int sdpa_b200_device_status(unsigned int* word, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned int w = 0;
  if (cudaStreamSynchronize(st) != cudaSuccess) return SDPA_B200_ECUDA;
  const unsigned int zero = 0;
  if (cudaMemcpyFromSymbol(&w, g_status_word, sizeof(w)) != cudaSuccess) return SDPA_B200_ECUDA;
  if (cudaMemcpyToSymbol(g_status_word, &zero, sizeof(zero)) != cudaSuccess) return SDPA_B200_ECUDA;
  if (status_exchange_fwd_tc(&w) || status_exchange_bwd_tc(&w) || status_exchange_tf32(&w) || status_exchange_simt_fwd_f16(&w) ||
      status_exchange_simt_fwd_f32(&w) || status_exchange_simt_bwd_f16(&w) || status_exchange_simt_bwd_f32(&w)) return SDPA_B200_ECUDA;
  if (word) *word = w;
  return (w & kStatusTimeout) ? SDPA_B200_ETIMEOUT : SDPA_B200_OK;
}

void sdpa_b200_set_wait_timeout_ns(uint64_t ns) { g_timeout_ns.store(ns ? ns : kDefaultTimeoutNs); }

int sdpa_b200_test_wait_timeout(uint64_t timeout_ns, void* stream) {
  wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(timeout_ns);
  return launch_result();
}

int sdpa_b200_path(int dtype, int64_t D_qk, int64_t D_v, int backward) {
  if (force_simt()) return 0;
  if (dtype == SDPA_B200_F16) return (D_qk % 8 == 0 && D_v % 8 == 0 && D_qk >= 16) ? 1 : 0;
  // the fp32 backward with D_qk > 64 given the full workspace (GEMM route)
  (void)backward;
  if (dtype == SDPA_B200_F32 && D_qk % 4 == 0 && D_v % 4 == 0) return 2;
  return 0;
}

int sdpa_b200_last_launch_count(void) { return t_launches; }

int sdpa_b200_set_bwd_events(void* const* events, int n) {
  if (!events) {
    t_bwd_events = nullptr;
    return SDPA_B200_OK;
  }
  if (n < 4 || n > 8) return SDPA_B200_EINVAL;
  for (int i = 0; i < 8; ++i) t_bwd_event_store[i] = i < n ? events[i] : nullptr;
  t_bwd_events = t_bwd_event_store;
  return SDPA_B200_OK;
}

int sdpa_b200_version(void) { return 100; }

}  // extern "C"

// ------------------------------------------------ backward without allocation
// The per-row scratch of sdpa_b200_bwd_noalloc.  Host code must not pass the
// symbol itself to a kernel (on the host it only names a stand-in); its device
// address is looked up once per device with cudaGetSymbolAddress.
static __device__ __align__(256) float g_noalloc_scratch[SDPA_B200_NOALLOC_MAX_ROWS];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};  // device address of g_noalloc_scratch, per device ordinal

// Device address of the scratch array on the current device (looked up on
// the first call per device).  Returns nullptr when the lookup fails.
void* noalloc_scratch_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
    g_noalloc_ptr[dev] = p;
  }
  return g_noalloc_ptr[dev];
}
}  // namespace

extern "C" {

int sdpa_b200_bwd_noalloc(int dtype, const void* q, const void* k, const void* v, const void* out,
                          const float* stats, const void* d_out, void* dq, void* dk, void* dv, int64_t B,
                          int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout,
                          int causal, uint64_t seed, uint64_t offset, void* stream) {
  t_launches = 0;
  if (int r = check_common(dtype, B, S_q, S_kv, D_qk, D_v, causal)) return r;
  if (B * S_q > SDPA_B200_NOALLOC_MAX_ROWS) return SDPA_B200_ESCRATCH;
  // the symbol lookup and the launches must use the same (primary) context
  if (int r = bind_context()) return r;
  void* scratch = noalloc_scratch_ptr();
  if (!scratch) return SDPA_B200_ECUDA;
  return sdpa_b200_bwd(dtype, q, k, v, out, stats, d_out, dq, dk, dv, B, S_q, S_kv, D_qk, D_v, scale, dropout,
                       causal, seed, offset, scratch, sizeof(float) * SDPA_B200_NOALLOC_MAX_ROWS, stream);
}

}  // extern "C"
