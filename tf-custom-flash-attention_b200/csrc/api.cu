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

#include "../../include/sdpa_b200.h"
#include "common.cuh"
#include "ptx.cuh"
#include "simt.cuh"
#include "fwd_tc.cuh"
#include "bwd_tc.cuh"

using namespace sdpa_b200;

namespace {

constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;
std::atomic<uint64_t> g_timeout_ns{kDefaultTimeoutNs};
thread_local int t_launches = 0;

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

int dmax_bucket(int64_t d) {
  if (d <= 8) return 8;
  if (d <= 16) return 16;
  if (d <= 32) return 32;
  if (d <= 64) return 64;
  return 128;
}

Params make_params(int64_t B, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout,
                   int causal, uint64_t seed, uint64_t offset) {
  Params p;
  std::memset(&p, 0, sizeof(p));
  p.B = B;
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
  p.timeout_ns = g_timeout_ns.load();
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

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- TMA maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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
bool make_map_f16(CUtensorMap* m, const void* base, int64_t B, int64_t S, int64_t D, int rows) {
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
cudaError_t ensure_smem(K kernel, size_t bytes, std::atomic<uint64_t>& done_mask) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done_mask.load() & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess) done_mask.fetch_or(bit);
  return e;
}

int launch_result() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SDPA_B200_OK : SDPA_B200_ECUDA;
}

bool tc_fwd_ok(int dtype, int64_t S_kv, int64_t D_qk, int64_t D_v, const void* q, const void* k, const void* v,
               const void* o) {
  if (force_simt() || dtype != SDPA_B200_F16) return false;
  if (S_kv == 0) return false;  // a TMA map cannot have a zero extent
  if (D_qk % 8 != 0 || D_v % 8 != 0) return false;  // TMA row strides must be 16-byte multiples
  return aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o);
}

// ----------------------------------------------------------------- forward
template <int DQK, int DV>
int launch_tc_fwd(const Params& p, cudaStream_t st) {
  static std::atomic<uint64_t> attr_done{0};
  using Cfg = tc::FwdCfg<DQK, DV>;
  auto kern = tc::fwd_kernel<DQK, DV>;
  if (ensure_smem(kern, Cfg::kSmemBytes, attr_done) != cudaSuccess) return SDPA_B200_ECUDA;
  CUtensorMap mq, mk, mv;
  if (!make_map_f16(&mq, p.q, p.B, p.S_q, p.D_qk, tc::kBM) || !make_map_f16(&mk, p.k, p.B, p.S_kv, p.D_qk, tc::kBN) ||
      !make_map_f16(&mv, p.v, p.B, p.S_kv, p.D_v, tc::kBN))
    return SDPA_B200_ECUDA;
  const int64_t n_qt = (p.S_q + tc::kBM - 1) / tc::kBM;
  const int64_t grid = n_qt * p.B;
  if (grid > 0x7fffffffLL) return SDPA_B200_EINVAL;
  kern<<<static_cast<unsigned>(grid), tc::kFwdThreads, Cfg::kSmemBytes, st>>>(mq, mk, mv, p);
  ++t_launches;
  return launch_result();
}

template <typename T, int DM>
int launch_simt_fwd(const Params& p, cudaStream_t st) {
  const int64_t grid = ((p.S_q + simt::kFwdRows - 1) / simt::kFwdRows) * p.B;
  if (grid > 0x7fffffffLL) return SDPA_B200_EINVAL;
  simt::fwd_kernel<T, DM><<<static_cast<unsigned>(grid), simt::kFwdRows, 0, st>>>(p);
  ++t_launches;
  return launch_result();
}

template <typename T>
int simt_fwd_dispatch(const Params& p, cudaStream_t st) {
  switch (dmax_bucket(p.D_qk > p.D_v ? p.D_qk : p.D_v)) {
    case 8: return launch_simt_fwd<T, 8>(p, st);
    case 16: return launch_simt_fwd<T, 16>(p, st);
    case 32: return launch_simt_fwd<T, 32>(p, st);
    case 64: return launch_simt_fwd<T, 64>(p, st);
    default: return launch_simt_fwd<T, 128>(p, st);
  }
}

int tc_fwd_dispatch(const Params& p, cudaStream_t st) {
  const bool q128 = p.D_qk > 64, v128 = p.D_v > 64;
  if (q128 && v128) return launch_tc_fwd<128, 128>(p, st);
  if (q128) return launch_tc_fwd<128, 64>(p, st);
  if (v128) return launch_tc_fwd<64, 128>(p, st);
  return launch_tc_fwd<64, 64>(p, st);
}

// ---------------------------------------------------------------- backward
template <typename T, int DM>
int launch_simt_bwd(const Params& p, cudaStream_t st) {
  static std::atomic<uint64_t> attr_kv{0}, attr_q{0};
  const int64_t rows = p.B * p.S_q;
  if (rows > 0) {
    simt::delta_kernel<T><<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(p);
    ++t_launches;
    if (int r = launch_result()) return r;
  }
  const size_t smkv = simt::dkdv_smem<DM>(), smq = simt::dq_smem<DM>();
  if (ensure_smem(simt::dkdv_kernel<T, DM>, smkv, attr_kv) != cudaSuccess) return SDPA_B200_ECUDA;
  if (ensure_smem(simt::dq_kernel<T, DM>, smq, attr_q) != cudaSuccess) return SDPA_B200_ECUDA;
  const int64_t gkv = ((p.S_kv + simt::kBwdRows - 1) / simt::kBwdRows) * p.B;
  const int64_t gq = ((p.S_q + simt::kBwdRows - 1) / simt::kBwdRows) * p.B;
  if (gkv > 0x7fffffffLL || gq > 0x7fffffffLL) return SDPA_B200_EINVAL;
  if (gkv > 0) {
    simt::dkdv_kernel<T, DM><<<static_cast<unsigned>(gkv), simt::kBwdRows, smkv, st>>>(p);
    ++t_launches;
    if (int r = launch_result()) return r;
  }
  if (gq > 0) {
    simt::dq_kernel<T, DM><<<static_cast<unsigned>(gq), simt::kBwdRows, smq, st>>>(p);
    ++t_launches;
    if (int r = launch_result()) return r;
  }
  return SDPA_B200_OK;
}

template <typename T>
int simt_bwd_dispatch(const Params& p, cudaStream_t st) {
  switch (dmax_bucket(p.D_qk > p.D_v ? p.D_qk : p.D_v)) {
    case 8: return launch_simt_bwd<T, 8>(p, st);
    case 16: return launch_simt_bwd<T, 16>(p, st);
    case 32: return launch_simt_bwd<T, 32>(p, st);
    case 64: return launch_simt_bwd<T, 64>(p, st);
    default: return launch_simt_bwd<T, 128>(p, st);
  }
}

// tcgen05 backward: delta (rowsum dO*O) -> dK/dV kernel -> dQ kernel.
template <int DQK, int DV>
int launch_tc_bwd(const Params& p, cudaStream_t st) {
  static std::atomic<uint64_t> attr_kv{0}, attr_q{0};
  using Cfg = tc::BwdCfg<DQK, DV>;
  auto kkv = tc::dkdv_kernel<DQK, DV>;
  auto kq = tc::dq_kernel<DQK, DV>;
  if (ensure_smem(kkv, Cfg::kSmemBytes, attr_kv) != cudaSuccess) return SDPA_B200_ECUDA;
  if (ensure_smem(kq, Cfg::kSmemBytes, attr_q) != cudaSuccess) return SDPA_B200_ECUDA;
  CUtensorMap k128, v128, q64, do64, q128, do128, k64, v64;
  if (!make_map_f16(&k128, p.k, p.B, p.S_kv, p.D_qk, tc::kBwdRows) ||
      !make_map_f16(&v128, p.v, p.B, p.S_kv, p.D_v, tc::kBwdRows) ||
      !make_map_f16(&q64, p.q, p.B, p.S_q, p.D_qk, tc::kBwdTile) ||
      !make_map_f16(&do64, p.d_o, p.B, p.S_q, p.D_v, tc::kBwdTile) ||
      !make_map_f16(&q128, p.q, p.B, p.S_q, p.D_qk, tc::kBwdRows) ||
      !make_map_f16(&do128, p.d_o, p.B, p.S_q, p.D_v, tc::kBwdRows) ||
      !make_map_f16(&k64, p.k, p.B, p.S_kv, p.D_qk, tc::kBwdTile) ||
      !make_map_f16(&v64, p.v, p.B, p.S_kv, p.D_v, tc::kBwdTile))
    return SDPA_B200_ECUDA;
  const int64_t rows = p.B * p.S_q;
  simt::delta_kernel<__half><<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(p);
  ++t_launches;
  if (int r = launch_result()) return r;
  const int64_t gkv = ((p.S_kv + tc::kBwdRows - 1) / tc::kBwdRows) * p.B;
  const int64_t gq = ((p.S_q + tc::kBwdRows - 1) / tc::kBwdRows) * p.B;
  if (gkv > 0x7fffffffLL || gq > 0x7fffffffLL) return SDPA_B200_EINVAL;
  kkv<<<static_cast<unsigned>(gkv), tc::kBwdThreads, Cfg::kSmemBytes, st>>>(k128, v128, q64, do64, p);
  ++t_launches;
  if (int r = launch_result()) return r;
  kq<<<static_cast<unsigned>(gq), tc::kBwdThreads, Cfg::kSmemBytes, st>>>(q128, do128, k64, v64, p);
  ++t_launches;
  return launch_result();
}

int tc_bwd_dispatch(const Params& p, cudaStream_t st) {
  const bool q128 = p.D_qk > 64, v128 = p.D_v > 64;
  if (q128 && v128) return launch_tc_bwd<128, 128>(p, st);
  if (q128) return launch_tc_bwd<128, 64>(p, st);
  if (v128) return launch_tc_bwd<64, 128>(p, st);
  return launch_tc_bwd<64, 64>(p, st);
}

bool tc_bwd_ok(int dtype, int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, const void* const* ptrs, int n) {
  if (force_simt() || dtype != SDPA_B200_F16 || S_q == 0 || S_kv == 0) return false;
  if (D_qk % 8 != 0 || D_v % 8 != 0) return false;
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

int sdpa_b200_fwd(int dtype, const void* q, const void* k, const void* v, void* out, float* stats, int64_t B,
                  int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout, int causal,
                  uint64_t seed, uint64_t offset, void* stream) {
  t_launches = 0;
  if (int r = check_common(dtype, B, S_q, S_kv, D_qk, D_v, causal)) return r;
  if (B == 0 || S_q == 0) return SDPA_B200_OK;
  if (!out || !stats || (S_kv > 0 && (!q || !k || !v))) return SDPA_B200_EINVAL;
  Params p = make_params(B, S_q, S_kv, D_qk, D_v, scale, dropout, causal, seed, offset);
  p.q = q;
  p.k = k;
  p.v = v;
  p.out = out;
  p.stats = stats;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (tc_fwd_ok(dtype, S_kv, D_qk, D_v, q, k, v, out)) return tc_fwd_dispatch(p, st);
  return dtype == SDPA_B200_F16 ? simt_fwd_dispatch<__half>(p, st) : simt_fwd_dispatch<float>(p, st);
}

size_t sdpa_b200_bwd_workspace_bytes(int, int64_t B, int64_t S_q, int64_t, int64_t, int64_t) {
  if (B <= 0 || S_q <= 0) return 0;
  return static_cast<size_t>(B) * static_cast<size_t>(S_q) * sizeof(float);
}

int sdpa_b200_bwd(int dtype, const void* q, const void* k, const void* v, const void* out, const float* stats,
                  const void* d_out, void* dq, void* dk, void* dv, int64_t B, int64_t S_q, int64_t S_kv, int64_t D_qk,
                  int64_t D_v, float scale, float dropout, int causal, uint64_t seed, uint64_t offset,
                  void* workspace, size_t workspace_bytes, void* stream) {
  t_launches = 0;
  if (int r = check_common(dtype, B, S_q, S_kv, D_qk, D_v, causal)) return r;
  if (B == 0 || (S_q == 0 && S_kv == 0)) return SDPA_B200_OK;
  const size_t need = sdpa_b200_bwd_workspace_bytes(dtype, B, S_q, S_kv, D_qk, D_v);
  if (need > 0 && (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 3u)))
    return SDPA_B200_EWORKSPACE;
  if ((S_q > 0 && (!q || !out || !stats || !d_out || !dq)) || (S_kv > 0 && (!k || !v || !dk || !dv)))
    return SDPA_B200_EINVAL;
  Params p = make_params(B, S_q, S_kv, D_qk, D_v, scale, dropout, causal, seed, offset);
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
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const void* ptrs[] = {q, k, v, out, d_out, dq, dk, dv};
  if (tc_bwd_ok(dtype, S_q, S_kv, D_qk, D_v, ptrs, 8)) return tc_bwd_dispatch(p, st);
  return dtype == SDPA_B200_F16 ? simt_bwd_dispatch<__half>(p, st) : simt_bwd_dispatch<float>(p, st);
}

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
  if (cudaMemcpyFromSymbol(&w, g_status_word, sizeof(w)) != cudaSuccess) return SDPA_B200_ECUDA;
  const unsigned int zero = 0;
  if (cudaMemcpyToSymbol(g_status_word, &zero, sizeof(zero)) != cudaSuccess) return SDPA_B200_ECUDA;
  if (word) *word = w;
  return (w & kStatusTimeout) ? SDPA_B200_ETIMEOUT : SDPA_B200_OK;
}

void sdpa_b200_set_wait_timeout_ns(uint64_t ns) { g_timeout_ns.store(ns ? ns : kDefaultTimeoutNs); }

int sdpa_b200_test_wait_timeout(uint64_t timeout_ns, void* stream) {
  wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(timeout_ns);
  return launch_result();
}

int sdpa_b200_path(int dtype, int64_t D_qk, int64_t D_v, int backward) {
  (void)backward;
  if (force_simt() || dtype != SDPA_B200_F16) return 0;
  return (D_qk % 8 == 0 && D_v % 8 == 0) ? 1 : 0;
}

int sdpa_b200_last_launch_count(void) { return t_launches; }

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
  void* scratch = noalloc_scratch_ptr();
  if (!scratch) return SDPA_B200_ECUDA;
  return sdpa_b200_bwd(dtype, q, k, v, out, stats, d_out, dq, dk, dv, B, S_q, S_kv, D_qk, D_v, scale, dropout,
                       causal, seed, offset, scratch, sizeof(float) * SDPA_B200_NOALLOC_MAX_ROWS, stream);
}

}  // extern "C"
