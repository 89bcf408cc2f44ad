// Translation unit: fp32 (3xTF32) tcgen05 forward and backward kernels
#include "host.cuh"
#include "ptx.cuh"
#include "tf32_bwd.cuh"
#include "tf32_fwd.cuh"
#include "tf32_gemm.cuh"
#include "tf32_scores.cuh"

using namespace sdpa_b200;
using namespace sdpa_b200::host;

namespace {

template <int DQK, int DV, bool DROP, bool HEADS>
int launch_fwd_t(const Params& p, cudaStream_t st, int* launches) {
  static std::atomic<uint64_t> attr_done{0};
  using Cfg = tf32::FwdCfg<DQK, DV>;
  auto kern = tf32::fwd_kernel<DQK, DV, DROP, HEADS>;
  if (cudaError_t e = ensure_smem(kern, Cfg::kSmemBytes, attr_done)) return cuda_failure("shared-memory attribute", e);
  CUtensorMap mk, mv;
  if (!make_map_f32(&mk, p.k, p.B, p.H, p.S_kv, p.D_qk, Cfg::kBN) ||
      !make_map_f32_mn(&mv, p.v, p.B, p.H, p.S_kv, p.D_v, Cfg::kBN))
    return SDPA_B200_ECUDA;  // detail recorded by make_map
  const int64_t grid = ((p.S_q + tf32::kBM - 1) / tf32::kBM) * p.B;
  if (int r = launch_tc(kern, grid, tf32::kFwdThreads, Cfg::kSmemBytes, st, mk, mv, p)) return r;
  ++*launches;
  return SDPA_B200_OK;
}

template <int DQK, int DV>
int launch_fwd_d(const Params& p, cudaStream_t st, int* launches) {
  if (p.H > 1)
    return p.dropout_on ? launch_fwd_t<DQK, DV, true, true>(p, st, launches)
                        : launch_fwd_t<DQK, DV, false, true>(p, st, launches);
  return p.dropout_on ? launch_fwd_t<DQK, DV, true, false>(p, st, launches)
                      : launch_fwd_t<DQK, DV, false, false>(p, st, launches);
}

template <int MODE, int DQK, int DV, bool DROP, bool HEADS>
int launch_bwd_mode(const Params& p, cudaStream_t st, int* launches) {
  static std::atomic<uint64_t> attr_done{0};
  using Cfg = tf32::BwdCfg<MODE, DQK, DV>;
  auto kern = tf32::bwd_kernel<MODE, DQK, DV, DROP, HEADS>;
  if (cudaError_t e = ensure_smem(kern, Cfg::kSmemBytes, attr_done)) return cuda_failure("shared-memory attribute", e);
  const bool rows_q = MODE == tf32::kDQ;
  CUtensorMap ma, mb;
  // streamed tiles: K, V (DQ) or Q, dO (DK, DV); DV reads dO only MN-major
  const int64_t S_str = rows_q ? p.S_kv : p.S_q;
  const bool ok_a = make_map_f32(&ma, rows_q ? p.k : p.q, p.B, p.H, S_str, p.D_qk, Cfg::kN);
  const bool ok_b = MODE == tf32::kDV ? make_map_f32_mn(&mb, p.d_o, p.B, p.H, S_str, p.D_v, Cfg::kN)
                                      : make_map_f32(&mb, rows_q ? p.v : p.d_o, p.B, p.H, S_str, p.D_v, Cfg::kN);
  if (!ok_a || !ok_b) return SDPA_B200_ECUDA;  // detail recorded by make_map
  const int64_t grid = (((rows_q ? p.S_q : p.S_kv) + 127) / 128) * p.B;
  if (int r = launch_tc(kern, grid, tf32::kBwdThreads, Cfg::kSmemBytes, st, ma, mb, p)) return r;
  ++*launches;
  return SDPA_B200_OK;
}

// DQ first: it writes D = rowsum(dO * O) (into the workspace), which DK reads.
template <int DQK, int DV, bool DROP, bool HEADS>
int launch_bwd_t(const Params& p, cudaStream_t st, int* launches) {
  sdpa_b200::record_bwd_event(0, st);
  if (int r = launch_bwd_mode<tf32::kDQ, DQK, DV, DROP, HEADS>(p, st, launches)) return r;
  sdpa_b200::record_bwd_event(1, st);
  if (int r = launch_bwd_mode<tf32::kDK, DQK, DV, DROP, HEADS>(p, st, launches)) return r;
  sdpa_b200::record_bwd_event(2, st);
  if (int r = launch_bwd_mode<tf32::kDV, DQK, DV, DROP, HEADS>(p, st, launches)) return r;
  sdpa_b200::record_bwd_event(3, st);
  return SDPA_B200_OK;
}

// C = alpha * A B over the materialised matrix a ([B, rows, ld]; A itself,
// or with A_MN its transpose) and the [B/H, K, H, N] operand b_src.
template <int N, bool HEADS, bool A_MN>
int launch_gemm(const float* a, int64_t ld, const void* b_src, int d_b, float* c, const Params& p, int64_t M,
                int64_t K, float alpha, int range, cudaStream_t st, int* launches) {
  static std::atomic<uint64_t> attr_done{0};
  using Cfg = tf32::GemmCfg<N>;
  auto kern = tf32::gemm_kernel<N, HEADS, A_MN>;
  if (cudaError_t e = ensure_smem(kern, Cfg::kSmemBytes, attr_done)) return cuda_failure("shared-memory attribute", e);
  CUtensorMap ma, mb;
  const bool ok_a = A_MN ? make_map_rows_f32(&ma, a, p.B, K, M, ld, Cfg::kK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)
                         : make_map_rows_f32(&ma, a, p.B, M, K, ld, 128);
  if (!ok_a || !make_map_f32_mn(&mb, b_src, p.B, p.H, K, d_b, Cfg::kK))
    return SDPA_B200_ECUDA;  // detail recorded by make_map
  tf32::GemmArgs g;
  g.c = c;
  g.B = p.B;
  g.H = p.H;
  g.M = M;
  g.K = K;
  g.D = d_b;
  g.alpha = alpha;
  g.range = range;
  g.timeout_ns = p.timeout_ns;
  // Persistent (one CTA per SM: the shared memory admits no second) for short
  // items, whose pipeline fill and drain it hides; long items (dQ at cfg5: 128
  // tiles) run one CTA each, which the hardware balances better than a
  // static round-robin (measured).
  const int64_t items = ((M + 127) / 128) * p.B;
  const int64_t grid = (K + Cfg::kK - 1) / Cfg::kK >= 64 || items < num_sms() ? items : num_sms();
  if (int r = launch_tc(kern, grid, tf32::kGemmThreads, Cfg::kSmemBytes, st, ma, mb, g)) return r;
  ++*launches;
  return SDPA_B200_OK;
}

template <int DQK, int DV, bool DROP, bool HEADS>
int launch_scores(const Params& p, cudaStream_t st, int* launches) {
  static std::atomic<uint64_t> attr_done{0};
  using Cfg = tf32::ScoreCfg<DQK, DV>;
  auto kern = tf32::score_kernel<DQK, DV, DROP, HEADS>;
  if (cudaError_t e = ensure_smem(kern, Cfg::kSmemBytes, attr_done)) return cuda_failure("shared-memory attribute", e);
  CUtensorMap mq, mo;
  if (!make_map_f32(&mq, p.q, p.B, p.H, p.S_q, p.D_qk, Cfg::kN) ||
      !make_map_f32(&mo, p.d_o, p.B, p.H, p.S_q, p.D_v, Cfg::kN))
    return SDPA_B200_ECUDA;  // detail recorded by make_map
  const int64_t grid = ((p.S_kv + 127) / 128) * p.B;
  if (int r = launch_tc(kern, grid, tf32::kScoreThreads, Cfg::kSmemBytes, st, mq, mo, p)) return r;
  ++*launches;
  return SDPA_B200_OK;
}

// The GEMM route (p.ws_ds / p.ws_p set): D, the score pass writing dS and
// P~, then dQ = scale dS K, dK = scale dS^T Q and dV = P~^T dO as GEMMs (the
// last two read their A operand MN-major).
template <int DQK, int DV, bool DROP, bool HEADS>
int launch_bwd_gemm_t(const Params& p, cudaStream_t st, int* launches) {
  sdpa_b200::record_bwd_event(0, st);
  const int64_t rows = p.B * p.S_q;
  if ((rows + 7) / 8 > 0x7fffffffLL) return SDPA_B200_EINVAL;
  tf32::delta_kernel<HEADS><<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(p);
  ++*launches;
  if (int r = launch_result()) return r;
  if (int r = launch_scores<DQK, DV, DROP, HEADS>(p, st, launches)) return r;
  sdpa_b200::record_bwd_event(1, st);
  const int range_q = p.causal ? 1 : 0, range_kv = p.causal ? 2 : 0;
  if (int r = launch_gemm<DQK, HEADS, false>(p.ws_ds, p.ld_k, p.k, p.D_qk, static_cast<float*>(p.dq), p, p.S_q,
                                             p.S_kv, p.scale, range_q, st, launches))
    return r;
  sdpa_b200::record_bwd_event(2, st);
  if (int r = launch_gemm<DQK, HEADS, true>(p.ws_ds, p.ld_k, p.q, p.D_qk, static_cast<float*>(p.dk), p, p.S_kv,
                                            p.S_q, p.scale, range_kv, st, launches))
    return r;
  sdpa_b200::record_bwd_event(3, st);
  if (int r = launch_gemm<DV, HEADS, true>(p.ws_p, p.ld_k, p.d_o, p.D_v, static_cast<float*>(p.dv), p, p.S_kv,
                                            p.S_q, 1.0f, range_kv, st, launches))
    return r;
  sdpa_b200::record_bwd_event(4, st);
  return SDPA_B200_OK;
}

template <int DQK, int DV>
int launch_bwd_d(const Params& p, cudaStream_t st, int* launches) {
  if (p.ws_ds) {
    if (p.H > 1)
      return p.dropout_on ? launch_bwd_gemm_t<DQK, DV, true, true>(p, st, launches)
                          : launch_bwd_gemm_t<DQK, DV, false, true>(p, st, launches);
    return p.dropout_on ? launch_bwd_gemm_t<DQK, DV, true, false>(p, st, launches)
                        : launch_bwd_gemm_t<DQK, DV, false, false>(p, st, launches);
  }
  if (p.H > 1)
    return p.dropout_on ? launch_bwd_t<DQK, DV, true, true>(p, st, launches)
                        : launch_bwd_t<DQK, DV, false, true>(p, st, launches);
  return p.dropout_on ? launch_bwd_t<DQK, DV, true, false>(p, st, launches)
                      : launch_bwd_t<DQK, DV, false, false>(p, st, launches);
}

// D_qk = 128: the GEMM route only (the recomputing passes do not fit TMEM;
// the score pass holds K, V hi / lo in 2*128 + 2*64 columns, or with D_v =
// 128 keeps V lo in shared memory).
template <int DQK, int DV>
int launch_bwd_gemm_d(const Params& p, cudaStream_t st, int* launches) {
  if (p.H > 1)
    return p.dropout_on ? launch_bwd_gemm_t<DQK, DV, true, true>(p, st, launches)
                        : launch_bwd_gemm_t<DQK, DV, false, true>(p, st, launches);
  return p.dropout_on ? launch_bwd_gemm_t<DQK, DV, true, false>(p, st, launches)
                      : launch_bwd_gemm_t<DQK, DV, false, false>(p, st, launches);
}

}  // namespace

// Every D_qk, D_v <= 128 (both over 64: Q lo in shared memory, see FwdCfg).
int sdpa_b200::launch_fwd_tf32(const Params& p, cudaStream_t st, int* launches) {
  const bool q128 = p.D_qk > 64, v128 = p.D_v > 64;
  if (q128 && v128) return launch_fwd_d<128, 128>(p, st, launches);
  if (q128) return launch_fwd_d<128, 64>(p, st, launches);
  if (v128) return launch_fwd_d<64, 128>(p, st, launches);
#ifndef SDPA_B200_TF32_NARROW_FWD
#define SDPA_B200_TF32_NARROW_FWD 1
#endif
  if (SDPA_B200_TF32_NARROW_FWD && p.D_v <= 32) return launch_fwd_d<64, 32>(p, st, launches);  // N = 32 output MMAs
  return launch_fwd_d<64, 64>(p, st, launches);
}

// D_qk <= 64 on either route; D_qk = 128 on the GEMM route only (the caller
// checks): with D_qk = 128 the resident operands and accumulators of the DQ
// pass exceed TMEM.
static int launch_bwd_tf32_one(const Params& p, cudaStream_t st, int* launches) {
  if (p.D_qk > 64) {
    if (!p.ws_ds) return SDPA_B200_EUNSUPPORTED;
    if (p.D_v > 64) return launch_bwd_gemm_d<128, 128>(p, st, launches);  // V lo in shared memory
    return p.D_v <= 32 ? launch_bwd_gemm_d<128, 32>(p, st, launches) : launch_bwd_gemm_d<128, 64>(p, st, launches);
  }
  if (p.D_v > 64) return launch_bwd_d<64, 128>(p, st, launches);
  if (p.D_v <= 32) return launch_bwd_d<64, 32>(p, st, launches);
  return launch_bwd_d<64, 64>(p, st, launches);
}

// The GEMM route with a workspace for fewer rows than the batch: chunks of
// p.ws_rows batch rows (a multiple of H), each a complete backward of its
// rows; every per-row quantity (tensors, stats, D, the dropout counter base
// (b S_q + i) S_kv) is offset to the chunk's first row.
int sdpa_b200::launch_bwd_tf32(const Params& p, cudaStream_t st, int* launches) {
  if (!p.ws_ds || p.ws_rows >= p.B) return launch_bwd_tf32_one(p, st, launches);
  for (int64_t b0 = 0; b0 < p.B; b0 += p.ws_rows) {
    Params c = p;
    c.B = p.B - b0 < p.ws_rows ? p.B - b0 : p.ws_rows;
    const int64_t rq = b0 * p.S_q, rk = b0 * p.S_kv;  // first row of the chunk in [B*S, D] terms
    c.q = static_cast<const float*>(p.q) + rq * p.D_qk;
    c.k = static_cast<const float*>(p.k) + rk * p.D_qk;
    c.v = static_cast<const float*>(p.v) + rk * p.D_v;
    c.o = static_cast<const float*>(p.o) + rq * p.D_v;
    c.d_o = static_cast<const float*>(p.d_o) + rq * p.D_v;
    c.dq = static_cast<float*>(p.dq) + rq * p.D_qk;
    c.dk = static_cast<float*>(p.dk) + rk * p.D_qk;
    c.dv = static_cast<float*>(p.dv) + rk * p.D_v;
    c.lse = p.lse + rq;
    c.delta = p.delta + rq;
    if (p.d_stats) c.d_stats = p.d_stats + rq;
    c.rng_base = p.rng_base + static_cast<uint64_t>(rq) * static_cast<uint64_t>(p.S_kv);
    c.ws_rows = c.B;
    if (int r = launch_bwd_tf32_one(c, st, launches)) return r;
  }
  return SDPA_B200_OK;
}

SDPA_B200_STATUS_EXCHANGE(tf32)

#ifdef SDPA_B200_TF32_PROBE
// Reads and clears the timing probe of tuning builds.
extern "C" int sdpa_b200_tf32_probe_read(unsigned long long* out) {
  const unsigned long long zero[16] = {};
  if (cudaMemcpyFromSymbol(out, tf32::g_tf32_probe, sizeof(zero)) != cudaSuccess) return 1;
  return cudaMemcpyToSymbol(tf32::g_tf32_probe, zero, sizeof(zero)) == cudaSuccess ? 0 : 1;
}
#endif

#ifdef SDPA_B200_TF32_FWD_PROBE
// Reads and clears the forward timing probe of tuning builds.
extern "C" int sdpa_b200_tf32_fwd_probe_read(unsigned long long* out) {
  const unsigned long long zero[16] = {};
  if (cudaMemcpyFromSymbol(out, tf32::g_tf32_fwd_probe, sizeof(zero)) != cudaSuccess) return 1;
  return cudaMemcpyToSymbol(tf32::g_tf32_fwd_probe, zero, sizeof(zero)) == cudaSuccess ? 0 : 1;
}
#endif
