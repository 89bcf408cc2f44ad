// Translation unit: tcgen05 forward kernels
#include "host.cuh"
#include "ptx.cuh"
#include "fwd_tc.cuh"

#include <cstdlib>

using namespace sdpa_b200;
using namespace sdpa_b200::host;

namespace {

// ----------------------------------------------------------------- forward
template <int DQK, int DV, bool DROP, bool HEADS>
int launch_tc_fwd_t(const Params& p, cudaStream_t st, int* launches) {
  static std::atomic<uint64_t> attr_done{0};
  using Cfg = tc::FwdCfg<DQK, DV>;
  auto kern = tc::fwd_kernel<DQK, DV, DROP, HEADS>;
  if (cudaError_t e = ensure_smem(kern, Cfg::kSmemBytes, attr_done)) return cuda_failure("shared-memory attribute", e);
  CUtensorMap mq, mk, mv;
  if (!make_map_f16(&mq, p.q, p.B, p.H, p.S_q, p.D_qk, tc::kBM) || !make_map_f16(&mk, p.k, p.B, p.H, p.S_kv, p.D_qk, tc::kBN) ||
      !make_map_f16(&mv, p.v, p.B, p.H, p.S_kv, p.D_v, tc::kBN))
    return SDPA_B200_ECUDA;  // detail recorded by make_map_f16
  const int64_t n_qt = (p.S_q + tc::kBM - 1) / tc::kBM;
  const int64_t grid = n_qt * p.B;
  if (int r = launch_tc(kern, grid, tc::kFwdThreads, Cfg::kSmemBytes, st, mq, mk, mv, p)) return r;
  ++*launches;
  return SDPA_B200_OK;
}

template <int DQK, int DV, bool HEADS>
int launch_tc_fwd_h(const Params& p, cudaStream_t st, int* launches) {
  return p.dropout_on ? launch_tc_fwd_t<DQK, DV, true, HEADS>(p, st, launches)
                      : launch_tc_fwd_t<DQK, DV, false, HEADS>(p, st, launches);
}
// HEADS: [B/H, S, H, D] tensors (4-D TMA maps); else contiguous [B, S, D].
template <int DQK, int DV>
int launch_tc_fwd(const Params& p, cudaStream_t st, int* launches) {
  return p.H > 1 ? launch_tc_fwd_h<DQK, DV, true>(p, st, launches) : launch_tc_fwd_h<DQK, DV, false>(p, st, launches);
}

// Paired-tile forward (two 128-row query tiles per CTA).
template <int DQK, int DV, bool DROP, bool HEADS>
int launch_pair_fwd_t(const Params& p, cudaStream_t st, int* launches) {
  static std::atomic<uint64_t> attr_done{0};
  using Cfg = tc::PairCfg<DQK, DV>;
  auto kern = tc::fwd_pair_kernel<DQK, DV, DROP, HEADS>;
  if (cudaError_t e = ensure_smem(kern, Cfg::kSmemBytes, attr_done)) return cuda_failure("shared-memory attribute", e);
  CUtensorMap mq, mk, mv;
  if (!make_map_f16(&mq, p.q, p.B, p.H, p.S_q, p.D_qk, tc::kBM) || !make_map_f16(&mk, p.k, p.B, p.H, p.S_kv, p.D_qk, tc::kBN) ||
      !make_map_f16(&mv, p.v, p.B, p.H, p.S_kv, p.D_v, tc::kBN))
    return SDPA_B200_ECUDA;  // detail recorded by make_map_f16
  const int64_t grid = ((p.S_q + 2 * tc::kBM - 1) / (2 * tc::kBM)) * p.B;
  if (int r = launch_tc(kern, grid, tc::kPairThreads, Cfg::kSmemBytes, st, mq, mk, mv, p)) return r;
  ++*launches;
  return SDPA_B200_OK;
}

template <int DQK, int DV>
int launch_pair_fwd(const Params& p, cudaStream_t st, int* launches) {
  // A single 128-row query tile per batch row leaves half of a pair idle:
  // the one-tile kernel serves those shapes.
  if (p.S_q <= tc::kBM) return launch_tc_fwd<DQK, DV>(p, st, launches);
  if (p.H > 1)
    return p.dropout_on ? launch_pair_fwd_t<DQK, DV, true, true>(p, st, launches)
                        : launch_pair_fwd_t<DQK, DV, false, true>(p, st, launches);
  return p.dropout_on ? launch_pair_fwd_t<DQK, DV, true, false>(p, st, launches)
                      : launch_pair_fwd_t<DQK, DV, false, false>(p, st, launches);
}

// Paired tiles share every K/V tile between two 128-row query tiles, but
// halve the number of CTAs.  With a causal mask and few batch rows (a batch
// sharded over many GPUs) the paired grid is about one wave of CTAs of very
// unequal length, and the one-tile kernel is faster (cfg4 rows on one GPU:
// 4 rows 593 vs 397 TFLOP/s forward; 8 rows 686 vs 788 the other way round;
// non-causal 16 x 2048 rows still favour pairs, 665 vs 549).  Causal problems
// use pairs from pair_min_ctas() paired CTAs on.
int64_t pair_min_ctas() {
  static const int64_t v = [] {
    const char* e = std::getenv("SDPA_B200_FWD_PAIR_MIN_CTAS");
    return e ? std::atoll(e) : static_cast<int64_t>(200);
  }();
  return v;
}

int tc_fwd_dispatch(const Params& p, cudaStream_t st, int* launches) {
  const int64_t pair_ctas = ((p.S_q + 2 * tc::kBM - 1) / (2 * tc::kBM)) * p.B;
  if (!std::getenv("SDPA_B200_FWD_SINGLE") && (!p.causal || pair_ctas >= pair_min_ctas())) {
    const bool q128 = p.D_qk > 64, v128 = p.D_v > 64;
    if (q128 && v128) return launch_pair_fwd<128, 128>(p, st, launches);
    if (q128) return launch_pair_fwd<128, 64>(p, st, launches);
    if (v128) return launch_pair_fwd<64, 128>(p, st, launches);
    return launch_pair_fwd<64, 64>(p, st, launches);
  }
  const bool q128 = p.D_qk > 64, v128 = p.D_v > 64;
  if (q128 && v128) return launch_tc_fwd<128, 128>(p, st, launches);
  if (q128) return launch_tc_fwd<128, 64>(p, st, launches);
  if (v128) return launch_tc_fwd<64, 128>(p, st, launches);
  return launch_tc_fwd<64, 64>(p, st, launches);
}


}  // namespace

int sdpa_b200::launch_fwd_tc(const Params& p, cudaStream_t st, int* launches) { return tc_fwd_dispatch(p, st, launches); }

SDPA_B200_STATUS_EXCHANGE(fwd_tc)
