// Translation unit: tcgen05 backward kernels
#include "host.cuh"
#include "ptx.cuh"
#include "simt.cuh"
#include "bwd_tc.cuh"

using namespace sdpa_b200;
using namespace sdpa_b200::host;

namespace {

// tcgen05 backward: dQ kernel (which also writes D = rowsum(dO*O)) -> dK/dV kernel.
template <int DQK, int DV, bool DROP, bool HEADS>
int launch_tc_bwd_t(const Params& p, cudaStream_t st, int* launches) {
  static std::atomic<uint64_t> attr_kv{0}, attr_q{0};
  using Cfg = tc::BwdCfg<DQK, DV>;
  auto kkv = tc::dkdv_kernel<DQK, DV, DROP, HEADS>;
  auto kq = tc::dq2_kernel<DQK, DV, DROP, HEADS>;
  using QCfg = tc::Dq2Cfg<DQK, DV>;
  if (cudaError_t e = ensure_smem(kkv, Cfg::kSmemBytes, attr_kv)) return cuda_failure("shared-memory attribute", e);
  if (cudaError_t e = ensure_smem(kq, QCfg::kSmemBytes, attr_q)) return cuda_failure("shared-memory attribute", e);
  CUtensorMap k128, v128, q64, do64, q128, do128;
  if (!make_map_f16(&k128, p.k, p.B, p.H, p.S_kv, p.D_qk, tc::kBwdRows) ||
      !make_map_f16(&v128, p.v, p.B, p.H, p.S_kv, p.D_v, tc::kBwdRows) ||
      !make_map_f16(&q64, p.q, p.B, p.H, p.S_q, p.D_qk, tc::kBwdTile) ||
      !make_map_f16(&do64, p.d_o, p.B, p.H, p.S_q, p.D_v, tc::kBwdTile) ||
      !make_map_f16(&q128, p.q, p.B, p.H, p.S_q, p.D_qk, tc::kBwdRows) ||
      !make_map_f16(&do128, p.d_o, p.B, p.H, p.S_q, p.D_v, tc::kBwdRows))
    return SDPA_B200_ECUDA;  // detail recorded by make_map_f16
  const int64_t gkv = ((p.S_kv + tc::kBwdRows - 1) / tc::kBwdRows) * p.B;
  const int64_t gq = ((p.S_q + tc::kBwdRows - 1) / tc::kBwdRows) * p.B;
  if (gkv > 0x7fffffffLL || gq > 0x7fffffffLL) return SDPA_B200_EINVAL;
  // dQ first: it also computes D = rowsum(dO * O) (into the workspace), which
  // the dK/dV kernel reads.
  sdpa_b200::record_bwd_event(0, st);
  if (int r = launch_tc(kq, gq, tc::kBwdTcThreads, QCfg::kSmemBytes, st, q128, do128, k128, v128, p)) return r;
  ++*launches;
  sdpa_b200::record_bwd_event(1, st);
  if (int r = launch_tc(kkv, gkv, tc::kBwdTcThreads, Cfg::kSmemBytes, st, k128, v128, q64, do64, p)) return r;
  ++*launches;
  sdpa_b200::record_bwd_event(2, st);
  sdpa_b200::record_bwd_event(3, st);
  return SDPA_B200_OK;
}

// HEADS: [B/H, S, H, D] tensors (4-D TMA maps); else contiguous [B, S, D].
template <int DQK, int DV>
int launch_tc_bwd(const Params& p, cudaStream_t st, int* launches) {
  if (p.H > 1)
    return p.dropout_on ? launch_tc_bwd_t<DQK, DV, true, true>(p, st, launches)
                        : launch_tc_bwd_t<DQK, DV, false, true>(p, st, launches);
  return p.dropout_on ? launch_tc_bwd_t<DQK, DV, true, false>(p, st, launches)
                      : launch_tc_bwd_t<DQK, DV, false, false>(p, st, launches);
}

int tc_bwd_dispatch(const Params& p, cudaStream_t st, int* launches) {
  const bool q128 = p.D_qk > 64, v128 = p.D_v > 64;
  if (q128 && v128) return launch_tc_bwd<128, 128>(p, st, launches);
  if (q128) return launch_tc_bwd<128, 64>(p, st, launches);
  if (v128) return launch_tc_bwd<64, 128>(p, st, launches);
  return launch_tc_bwd<64, 64>(p, st, launches);
}


}  // namespace

int sdpa_b200::launch_bwd_tc(const Params& p, cudaStream_t st, int* launches) { return tc_bwd_dispatch(p, st, launches); }

SDPA_B200_STATUS_EXCHANGE(bwd_tc)
