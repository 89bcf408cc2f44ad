// Templated launchers of the SIMT kernels, instantiated per dtype and
// direction by simt_{fwd,bwd}_{f16,f32}.cu so they compile in parallel.
#pragma once
#include "host.cuh"
#include "ptx.cuh"
#include "simt.cuh"

namespace sdpa_b200 {
namespace simt_launch {
using namespace sdpa_b200::host;

template <typename T, int DM>
int launch_simt_fwd(const Params& p, cudaStream_t st, int* launches) {
  const int64_t grid = ((p.S_q + simt::kFwdRows - 1) / simt::kFwdRows) * p.B;
  if (grid > 0x7fffffffLL) return SDPA_B200_EINVAL;
  simt::fwd_kernel<T, DM><<<static_cast<unsigned>(grid), simt::kFwdRows, 0, st>>>(p);
  ++*launches;
  return launch_result();
}

template <typename T>
int simt_fwd_dispatch(const Params& p, cudaStream_t st, int* launches) {
  switch (dmax_bucket(p.D_qk > p.D_v ? p.D_qk : p.D_v)) {
    case 8: return launch_simt_fwd<T, 8>(p, st, launches);
    case 16: return launch_simt_fwd<T, 16>(p, st, launches);
    case 32: return launch_simt_fwd<T, 32>(p, st, launches);
    case 64: return launch_simt_fwd<T, 64>(p, st, launches);
    default: return launch_simt_fwd<T, 128>(p, st, launches);
  }
}

// ---------------------------------------------------------------- backward
template <typename T, int DM>
int launch_simt_bwd(const Params& p, cudaStream_t st, int* launches) {
  static std::atomic<uint64_t> attr_kv{0}, attr_q{0};
  const int64_t rows = p.B * p.S_q;
  if (rows > 0) {
    simt::delta_kernel<T><<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(p);
    ++*launches;
    if (int r = launch_result()) return r;
  }
  const size_t smkv = simt::dkdv_smem<DM>(), smq = simt::dq_smem<DM>();
  if (cudaError_t e = ensure_smem(simt::dkdv_kernel<T, DM>, smkv, attr_kv)) return cuda_failure("shared-memory attribute", e);
  if (cudaError_t e = ensure_smem(simt::dq_kernel<T, DM>, smq, attr_q)) return cuda_failure("shared-memory attribute", e);
  const int64_t gkv = ((p.S_kv + simt::kBwdRows - 1) / simt::kBwdRows) * p.B;
  const int64_t gq = ((p.S_q + simt::kBwdRows - 1) / simt::kBwdRows) * p.B;
  if (gkv > 0x7fffffffLL || gq > 0x7fffffffLL) return SDPA_B200_EINVAL;
  if (gkv > 0) {
    simt::dkdv_kernel<T, DM><<<static_cast<unsigned>(gkv), simt::kBwdRows * simt::dkdv_split<DM>(), smkv, st>>>(p);
    ++*launches;
    if (int r = launch_result()) return r;
  }
  if (gq > 0) {
    simt::dq_kernel<T, DM><<<static_cast<unsigned>(gq), simt::kBwdRows, smq, st>>>(p);
    ++*launches;
    if (int r = launch_result()) return r;
  }
  return SDPA_B200_OK;
}

template <typename T>
int simt_bwd_dispatch(const Params& p, cudaStream_t st, int* launches) {
  switch (dmax_bucket(p.D_qk > p.D_v ? p.D_qk : p.D_v)) {
    case 8: return launch_simt_bwd<T, 8>(p, st, launches);
    case 16: return launch_simt_bwd<T, 16>(p, st, launches);
    case 32: return launch_simt_bwd<T, 32>(p, st, launches);
    case 64: return launch_simt_bwd<T, 64>(p, st, launches);
    default: return launch_simt_bwd<T, 128>(p, st, launches);
  }
}


}  // namespace simt_launch
}  // namespace sdpa_b200
