// Translation unit: SIMT bwd kernels for __half.
#include "simt_launch.cuh"

int sdpa_b200::launch_bwd_simt_f16(const Params& p, cudaStream_t st, int* launches) {
  return simt_launch::simt_bwd_dispatch<__half>(p, st, launches);
}

SDPA_B200_STATUS_EXCHANGE(simt_bwd_f16)
