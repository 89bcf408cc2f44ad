// Translation unit: SIMT fwd kernels for float.
#include "simt_launch.cuh"

int sdpa_b200::launch_fwd_simt_f32(const Params& p, cudaStream_t st, int* launches) {
  return simt_launch::simt_fwd_dispatch<float>(p, st, launches);
}

SDPA_B200_STATUS_EXCHANGE(simt_fwd_f32)
