// Kernels of one or two batch rows for wide models with head dimension 256 at long contexts: the
// one-tile-per-warp GEMV stages of decode_wide.cu and the position-block attention items of
// decode_long.cu in one instantiation.
#include "decode_kernel.cuh"

namespace xb {

cudaError_t launch_wide_long(int NB, const StepParams &prm, size_t smem, int ncta, cudaStream_t stream) {
  return NB == 1 ? launch_decode<1, 4, 8, 1>(prm, smem, ncta, stream) : launch_decode<2, 4, 8, 1>(prm, smem, ncta, stream);
}

cudaError_t set_fault_wide_long(int stage, unsigned long long limit) { return set_fault_constants(stage, limit); }

} // namespace xb
