// Kernels of one or two batch rows for wide models (hidden size >= kWideHidden): the decode
// megakernel whose GEMV stages with few rows per ring slot and at least one tile per consumer warp
// run one tile per warp over all of K (Consumer::tile_loop_fma with LK = 1). A separate
// instantiation, so that the standard kernel's code and registers are untouched.
#include "decode_kernel.cuh"

namespace xb {

cudaError_t launch_wide(int NB, const StepParams &prm, size_t smem, int ncta, cudaStream_t stream) {
  return NB == 1 ? launch_decode<1, 0, 0, 1>(prm, smem, ncta, stream) : launch_decode<2, 0, 0, 1>(prm, smem, ncta, stream);
}

cudaError_t set_fault_wide(int stage, unsigned long long limit) { return set_fault_constants(stage, limit); }

} // namespace xb
