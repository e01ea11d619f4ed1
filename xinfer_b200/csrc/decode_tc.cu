// Kernels of batch rows 4 and 8: the decode megakernel compiled with tensor-core GEMV tiles.
#define XB_TENSOR_TILES 1
#include "decode_kernel.cuh"

namespace xb {

cudaError_t launch_tensor_tiles(int NB, const StepParams &prm, size_t smem, int ncta, cudaStream_t stream) {
  return NB == 4 ? launch_decode<4>(prm, smem, ncta, stream) : launch_decode<8>(prm, smem, ncta, stream);
}

cudaError_t set_fault_tensor_tiles(int stage, unsigned long long limit) {
  return set_fault_constants(stage, limit);
}

} // namespace xb
