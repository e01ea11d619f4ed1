// Kernels of one or two batch rows for long contexts: the decode megakernel with the split-KV
// attention items in position blocks (Consumer::attn_blocks), picked by the host when an item
// spans at least kAttBlockMin positions. A separate instantiation, so that the standard kernel's
// code and registers are untouched.
#include "decode_kernel.cuh"

namespace xb {

cudaError_t launch_long_attention(int NB, int kind, const StepParams &prm, size_t smem, int ncta,
                                  cudaStream_t stream) {
  if (kind == 1)
    return NB == 1 ? launch_decode<1, 2, 4>(prm, smem, ncta, stream) : launch_decode<2, 2, 4>(prm, smem, ncta, stream);
  return NB == 1 ? launch_decode<1, 4, 8>(prm, smem, ncta, stream) : launch_decode<2, 4, 8>(prm, smem, ncta, stream);
}

cudaError_t set_fault_long_attention(int stage, unsigned long long limit) {
  return set_fault_constants(stage, limit);
}

} // namespace xb
