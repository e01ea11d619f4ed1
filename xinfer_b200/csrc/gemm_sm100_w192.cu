// The 128 x 192 configuration of the prefill GEMM (gemm_sm100.cuh), in its own translation unit so
// that the configurations compile in parallel.
#include "gemm_sm100.cuh"

namespace xbgemm {
int run_wide192(int m, int n, int k, const void *x, const void *w, void *out, long long ldo, cudaStream_t st,
               int device) {
  return run<Wide192>(m, n, k, x, w, out, ldo, st, device);
}
} // namespace xbgemm
