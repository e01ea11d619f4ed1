// Dense bf16 GEMM of the prefill projections (out[M, N] = x[M, K] . W[N, K]^T, fp32 accumulation,
// one rounding to bf16): the choice among the sm_100a tensor-core configurations of
// gemm_sm100.cuh by shape, and a plain kernel for outputs the tensor-core epilogue cannot store
// (N or the row stride not a multiple of 8 elements).
#include "gemm_sm100.cuh"

namespace xbgemm {
int run_narrow(int m, int n, int k, const void *x, const void *w, void *out, long long ldo, cudaStream_t st,
               int device) {
  return run<Narrow>(m, n, k, x, w, out, ldo, st, device);
}
int run_rows(int m, int n, int k, const void *x, const void *w, void *out, long long ldo, cudaStream_t st, int device) {
  return run<Rows>(m, n, k, x, w, out, ldo, st, device);
}
} // namespace xbgemm

namespace {
// out[m, n] = x[m, :] . w[n, :] for shapes the tensor-core kernel cannot take (n not a multiple
// of 8): one warp per output element, fp32 sum, one rounding.
__global__ void gemm_rows_kernel(int m, int n, int k, const __nv_bfloat16 *x, const __nv_bfloat16 *w,
                                 __nv_bfloat16 *out, long long ldo) {
  const long long e = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (e >= (long long)m * n) return;
  const int row = (int)(e / n), col = (int)(e % n);
  const uint4 *a = reinterpret_cast<const uint4 *>(x + (long long)row * k);
  const uint4 *b = reinterpret_cast<const uint4 *>(w + (long long)col * k);
  float acc = 0.f;
  for (int c = lane; c < k / 8; c += 32) {
    const uint4 av = a[c], bv = b[c];
    const __nv_bfloat162 *ap = reinterpret_cast<const __nv_bfloat162 *>(&av);
    const __nv_bfloat162 *bp = reinterpret_cast<const __nv_bfloat162 *>(&bv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 af = __bfloat1622float2(ap[i]), bf = __bfloat1622float2(bp[i]);
      acc = fmaf(af.x, bf.x, acc);
      acc = fmaf(af.y, bf.y, acc);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[(long long)row * ldo + col] = __float2bfloat16_rn(acc);
}
} // namespace

int xb::gemm_bf16(int m, int n, int k, const void *x, const void *w, void *out, long long ldo, void *stream) {
  using namespace xbgemm;
  if (m < 1 || n < 1 || k < 1 || !x || !w || !out || ldo < n) return xb::fail(XB_ERR_INVALID, "invalid GEMM arguments");
  if (k % kAlign) return xb::fail(XB_ERR_INVALID, "GEMM K must be a multiple of 8");
  if (((uintptr_t)x | (uintptr_t)w) & 15) return xb::fail(XB_ERR_INVALID, "GEMM operands must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n % kAlign || ldo % kAlign || ((uintptr_t)out & 15)) {
    const long long total = (long long)m * n;
    gemm_rows_kernel<<<(unsigned)((total + 7) / 8), 256, 0, st>>>(m, n, k, static_cast<const __nv_bfloat16 *>(x),
                                                                 static_cast<const __nv_bfloat16 *>(w),
                                                                 static_cast<__nv_bfloat16 *>(out), ldo);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? XB_OK : xb::fail(XB_ERR_CUDA, std::string("GEMM launch: ") + cudaGetErrorString(e));
  }
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return xb::fail(XB_ERR_CUDA, "GEMM: no current device");
  // measured on B200 over the prefill shapes of Qwen3.5-0.8B / 4B at 512 tokens
  if (m <= 64) return run_rows(m, n, k, x, w, out, ldo, st, device);
  if (n < 2048) return run_narrow(m, n, k, x, w, out, ldo, st, device);
  // the width whose tiles need the fewest waves over the SMs, time ~ waves x width (wider on ties)
  static int sms = 0;
  if (!sms && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) sms = 148;
  const int widths[3] = {256, 192, 128};
  const RunFn fns[3] = {run_wide256, run_wide192, run_wide128};
  int best = 0;
  long long best_cost = -1;
  for (int i = 0; i < 3; ++i) {
    const long long tiles = (long long)((m + 127) / 128) * ((n + widths[i] - 1) / widths[i]);
    const long long cost = (tiles + sms - 1) / sms * widths[i];
    if (best_cost < 0 || cost < best_cost) { best = i; best_cost = cost; }
  }
  return fns[best](m, n, k, x, w, out, ldo, st, device);
}

extern "C" int xb_gemm_bf16(int32_t m, int32_t n, int32_t k, const void *x, const void *w, void *out,
                            void *stream) {
  return xb::gemm_bf16(m, n, k, x, w, out, n, stream);
}
