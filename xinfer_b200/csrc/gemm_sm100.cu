// Dense bf16 GEMM of the prefill projections on sm_100a tensor cores:
//   out[M, N] = x[M, K] . W[N, K]^T      (x: M tokens of activations, W: an HF [out, in] weight)
// with fp32 accumulation and one rounding to bf16, the rounding of the reference's cuBLAS
// linears as lowered by Inductor (a bf16 nn.Linear).
//
// The kernel is CUTLASS's SM100 warp-specialised GEMM (cute/CUTLASS 4.x templates): TMA tile
// loads of A and B into shared memory (one CTA per tile, cluster 1x1x1, so no multicast), MMAs
// issued by a single thread with tcgen05.mma into a TMEM accumulator, a TMA-store epilogue.
// Tiles of 128 (tokens) x 128 (weight rows) x 64.
#include "cutlass/cutlass.h"
#include "cute/tensor.hpp"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"

#include <string>

#include "xb_host.h"


namespace xbgemm {
using namespace cute;
using ElementA = cutlass::bfloat16_t;
using LayoutA = cutlass::layout::RowMajor;     // x [M, K]
using ElementB = cutlass::bfloat16_t;
using LayoutB = cutlass::layout::ColumnMajor;  // W [N, K] read as a K x N column-major matrix
using ElementD = cutlass::bfloat16_t;
using LayoutD = cutlass::layout::RowMajor;     // out [M, N]
using Accumulator = float;
constexpr int kAlign = 8;  // 16-byte rows
using TileShape = Shape<_128, _128, _64>;
using ClusterShape = Shape<_1, _1, _1>;
using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, TileShape, ClusterShape,
    cutlass::epilogue::collective::EpilogueTileAuto, Accumulator, Accumulator, void, LayoutD, kAlign,
    ElementD, LayoutD, kAlign, cutlass::epilogue::TmaWarpSpecialized1Sm>::CollectiveOp;
using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, ElementA, LayoutA, kAlign, ElementB, LayoutB,
    kAlign, Accumulator, TileShape, ClusterShape,
    cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epilogue::SharedStorage))>,
    cutlass::gemm::KernelTmaWarpSpecialized1SmSm100>::CollectiveOp;
using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Mainloop, Epilogue>;
using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;
} // namespace xbgemm

extern "C" int xb_gemm_bf16(int32_t m, int32_t n, int32_t k, const void *x, const void *w, void *out,
                            void *stream) {
  using namespace xbgemm;
  if (m < 1 || n < 1 || k < 1 || !x || !w || !out) return xb::fail(XB_ERR_INVALID, "invalid GEMM arguments");
  if (n % kAlign || k % kAlign) return xb::fail(XB_ERR_INVALID, "GEMM N and K must be multiples of 8");
  if (((uintptr_t)x | (uintptr_t)w | (uintptr_t)out) & 15)
    return xb::fail(XB_ERR_INVALID, "GEMM operands must be 16-byte aligned");
  using SA = typename Kernel::StrideA;
  using SB = typename Kernel::StrideB;
  using SD = typename Kernel::StrideD;
  const SA sa = cutlass::make_cute_packed_stride(SA{}, make_shape(m, k, 1));
  const SB sb = cutlass::make_cute_packed_stride(SB{}, make_shape(n, k, 1));
  const SD sd = cutlass::make_cute_packed_stride(SD{}, make_shape(m, n, 1));
  typename Gemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                {m, n, k, 1},
                                {static_cast<const ElementA *>(x), sa, static_cast<const ElementB *>(w), sb},
                                {{1.f, 0.f}, nullptr, sd, static_cast<ElementD *>(out), sd}};
  Gemm gemm;
  if (gemm.can_implement(args) != cutlass::Status::kSuccess)
    return xb::fail(XB_ERR_UNSUPPORTED, "GEMM shape not supported by the sm_100 kernel");
  if (Gemm::get_workspace_size(args) != 0) return xb::fail(XB_ERR_UNSUPPORTED, "GEMM needs a workspace");
  if (gemm.initialize(args, nullptr, static_cast<cudaStream_t>(stream)) != cutlass::Status::kSuccess)
    return xb::fail(XB_ERR_CUDA, "GEMM initialisation failed");
  if (gemm.run(static_cast<cudaStream_t>(stream)) != cutlass::Status::kSuccess)
    return xb::fail(XB_ERR_CUDA, "GEMM launch failed");
  return XB_OK;
}
