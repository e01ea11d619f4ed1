// One configuration of the prefill GEMM on sm_100a tensor cores:
//   out[M, N] (rows ldo elements apart) = x[M, K] . W[N, K]^T
// with fp32 accumulation in TMEM and one rounding to bf16, the rounding of the reference's cuBLAS
// linears as lowered by Inductor (a bf16 nn.Linear).
//
// The kernel is CUTLASS's SM100 warp-specialised GEMM (cute/CUTLASS 4.x templates): TMA tile
// loads of A and B into shared memory, MMAs issued by one thread with tcgen05.mma into a TMEM
// accumulator, a TMA-store epilogue. Every configuration runs one CTA per cluster (1 x 1 x 1), so
// each CTA loads its own operand tiles. Each translation unit instantiates one configuration.
#pragma once

#include "cutlass/cutlass.h"
#include "cute/tensor.hpp"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"

#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

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

template <class TileShape> struct Config {
  using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, TileShape, cute::Shape<cute::_1, cute::_1, cute::_1>,
      cutlass::epilogue::collective::EpilogueTileAuto, Accumulator, Accumulator, void, LayoutD, kAlign, ElementD,
      LayoutD, kAlign, cutlass::epilogue::TmaWarpSpecialized1Sm>::CollectiveOp;
  using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, ElementA, LayoutA, kAlign, ElementB, LayoutB, kAlign,
      Accumulator, TileShape, cute::Shape<cute::_1, cute::_1, cute::_1>,
      cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epilogue::SharedStorage))>,
      cutlass::gemm::KernelTmaWarpSpecialized1SmSm100>::CollectiveOp;
  using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Mainloop, Epilogue>;
  using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;
};

// Tiles (tokens x weight rows x K), chosen from a sweep on B200 over the Qwen3.5-0.8B / 4B
// prefill shapes at 512 tokens: 128-row tiles of 128, 192 or 256 weight rows for the wide
// projections (the width that needs the fewest tile waves), 64 x 64 for narrow outputs over long
// K (N < 2048), 64 x 128 for a few rows (the last token's lm_head).
using Wide128 = Config<Shape<_128, _128, _64>>;
using Wide192 = Config<Shape<_128, _192, _64>>;
using Wide256 = Config<Shape<_128, _256, _64>>;
using Narrow = Config<Shape<_64, _64, _64>>;
using Rows = Config<Shape<_64, _128, _64>>;

// Launch parameters (TMA descriptors included) of every (shape, operands, device) seen: a prefill
// chunk runs the same GEMMs on the same buffers again and again, and building the descriptors is
// host work comparable to the kernel itself at these sizes.
struct PlanKey {
  int m, n, k, device;
  long long ldo;
  const void *x, *w;
  void *out;
  bool operator==(const PlanKey &o) const { return std::memcmp(this, &o, sizeof(PlanKey)) == 0; }
};
struct PlanHash {
  size_t operator()(const PlanKey &p) const {
    size_t h = 1469598103934665603ull;
    const unsigned char *b = reinterpret_cast<const unsigned char *>(&p);
    for (size_t i = 0; i < sizeof(PlanKey); ++i) h = (h ^ b[i]) * 1099511628211ull;
    return h;
  }
};
constexpr size_t kMaxPlans = 4096;

template <class Cfg>
int run(int m, int n, int k, const void *x, const void *w, void *out, long long ldo, cudaStream_t st, int device) {
  using Gemm = typename Cfg::Gemm;
  using Kernel = typename Cfg::Kernel;
  static std::mutex mu;
  static std::unordered_map<PlanKey, typename Gemm::Params, PlanHash> plans;
  PlanKey key;
  std::memset(&key, 0, sizeof(key));
  key.m = m; key.n = n; key.k = k; key.device = device; key.ldo = ldo; key.x = x; key.w = w; key.out = out;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = plans.find(key);
    if (it != plans.end()) {
      if (Gemm::run(it->second, st) != cutlass::Status::kSuccess) return xb::fail(XB_ERR_CUDA, "GEMM launch failed");
      return XB_OK;
    }
  }
  using SA = typename Kernel::StrideA;
  using SB = typename Kernel::StrideB;
  using SD = typename Kernel::StrideD;
  const SA sa = cutlass::make_cute_packed_stride(SA{}, make_shape(m, k, 1));
  const SB sb = cutlass::make_cute_packed_stride(SB{}, make_shape(n, k, 1));
  SD sd = cutlass::make_cute_packed_stride(SD{}, make_shape(m, n, 1));
  cute::get<0>(sd) = ldo;
  typename Gemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                {m, n, k, 1},
                                {static_cast<const ElementA *>(x), sa, static_cast<const ElementB *>(w), sb},
                                {{1.f, 0.f}, nullptr, sd, static_cast<ElementD *>(out), sd}};
  Gemm gemm;
  if (gemm.can_implement(args) != cutlass::Status::kSuccess)
    return xb::fail(XB_ERR_UNSUPPORTED, "GEMM shape not supported by the sm_100 kernel");
  if (Gemm::get_workspace_size(args) != 0) return xb::fail(XB_ERR_UNSUPPORTED, "GEMM needs a workspace");
  if (gemm.initialize(args, nullptr, st) != cutlass::Status::kSuccess)
    return xb::fail(XB_ERR_CUDA, "GEMM initialisation failed");
  if (gemm.run(st) != cutlass::Status::kSuccess) return xb::fail(XB_ERR_CUDA, "GEMM launch failed");
  std::lock_guard<std::mutex> lock(mu);
  if (plans.size() >= kMaxPlans) plans.clear();
  plans.emplace(key, gemm.params());
  return XB_OK;
}

// one instantiation per translation unit (gemm_sm100.cu, gemm_sm100_w*.cu)
using RunFn = int (*)(int m, int n, int k, const void *x, const void *w, void *out, long long ldo, cudaStream_t st,
                      int device);
int run_wide128(int, int, int, const void *, const void *, void *, long long, cudaStream_t, int);
int run_wide192(int, int, int, const void *, const void *, void *, long long, cudaStream_t, int);
int run_wide256(int, int, int, const void *, const void *, void *, long long, cudaStream_t, int);
int run_narrow(int, int, int, const void *, const void *, void *, long long, cudaStream_t, int);
int run_rows(int, int, int, const void *, const void *, void *, long long, cudaStream_t, int);
} // namespace xbgemm
