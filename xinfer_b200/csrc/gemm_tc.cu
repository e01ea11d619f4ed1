// Dense bf16 GEMM of the prefill projections on sm_100a tensor cores:
//   out[M, N] (rows ldo elements apart) = x[M, K] . W[N, K]^T
// with fp32 accumulation in tensor memory and one rounding to bf16, the rounding of the
// reference's cuBLAS linears as lowered by Inductor (a bf16 nn.Linear).
//
// One CTA per RM x BN output tile (BN = 64, 128 or 256; RM = 128, or 64 for narrow outputs, whose
// MMA rows 64..127 are computed from stale shared memory and discarded), 192 threads in three roles:
//   warp 0  TMA producer: RM x 64 tiles of x and BN x 64 tiles of W (K-major, 128-byte swizzle)
//           into a ring of shared-memory stages, completion counted on the stage's mbarrier;
//   warp 1  allocates BN columns of tensor memory; one lane issues four tcgen05.mma (M = 128,
//           N = BN, K = 16, bf16 x bf16 -> fp32) per stage and frees the stage with
//           tcgen05.commit, then commits the finished accumulator;
//   warps 2-5  epilogue: tcgen05.ld of their 32 accumulator rows, bf16 rounding, stores.
// Each CTA loads only its own tiles (no cluster). Every mbarrier wait is bounded: on expiry the
// waiting role records an error word and goes on, so a launch always ends.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "xb_host.h"

namespace xbtc {

constexpr int kBM = 128, kBK = 64;  // tokens per tile, K elements per stage (one 128-byte row)
constexpr int kThreads = 192;
constexpr unsigned long long kWaitNs = 2000000000ull;  // an mbarrier wait longer than this has expired
enum { GERR_WAIT = 1 };

__device__ unsigned g_error;  // error word of launches that were given none

// A stage holds RM rows of x then BN rows of W, 128 bytes each (64 bf16 of K). With RM = 64 the
// 128-row MMA operand A runs on into the W rows: its upper half is discarded. As many stages as
// fit in 227 KB of shared memory: the bytes in flight set the streaming rate.
template <int BN, int RM> struct Shape {
  static constexpr int kStageBytes = (RM + BN) * kBK * 2;
  static constexpr int kSmemMax = 227 * 1024, kExtra = 1024 /* alignment */ + 512 /* barriers, flags */;
  static constexpr int kStages = (kSmemMax - kExtra) / kStageBytes < 16 ? (kSmemMax - kExtra) / kStageBytes : 16;
  static constexpr int kSmem = kStages * kStageBytes + kExtra;
  static_assert(kStages >= 2 && kBM * kBK * 2 <= kStageBytes, "stage layout");
};

__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// bounded wait for the phase with the given parity; false on expiry, which sets the error word
// and the CTA's `broken` flag (later waits of the CTA then give up at once)
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity, unsigned *err, volatile int *broken,
                                          unsigned long long limit_ns = kWaitNs) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try(bar, parity))
    if (*broken || global_ns() - t0 > limit_ns) {
      atomicOr(err, (unsigned)GERR_WAIT);
      *broken = 1;
      return false;
    }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle layout written by TMA:
// rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), start address in 16-byte
// units, descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(unsigned addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFF) >> 4);   // start address, bits 0-13
  d |= (uint64_t)1 << 16;                   // leading byte offset (unused with swizzling)
  d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset, bits 32-45
  d |= (uint64_t)1 << 46;                   // version
  d |= (uint64_t)2 << 61;                   // 128-byte swizzle
  return d;
}

// Instruction descriptor of kind::f16: fp32 accumulator, bf16 A and B, both K-major, M x N.
__host__ __device__ constexpr uint32_t instr_desc(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D (+)= A . B^T for one K = 16 slice; `acc` = 0 overwrites D. No output lane is disabled.
__device__ __forceinline__ void mma_bf16(unsigned tmem_d, uint64_t a, uint64_t b, uint32_t idesc, unsigned acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(unsigned taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&v);
}

template <int BN, int RM>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w, int M, int N,
                int K, __nv_bfloat16 *out, long long ldo, unsigned *err) {
  using S = Shape<BN, RM>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *base = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(base + S::kStages * S::kStageBytes);
  uint64_t *empty = full + S::kStages;
  uint64_t *accum = empty + S::kStages;
  unsigned *tmem_slot = reinterpret_cast<unsigned *>(accum + 1);
  volatile int *broken = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * RM;
  const int nk = (K + kBK - 1) / kBK;
  constexpr unsigned kTxBytes = (RM + BN) * kBK * 2;  // bytes the two TMA loads of a stage bring
  if (!err) err = &g_error;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *broken = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // BN columns of tensor memory for the 128 x BN fp32 accumulator
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const unsigned tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % S::kStages;
        if (kb >= S::kStages) mbar_wait(&empty[s], ((kb / S::kStages) - 1) & 1, err, broken);
        unsigned char *a = base + s * S::kStageBytes;
        unsigned char *b = a + RM * kBK * 2;
        mbar_expect_tx(&full[s], kTxBytes);
        tma_load_2d(a, &map_x, kb * kBK, m0, &full[s]);
        tma_load_2d(b, &map_w, kb * kBK, n0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(kBM, BN);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % S::kStages;
        mbar_wait(&full[s], (kb / S::kStages) & 1, err, broken);
        tmem_fence_after();
        const unsigned a = smem_u32(base + s * S::kStageBytes);
        const unsigned b = a + RM * kBK * 2;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          mma_bf16(tmem, smem_desc(a + kk * 32), smem_desc(b + kk * 32), idesc, (kb | kk) != 0);
        mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
      }
      mma_commit(accum);
    }
  } else {
    // epilogue: warp w reads accumulator rows 32 (w % 4) .. + 31 (its tensor-memory lane quarter)
    const int quarter = warp & 3;
    mbar_wait(accum, 0, err, broken);
    tmem_fence_after();
    const int trow = quarter * 32 + lane, row = m0 + trow;
    if (trow < RM) {
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((unsigned)(quarter * 32) << 16) + c, r);
        if (row < M) {
          __nv_bfloat16 *dst = out + (long long)row * ldo + n0 + c;
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (n0 + c + 8 * q < N) {
              uint4 v;
              v.x = pack_bf16(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
              v.y = pack_bf16(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
              v.z = pack_bf16(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
              v.w = pack_bf16(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
              *reinterpret_cast<uint4 *>(dst + 8 * q) = v;
            }
        }
      }
    }
  }
  tmem_fence_before();
  __syncthreads();
  if (*broken && threadIdx.x == 0) {
    // a wait expired: before the shared memory is released, wait (bounded again) for the last
    // loads issued into every stage
    volatile int drain_broken = 0;
    for (int s = 0; s < S::kStages && s < nk; ++s) {
      const int last = s + (nk - 1 - s) / S::kStages * S::kStages;
      mbar_wait(&full[s], (last / S::kStages) & 1, err, &drain_broken, kWaitNs / 8);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tmem_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
  }
}

// out[m, n] = x[m, :] . w[n, :] for outputs the tensor-core epilogue does not store (N or the row
// stride not a multiple of 8 elements): one warp per output element, fp32 sum, one rounding.
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

// ---- host ----------------------------------------------------------------------------------

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// rows x cols bf16 matrix, row-major with rows `cols` apart; boxes of box_rows x 64
bool make_map(CUtensorMap *map, const void *ptr, long long rows, long long cols, int box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

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
struct Plan {
  CUtensorMap mx, mw;
  int bn, rm;  // tile width (weight rows) and height (token rows)
};
// Tensor maps of every (shape, operands, device) seen: a prefill chunk runs the same GEMMs on the
// same buffers again and again.
constexpr size_t kMaxPlans = 4096;
std::mutex plan_mu;
std::unordered_map<PlanKey, Plan, PlanHash> plans;

// the kernel's shared-memory allowance on the current device (set when a plan is made)
template <int BN, int RM> cudaError_t allow_smem() {
  return cudaFuncSetAttribute(gemm_kernel<BN, RM>, cudaFuncAttributeMaxDynamicSharedMemorySize, Shape<BN, RM>::kSmem);
}
cudaError_t allow_smem(int bn, int rm) {
  if (rm == 64) return bn == 256 ? allow_smem<256, 64>() : bn == 128 ? allow_smem<128, 64>() : allow_smem<64, 64>();
  return bn == 256 ? allow_smem<256, kBM>() : bn == 128 ? allow_smem<128, kBM>() : allow_smem<64, kBM>();
}

template <int BN, int RM>
int launch(const Plan &p, int m, int n, int k, void *out, long long ldo, unsigned *err, cudaStream_t st) {
  const dim3 grid((n + BN - 1) / BN, (m + RM - 1) / RM);
  gemm_kernel<BN, RM><<<grid, kThreads, Shape<BN, RM>::kSmem, st>>>(p.mx, p.mw, m, n, k,
                                                                 static_cast<__nv_bfloat16 *>(out), ldo, err);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? XB_OK : xb::fail(XB_ERR_CUDA, std::string("GEMM launch: ") + cudaGetErrorString(e));
}

// Tile height: 64 rows for a few tokens (the last token's lm_head) and for narrow outputs
// (N < 2048: out_proj, o_proj, down of the small models; twice the CTAs of 128-row tiles), else 128.
int rows_per_tile(int m, int n) { return m <= 64 || n < 2048 ? 64 : kBM; }
// Tile width: 64 for narrow outputs, else the one whose tiles need the fewest waves over the SMs
// weighted by the bytes a tile streams per K step (time ~ waves x (rows + width); the wider on
// ties).
int choose_bn(int m, int n, int rm, int sms) {
  if (n < 2048) return 64;
  const int widths[3] = {256, 128, 64};
  int best = 256;
  long long best_cost = -1;
  for (int w : widths) {
    const long long tiles = (long long)((m + rm - 1) / rm) * ((n + w - 1) / w);
    const long long cost = (tiles + sms - 1) / sms * (rm + w);
    if (best_cost < 0 || cost < best_cost) { best = w; best_cost = cost; }
  }
  return best;
}

} // namespace xbtc

int xb::gemm_bf16(int m, int n, int k, const void *x, const void *w, void *out, long long ldo, void *stream,
                  unsigned *err) {
  using namespace xbtc;
  if (m < 1 || n < 1 || k < 1 || !x || !w || !out || ldo < n) return xb::fail(XB_ERR_INVALID, "invalid GEMM arguments");
  if (k % 8) return xb::fail(XB_ERR_INVALID, "GEMM K must be a multiple of 8");
  if (((uintptr_t)x | (uintptr_t)w) & 15) return xb::fail(XB_ERR_INVALID, "GEMM operands must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n % 8 || ldo % 8 || ((uintptr_t)out & 15)) {
    const long long total = (long long)m * n;
    gemm_rows_kernel<<<(unsigned)((total + 7) / 8), 256, 0, st>>>(m, n, k, static_cast<const __nv_bfloat16 *>(x),
                                                                 static_cast<const __nv_bfloat16 *>(w),
                                                                 static_cast<__nv_bfloat16 *>(out), ldo);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? XB_OK : xb::fail(XB_ERR_CUDA, std::string("GEMM launch: ") + cudaGetErrorString(e));
  }
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return xb::fail(XB_ERR_CUDA, "GEMM: no current device");
  PlanKey key;
  std::memset(&key, 0, sizeof(key));
  key.m = m; key.n = n; key.k = k; key.device = device;
  key.ldo = ldo; key.x = x; key.w = w; key.out = out;
  Plan plan;
  bool found = false;
  {
    std::lock_guard<std::mutex> lock(plan_mu);
    auto it = plans.find(key);
    if (it != plans.end()) { plan = it->second; found = true; }
  }
  if (!found) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    plan.rm = rows_per_tile(m, n);
    plan.bn = choose_bn(m, n, plan.rm, sms);
    if (!make_map(&plan.mx, x, m, k, plan.rm) || !make_map(&plan.mw, w, n, k, plan.bn))
      return xb::fail(XB_ERR_CUDA, "GEMM: tensor map creation failed");
    const cudaError_t e = allow_smem(plan.bn, plan.rm);
    if (e != cudaSuccess) return xb::fail(XB_ERR_CUDA, std::string("GEMM: ") + cudaGetErrorString(e));
    std::lock_guard<std::mutex> lock(plan_mu);
    if (plans.size() >= kMaxPlans) plans.clear();
    plans.emplace(key, plan);
  }
  if (plan.rm == 64) {
    switch (plan.bn) {
      case 256: return launch<256, 64>(plan, m, n, k, out, ldo, err, st);
      case 128: return launch<128, 64>(plan, m, n, k, out, ldo, err, st);
      default: return launch<64, 64>(plan, m, n, k, out, ldo, err, st);
    }
  }
  switch (plan.bn) {
    case 256: return launch<256, kBM>(plan, m, n, k, out, ldo, err, st);
    case 128: return launch<128, kBM>(plan, m, n, k, out, ldo, err, st);
    default: return launch<64, kBM>(plan, m, n, k, out, ldo, err, st);
  }
}

extern "C" int xb_gemm_bf16(int32_t m, int32_t n, int32_t k, const void *x, const void *w, void *out,
                            void *stream) {
  return xb::gemm_bf16(m, n, k, x, w, out, n, stream, nullptr);
}
