// Device helpers shared by the xinfer_b200 kernels: bf16 packing, coherent/streaming loads,
// mbarrier + bulk-copy (TMA) primitives for sm_100a, bounded waits on %globaltimer.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace xb {

typedef __nv_bfloat16 bf16;

// Bounded waits: every spin in these kernels gives up after this many nanoseconds, records an
// error word in the workspace and lets the kernel return (no trap, no endless loop).
constexpr uint64_t kWaitLimitNs = 2000000000ull;
// Waits shorter than this never leave the fast path (no global loads besides the polled data).
constexpr uint64_t kSlowWaitNs = 20000ull;

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ float bf(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ bf16 tobf(float x) { return __float2bfloat16_rn(x); }
// Round an fp32 value through bf16 (the reference's tensor dtype at that point).
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__device__ __forceinline__ void unpack8(const uint4 &v, float (&f)[8]) {
  f[0] = bf_lo(v.x); f[1] = bf_hi(v.x);
  f[2] = bf_lo(v.y); f[3] = bf_hi(v.y);
  f[4] = bf_lo(v.z); f[5] = bf_hi(v.z);
  f[6] = bf_lo(v.w); f[7] = bf_hi(v.w);
}

// acc + sum_{e=0..7} w[e] * x[e] for eight bf16 pairs, accumulated in order e = 0..7 with one
// rounding per step: fma with bf16 multiplicands and an fp32 addend/result, so no unpacking.
__device__ __forceinline__ float dot8_bf16(const uint4 &w, const uint4 &x, float acc) {
  asm("{\n\t"
      ".reg .b16 w0, w1, w2, w3, w4, w5, w6, w7, x0, x1, x2, x3, x4, x5, x6, x7;\n\t"
      "mov.b32 {w0, w1}, %1;\n\tmov.b32 {w2, w3}, %2;\n\t"
      "mov.b32 {w4, w5}, %3;\n\tmov.b32 {w6, w7}, %4;\n\t"
      "mov.b32 {x0, x1}, %5;\n\tmov.b32 {x2, x3}, %6;\n\t"
      "mov.b32 {x4, x5}, %7;\n\tmov.b32 {x6, x7}, %8;\n\t"
      "fma.rn.f32.bf16 %0, w0, x0, %0;\n\tfma.rn.f32.bf16 %0, w1, x1, %0;\n\t"
      "fma.rn.f32.bf16 %0, w2, x2, %0;\n\tfma.rn.f32.bf16 %0, w3, x3, %0;\n\t"
      "fma.rn.f32.bf16 %0, w4, x4, %0;\n\tfma.rn.f32.bf16 %0, w5, x5, %0;\n\t"
      "fma.rn.f32.bf16 %0, w6, x6, %0;\n\tfma.rn.f32.bf16 %0, w7, x7, %0;\n\t}"
      : "+f"(acc)
      : "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w), "r"(x.x), "r"(x.y), "r"(x.z), "r"(x.w));
  return acc;
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // .x = a (low), .y = b (high)
  return *reinterpret_cast<uint32_t *>(&h);
}

// Loads of data written earlier in the same launch by other CTAs: bypass L1 (.cg).
__device__ __forceinline__ bf16 ldcg_bf(const bf16 *p) {
  unsigned short v;
  asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return __ushort_as_bfloat16(v);
}
__device__ __forceinline__ float ldcg_f(const float *p) { return __ldcg(p); }
__device__ __forceinline__ uint4 ldcg_u4(const void *p) {
  return __ldcg(reinterpret_cast<const uint4 *>(p));
}
// Streaming loads of data that is read-only for the whole launch.
__device__ __forceinline__ uint4 ldnc_u4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldnc_u2(const void *p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}

// Reads of the L2-coherent copy that the compiler may neither cache nor hoist (polling loops).
__device__ __forceinline__ uint4 ld_poll_u4(const void *p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ uint2 ld_poll_u2(const void *p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_poll_u32(const void *p) {
  unsigned v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Read-only data shared by several warps of a CTA (L1-allocating, non-coherent path).
__device__ __forceinline__ uint4 ldg_u4(const void *p) {
  return __ldg(reinterpret_cast<const uint4 *>(p));
}
__device__ __forceinline__ uint2 ldg_u2(const void *p) {
  return __ldg(reinterpret_cast<const uint2 *>(p));
}

// ---- tagged inter-stage words --------------------------------------------------------------
// A bf16 value travels with a 16-bit tag in one 32-bit word, (tag << 16) | bits, so a consumer
// that sees the expected tag also sees the value: no fence or flag is needed between stages.
// tag = (epoch mod 511) * 128 + (2 * layer + k) + 1 (layer < 64, k in {0, 1}): never 0, so a
// zeroed word never looks ready; distinct for every (layer, k) of one launch; and equal for two
// launches only when their epochs differ by a multiple of kTagPeriod. The kernel clears every
// tagged buffer at least once per kScrubInterval (< kTagPeriod) launches, so no word a launch
// polls can carry a stale tag equal to the one it waits for.
constexpr unsigned kTagPeriod = 511;
constexpr unsigned kScrubInterval = 256;
__device__ __forceinline__ unsigned tag_of(unsigned epoch, int layer, int k) {
  return (epoch % kTagPeriod) * 128u + (unsigned)(layer * 2 + k) + 1u;
}
// {fp32 value, tag} pairs travel as one 64-bit word (value in the low half), stored and loaded
// as 64-bit scalars (or as vectors of them), each single-copy atomic.
typedef unsigned long long u64;
__device__ __forceinline__ u64 ftag(float v, unsigned tag) {
  return ((u64)tag << 32) | (u64)__float_as_uint(v);
}
__device__ __forceinline__ float ftag_val(u64 w) { return __uint_as_float((unsigned)w); }
__device__ __forceinline__ unsigned ftag_tag(u64 w) { return (unsigned)(w >> 32); }
__device__ __forceinline__ void st_u64(u64 *p, u64 v) {
  asm volatile("st.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_u64x2(u64 *p, u64 a, u64 b) {
  asm volatile("st.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ u64 ldcg_u64(const u64 *p) {
  u64 v;
  asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ ulonglong2 ldcg_u64x2(const u64 *p) {
  ulonglong2 v;
  asm volatile("ld.global.cg.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ u64 ld_poll_u64(const u64 *p) {
  u64 v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ ulonglong2 ld_poll_u64x2(const u64 *p) {
  ulonglong2 v;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned tagged(float v, unsigned tag) {
  return (tag << 16) | (unsigned)__bfloat16_as_ushort(__float2bfloat16_rn(v));
}
__device__ __forceinline__ bool tag4_ok(const uint4 &v, unsigned tag) {
  return (v.x >> 16) == tag && (v.y >> 16) == tag && (v.z >> 16) == tag && (v.w >> 16) == tag;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(unsigned *p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_volatile(const unsigned *p) {
  return *reinterpret_cast<const volatile unsigned *>(p);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier (CTA scope) -----------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
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

// One-dimensional bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, `bytes` a multiple of 16; the destination is this CTA only.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

template <int N> __device__ __forceinline__ void named_sync(int id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "n"(N) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1)
    v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// torch.argmax order on a row: NaN is the maximum, ties keep the smallest index.
__device__ __forceinline__ bool argmax_better(float v, int i, float bv, int bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn)
    return !bn || i < bi;
  if (bn)
    return false;
  return v > bv || (v == bv && i < bi);
}

} // namespace xb
