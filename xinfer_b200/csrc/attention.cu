// Prefix attention for the xinfer attention operators on sm_100a: the contract of
// xinfer::flash_attention and xinfer::batched_flash_attention
// (compiler/common/kernels/attention.cpp:14-124) without ATen's FlashAttention.
//
// For batch row b, query t (0 <= t < count_b) sits at position L_b - count_b + t of a KV prefix of
// L_b valid slots and attends to slots 0..L_b - count_b + t (lower-right causal); query head h
// reads KV head h / (Hq / Hkv) (grouped-query attention without expanding K/V). Queries at
// t >= count_b produce zeros. Nothing outside the valid prefix or the row's own cache is read.
//
// Numerics follow FlashAttention-2: fp32 scores, exponentials computed as exp2 of scores scaled by
// scale * log2(e), running maximum per 64-key block, fp32 row sums of the unrounded
// probabilities, probabilities rounded to bf16 for the P.V product (fp32 accumulation), output
// divided by the row sum and rounded to bf16.
//
// Head dims 64, 128 and 256 use a tensor-core kernel: a CTA of 4 warps owns 64 queries of one
// head; K/V tiles of 64 keys are staged in shared memory with cp.async (16-byte chunks XOR-swizzled
// by key so that ldmatrix reads are free of bank conflicts), double buffered; Q.K^T and P.V are
// mma.sync m16n8k16 bf16 products and P stays in registers between the two. Other head dims
// (multiples of 8 up to 256) use a warp-per-query kernel with the same rounding points.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "xb_host.h"


namespace xbattn {

typedef __nv_bfloat16 bf16;
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  const bf16 *q, *k, *v;
  bf16 *out;
  long long qs_b, qs_h, qs_t, ks_b, ks_h, ks_t, vs_b, vs_h, vs_t;  // element strides
  int B, HQ, HKV, T, C, D;
  const int *cu;       // device [2, B + 1] cumulative query / KV lengths, or nullptr
  int count, length;   // used when cu == nullptr
  float scale_log2;    // scale * log2(e)
  const int *blocks;   // cache row of each batch row, or nullptr (row b)
  long long blocks_stride;
};

__device__ __forceinline__ int cache_row(const Params &p, int b) {
  return p.blocks ? p.blocks[(long long)b * p.blocks_stride] : b;
}

__device__ __forceinline__ void row_extent(const Params &p, int b, int &count, int &length) {
  if (p.cu) {
    count = p.cu[b + 1] - p.cu[b];
    length = p.cu[p.B + 1 + b + 1] - p.cu[p.B + 1 + b];
  } else {
    count = p.count;
    length = p.length;
  }
}

__device__ __forceinline__ uint32_t smem_u32(const void *ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
  const int bytes = valid ? 16 : 0;  // zero-fill rows beyond the valid prefix
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

constexpr int BM = 64, BN = 64, NWARPS = 4;

// Byte offset of 16-byte chunk c of key row r in a [BN][D] tile (row = D * 2 bytes).
template <int D> __device__ __forceinline__ int swz(int r, int c) {
  return r * (D * 2) + ((c ^ (r & 7)) << 4);
}

template <int D>
__global__ void __launch_bounds__(NWARPS * 32) attn_mma_kernel(const Params p) {
  constexpr int CH = D / 8;         // 16-byte chunks per key row
  constexpr int KB = D / 16;        // 16-dim blocks
  constexpr int TILE = BN * D * 2;  // bytes of one K or V tile
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char *ks = smem, *vs = smem + 2 * TILE, *qs = smem + 4 * TILE;  // K, V: 2 buffers each
  const int b = blockIdx.z, h = blockIdx.y, m0 = blockIdx.x * BM;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  int count, length;
  row_extent(p, b, count, length);
  const int kvh = h / (p.HQ / p.HKV);
  bf16 *out = p.out + (((long long)b * p.HQ + h) * p.T) * D;
  const int q0 = m0 + warp * 16;  // this warp's first query
  if (m0 >= count) {
    // every query of this CTA is beyond the row's count: zeros
    for (int i = threadIdx.x; i < BM * D / 8; i += NWARPS * 32) {
      const int r = m0 + i / (D / 8);
      if (r < p.T) reinterpret_cast<uint4 *>(out + (long long)r * D)[i % (D / 8)] = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const int shift = length - count;  // position of query t is shift + t
  const int last_q = min(count, m0 + BM) - 1;
  const int kv_end = shift + last_q + 1;  // keys [0, kv_end) are visible to some query here
  const int nblk = (kv_end + BN - 1) / BN;
  const int cb = cache_row(p, b);
  const bf16 *kg = p.k + (long long)cb * p.ks_b + (long long)kvh * p.ks_h;
  const bf16 *vg = p.v + (long long)cb * p.vs_b + (long long)kvh * p.vs_h;

  auto load_tile = [&](int blk, int buf) {
    const int k0 = blk * BN;
    for (int i = threadIdx.x; i < BN * CH; i += NWARPS * 32) {
      const int r = i / CH, c = i % CH;
      const int key = k0 + r;
      const bool ok = key < kv_end;
      const long long kk = ok ? key : 0;
      cp_async16(ks + buf * TILE + swz<D>(r, c), kg + kk * p.ks_t + c * 8, ok);
      cp_async16(vs + buf * TILE + swz<D>(r, c), vg + kk * p.vs_t + c * 8, ok);
    }
    cp_commit();
  };

  // the CTA's 64 queries (rows beyond count as zeros), swizzled like the K/V tiles
  {
    const bf16 *qg = p.q + (long long)b * p.qs_b + (long long)h * p.qs_h;
    for (int i = threadIdx.x; i < BM * CH; i += NWARPS * 32) {
      const int r = i / CH, c = i % CH;
      const bool ok = m0 + r < count;
      cp_async16(qs + swz<D>(r, c), qg + (long long)(ok ? m0 + r : 0) * p.qs_t + c * 8, ok);
    }
    cp_commit();
  }
  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int pos0 = shift + q0 + g, pos1 = pos0 + 8;  // positions of this thread's two query rows

  load_tile(0, 0);
  for (int blk = 0; blk < nblk; ++blk) {
    const int buf = blk & 1;
    if (blk + 1 < nblk) {
      load_tile(blk + 1, buf ^ 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint32_t kbase = smem_u32(ks + buf * TILE), vbase = smem_u32(vs + buf * TILE), qbase = smem_u32(qs);
    // S = Q K^T for 64 keys: 8 n-blocks of 8 keys
    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
#pragma unroll
    for (int kb = 0; kb < KB; ++kb) {
      // A fragment of Q: (rows 0..7, dims kb*16..+7), (rows 8..15, same), (rows 0..7, +8..15), (8..15, +8..15)
      uint32_t qa[4];
      {
        const int mi = lane >> 3, r = warp * 16 + (mi & 1) * 8 + (lane & 7), c = kb * 2 + (mi >> 1);
        ldsm_x4(qbase + swz<D>(r, c), qa[0], qa[1], qa[2], qa[3]);
      }
#pragma unroll
      for (int nb = 0; nb < 8; nb += 2) {
        // matrices: (keys nb*8.., dims kb*16..+7), (same keys, +8..15), (keys +8, dims lo), (keys +8, hi)
        const int mi = lane >> 3, r = (nb + (mi >> 1)) * 8 + (lane & 7), c = kb * 2 + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbase + swz<D>(r, c), b0, b1, b2, b3);
        mma16816(s[nb], qa[0], qa[1], qa[2], qa[3], b0, b1);
        mma16816(s[nb + 1], qa[0], qa[1], qa[2], qa[3], b2, b3);
      }
    }
    // mask (causal and prefix) and running softmax
    const int k0 = blk * BN;
    float bm[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + nb * 8 + 2 * t4 + (e & 1);
        const int pos = e < 2 ? pos0 : pos1;
        float x = s[nb][e] * p.scale_log2;
        if (key > pos || key >= kv_end) x = -INFINITY;
        s[nb][e] = x;
        bm[e >> 1] = fmaxf(bm[e >> 1], x);
      }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      bm[i] = fmaxf(bm[i], __shfl_xor_sync(0xffffffffu, bm[i], 1));
      bm[i] = fmaxf(bm[i], __shfl_xor_sync(0xffffffffu, bm[i], 2));
    }
    float corr[2], mnew[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mnew[i] = fmaxf(mrow[i], bm[i]);
      corr[i] = mnew[i] == -INFINITY ? 1.f : exp2f(mrow[i] - mnew[i]);
      mrow[i] = mnew[i];
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[4][4];  // P as A fragments: 4 key blocks of 16
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = mnew[e >> 1];
        const float pe = m == -INFINITY ? 0.f : exp2f(s[nb][e] - m);
        s[nb][e] = pe;
        rs[e >> 1] += pe;
      }
      const int kb = nb >> 1, hi = nb & 1;
      pa[kb][hi * 2 + 0] = pack_bf16(s[nb][0], s[nb][1]);
      pa[kb][hi * 2 + 1] = pack_bf16(s[nb][2], s[nb][3]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) lrow[i] = lrow[i] * corr[i] + rs[i];
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= corr[0]; o[j][1] *= corr[0];
      o[j][2] *= corr[1]; o[j][3] *= corr[1];
    }
    // O += P V: 4 key blocks of 16, D / 8 dim blocks of 8
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) {
#pragma unroll
      for (int j = 0; j < D / 8; j += 2) {
        // matrices (transposed): (keys kb*16..+7, dims j*8..), (keys +8.., dims j*8..),
        // (keys kb*16.., dims (j+1)*8..), (keys +8.., dims (j+1)*8..)
        const int mi = lane >> 3, r = kb * 16 + (mi & 1) * 8 + (lane & 7), c = j + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + swz<D>(r, c), b0, b1, b2, b3);
        // A fragment: (row g, keys 2t..), (row g+8, keys 2t..), (row g, keys 8+2t..), (row g+8, 8+2t..)
        mma16816(o[j], pa[kb][0], pa[kb][1], pa[kb][2], pa[kb][3], b0, b1);
        mma16816(o[j + 1], pa[kb][0], pa[kb][1], pa[kb][2], pa[kb][3], b2, b3);
      }
    }
    __syncthreads();  // this buffer is refilled two blocks later
  }
  // row sums over the quad, normalise, store bf16
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    lrow[i] += __shfl_xor_sync(0xffffffffu, lrow[i], 1);
    lrow[i] += __shfl_xor_sync(0xffffffffu, lrow[i], 2);
  }
  const int r0 = q0 + g, r1 = q0 + g + 8;
  const float inv0 = lrow[0] > 0.f ? 1.f / lrow[0] : 0.f, inv1 = lrow[1] > 0.f ? 1.f / lrow[1] : 0.f;
#pragma unroll
  for (int j = 0; j < D / 8; ++j) {
    const int c = j * 8 + 2 * t4;
    if (r0 < p.T)
      *reinterpret_cast<uint32_t *>(out + (long long)r0 * D + c) =
          r0 < count ? pack_bf16(o[j][0] * inv0, o[j][1] * inv0) : 0u;
    if (r1 < p.T)
      *reinterpret_cast<uint32_t *>(out + (long long)r1 * D + c) =
          r1 < count ? pack_bf16(o[j][2] * inv1, o[j][3] * inv1) : 0u;
  }
}

// Any head dim that is a multiple of 8 up to 256: one warp per (row, head, query), 64-key blocks
// with the same rounding points (block maximum, fp32 row sum, bf16 probabilities for P.V).
__global__ void attn_generic_kernel(const Params p) {
  const int warps = blockDim.x >> 5;
  const int t = blockIdx.x * warps + (threadIdx.x >> 5), h = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, D = p.D;
  if (t >= p.T) return;
  int count, length;
  row_extent(p, b, count, length);
  bf16 *out = p.out + ((((long long)b * p.HQ + h) * p.T) + t) * D;
  if (t >= count) {
    for (int d = lane; d < D; d += 32) out[d] = __float2bfloat16(0.f);
    return;
  }
  const int kvh = h / (p.HQ / p.HKV), pos = length - count + t;
  const bf16 *qr = p.q + (long long)b * p.qs_b + (long long)h * p.qs_h + (long long)t * p.qs_t;
  const int cb = cache_row(p, b);
  const bf16 *kg = p.k + (long long)cb * p.ks_b + (long long)kvh * p.ks_h;
  const bf16 *vg = p.v + (long long)cb * p.vs_b + (long long)kvh * p.vs_h;
  float q[8], o[8];
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    q[i] = d < D ? __bfloat162float(qr[d]) : 0.f;
    o[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int k0 = 0; k0 <= pos; k0 += BN) {
    const int kend = min(pos + 1, k0 + BN);
    float bm = -INFINITY;
    for (int key = k0; key < kend; ++key) {
      float sc = 0.f;
      for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < D) sc = fmaf(q[i], __bfloat162float(kg[(long long)key * p.ks_t + d]), sc);
      }
      for (int off = 16; off; off >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
      bm = fmaxf(bm, sc * p.scale_log2);
    }
    const float mn = fmaxf(m, bm), corr = m == -INFINITY ? 1.f : exp2f(m - mn);
    m = mn;
    l *= corr;
    for (int i = 0; i < 8; ++i) o[i] *= corr;
    for (int key = k0; key < kend; ++key) {
      float sc = 0.f;
      for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < D) sc = fmaf(q[i], __bfloat162float(kg[(long long)key * p.ks_t + d]), sc);
      }
      for (int off = 16; off; off >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
      const float pe = exp2f(sc * p.scale_log2 - m);
      l += pe;
      const float pb = __bfloat162float(__float2bfloat16(pe));
      for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < D) o[i] = fmaf(pb, __bfloat162float(vg[(long long)key * p.vs_t + d]), o[i]);
      }
    }
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    if (d < D) out[d] = __float2bfloat16(o[i] * inv);
  }
}

template <int D> static cudaError_t launch_mma(const Params &p, cudaStream_t st) {
  const int smem = 4 * BN * D * 2 + BM * D * 2;
  static bool configured = false;  // per template instance
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_mma_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid((p.T + BM - 1) / BM, p.HQ, p.B);
  attn_mma_kernel<D><<<grid, NWARPS * 32, smem, st>>>(p);
  return cudaGetLastError();
}

} // namespace xbattn

extern "C" int xb_prefix_attention(const XbAttentionArgs *a, void *stream) {
  using namespace xbattn;
  if (!a || !a->q || !a->k || !a->v || !a->out) return xb::fail(XB_ERR_INVALID, "null argument");
  if (a->batch < 1 || a->q_heads < 1 || a->kv_heads < 1 || a->q_heads % a->kv_heads)
    return xb::fail(XB_ERR_INVALID, "Query heads must be a positive multiple of KV heads");
  if (a->head_dim < 8 || a->head_dim > 256 || a->head_dim % 8)
    return xb::fail(XB_ERR_INVALID, "Flash head dimension must be a multiple of 8 in 8..256");
  if (a->q_tokens < 1 || a->q_tokens > 512) return xb::fail(XB_ERR_INVALID, "Unsupported Q shape");
  if (a->capacity < 1) return xb::fail(XB_ERR_INVALID, "Invalid capacity");
  if (!a->cu_offsets && (a->count < 1 || a->count > a->q_tokens || a->length < a->count ||
                         a->length > a->capacity))
    return xb::fail(XB_ERR_INVALID, "Invalid valid-prefix length");
  const long long *s = a->strides;  // q (b, h, t), k (b, h, t), v (b, h, t), in elements
  for (int i = 0; i < 9; ++i)
    if (s[i] % 8) return xb::fail(XB_ERR_INVALID, "strides must keep 16-byte rows");
  if (((uintptr_t)a->q | (uintptr_t)a->k | (uintptr_t)a->v | (uintptr_t)a->out) & 15)
    return xb::fail(XB_ERR_INVALID, "tensors must be 16-byte aligned");
  Params p;
  p.q = (const bf16 *)a->q; p.k = (const bf16 *)a->k; p.v = (const bf16 *)a->v; p.out = (bf16 *)a->out;
  p.qs_b = s[0]; p.qs_h = s[1]; p.qs_t = s[2];
  p.ks_b = s[3]; p.ks_h = s[4]; p.ks_t = s[5];
  p.vs_b = s[6]; p.vs_h = s[7]; p.vs_t = s[8];
  p.B = a->batch; p.HQ = a->q_heads; p.HKV = a->kv_heads; p.T = a->q_tokens; p.C = a->capacity;
  p.D = a->head_dim;
  p.cu = a->cu_offsets;
  p.count = a->count;
  p.length = a->length;
  p.scale_log2 = a->scale * kLog2e;
  p.blocks = a->blocks;
  p.blocks_stride = a->blocks_stride;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e;
  switch (p.D) {
  case 64: e = launch_mma<64>(p, st); break;
  case 128: e = launch_mma<128>(p, st); break;
  case 256: e = launch_mma<256>(p, st); break;
  default: {
    dim3 grid((p.T + 3) / 4, p.HQ, p.B);
    attn_generic_kernel<<<grid, 128, 0, st>>>(p);
    e = cudaGetLastError();
  }
  }
  if (e != cudaSuccess) return xb::fail(XB_ERR_CUDA, std::string("attention launch: ") + cudaGetErrorString(e));
  return XB_OK;
}
