// Prefill of one row: ModelStep.forward with T > 1 tokens (compiler/qwen35/model.py:162-183,
// compiler/qwen3/model.py:70-95; exported as prefill.pt2 by compiler/qwen35/export.py:43-57).
//
// A sequence of launches on one stream: the embedding rows, then per layer
//   RMSNorm rows -> tensor-core GEMMs (xb_gemm_bf16, tcgen05) -> DeltaNet: conv/SiLU/l2-norm/gates
//   of every token in parallel, then the gated delta rule scanned over the tokens, gated RMSNorm,
//   out_proj GEMM | attention: q/k norm, RoPE, KV append, prefix attention over the cache,
//   sigmoid gate, o_proj GEMM -> residual add -> RMSNorm -> gate/up GEMMs -> SiLU*mul -> down GEMM
//   -> residual add,
// then the final norm of the last token, its lm_head GEMM and the argmax. Rounding points are the
// decode kernel's (bf16 tensors between ops, fp32 inside); the DeltaNet scan is the token-by-token
// recurrence (the reference's short path, recurrent.py:61-124) also for the chunks that the
// reference runs through its chunk-64 formulation (recurrent.py:234-281, chunked.py): the same
// gated delta rule, summed in another order.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>

#include "xb_device.cuh"
#include "xb_host.h"

namespace xbpre {
using namespace xb;

constexpr int kMaxTokens = 512;
constexpr int kArgmaxBlocks = 296;  // CTAs of the logits argmax
constexpr int kChunk = 32;  // tokens per step of the chunked gated delta rule
// per (chunk, head): T^-1 and M (column-major, [j][i]), A_i, beta_i, A_32 / A_j, A_32
constexpr int kRecFloats = 2 * kChunk * kChunk + 3 * kChunk + 32;
// the prefill workspace starts with the decode workspace's control words, so that
// xb_workspace_check reads its error word (word 64) the same way
constexpr int kCtlBytes = 1024;
enum { PERR_TOKEN = 4 };

struct Layout {
  size_t h, x, x2, out, proj, qn, kn, vv, beta, glog, rec, core, qatt, oatt, xlast, amax, total;
};

static int lin_channels(const XbGeometry &g) { return (2 * g.lin_key_heads + g.lin_value_heads) * g.lin_head_dim; }

// Row width of the projection buffer: the widest group of projections that read one input
// (DeltaNet qkv | z | b | a, attention q | k | v, MLP gate | up), each group's outputs side by side
// in one row per token, as the reference's packed linears produce them (pack_linears.py).
static int proj_width(const XbGeometry &g) {
  const bool q35 = g.family == XB_FAMILY_QWEN35;
  const int delta = q35 ? lin_channels(g) + g.lin_value_heads * g.lin_head_dim + 2 * g.lin_value_heads : 0;
  const int attn = g.num_q_heads * g.head_dim * (q35 ? 2 : 1) + 2 * g.num_kv_heads * g.head_dim;
  return std::max({delta, attn, 2 * g.intermediate});
}

static Layout layout(const XbGeometry &g, int T) {
  Layout L{};
  const bool q35 = g.family == XB_FAMILY_QWEN35;
  const int HVD = q35 ? g.lin_value_heads * g.lin_head_dim : 0;
  const int widest = std::max({g.hidden, g.intermediate, g.num_q_heads * g.head_dim, HVD});
  size_t off = kCtlBytes;
  auto take = [&](size_t bytes) { size_t o = off; off += (bytes + 255) & ~size_t(255); return o; };
  L.h = take((size_t)T * g.hidden * 2);
  L.x = take((size_t)T * widest * 2);
  L.x2 = take((size_t)T * widest * 2);
  L.out = take((size_t)T * g.hidden * 2);
  L.proj = take((size_t)T * proj_width(g) * 2);
  const size_t vec = q35 ? (size_t)T * HVD * 4 : 256;
  L.qn = take(vec);
  L.kn = take(vec);
  L.vv = take(vec);
  L.beta = take(q35 ? (size_t)T * g.lin_value_heads * 4 : 256);
  L.glog = take(q35 ? (size_t)T * g.lin_value_heads * 4 : 256);
  L.rec = take(q35 ? (size_t)((T + kChunk - 1) / kChunk) * g.lin_value_heads * kRecFloats * 4 : 256);
  L.core = take(q35 ? (size_t)T * HVD * 2 : 256);
  L.qatt = take((size_t)T * g.num_q_heads * g.head_dim * 2);
  L.oatt = take((size_t)T * g.num_q_heads * g.head_dim * 2);
  L.xlast = take((size_t)g.hidden * 2 + 16);
  L.amax = take(kArgmaxBlocks * 8);
  L.total = off;
  return L;
}

// ---- kernels -------------------------------------------------------------------------------

__global__ void embed_kernel(const int64_t *ids, const bf16 *embed, bf16 *h, int H, int V, unsigned *err) {
  const int t = blockIdx.x;
  const long long id = ids[t];
  const bool ok = id >= 0 && id < V;
  if (!ok && threadIdx.x == 0) atomicCAS(err, 0u, (unsigned)PERR_TOKEN);
  const uint4 *src = reinterpret_cast<const uint4 *>(embed + (ok ? id : 0) * (long long)H);
  uint4 *dst = reinterpret_cast<uint4 *>(h + (long long)t * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = ok ? src[c] : make_uint4(0, 0, 0, 0);
}

// Residual add and RMSNorm of rows: with `o`, h = bf16(h + o) first (the reference's residual
// add, both operands bf16) and h is written back; then out = RMSNorm(h) (HF Qwen3RMSNorm:
// w * bf16(x r); Qwen3_5RMSNorm: bf16(x r (1 + w))). 128 or 256 threads per row, each summing the
// squares of its 8-element chunks c and c + 256 in order. Row blockIdx.x + row0 of h is
// normalised into row blockIdx.x of out.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(bf16 *h, const bf16 *o, const bf16 *w, bf16 *out, int H,
                                                          float eps, int q35, int row0) {
  const int t = blockIdx.x + row0, tid = threadIdx.x, nc = H / 8, nt = blockDim.x;
  uint4 *row = reinterpret_cast<uint4 *>(h + (long long)t * H);
  const uint4 *orow = o ? reinterpret_cast<const uint4 *>(o + (long long)t * H) : nullptr;
  __shared__ float red[8];
  uint4 xv[2];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int c = tid + i * nt;
    xv[i] = c < nc ? row[c] : make_uint4(0, 0, 0, 0);
    float x[8];
    unpack8(xv[i], x);
    if (orow && c < nc) {
      float y[8];
      unpack8(orow[c], y);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = rbf(x[e] + y[e]);
      xv[i] = make_uint4(pack2(x[0], x[1]), pack2(x[2], x[3]), pack2(x[4], x[5]), pack2(x[6], x[7]));
      row[c] = xv[i];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (nt >> 5); ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)H + eps);
  uint4 *dst = reinterpret_cast<uint4 *>(out + (long long)blockIdx.x * H);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int c = tid + i * nt;
    if (c >= nc) continue;
    float x[8], wf[8], y[8];
    unpack8(xv[i], x);
    unpack8(reinterpret_cast<const uint4 *>(w)[c], wf);
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = q35 ? x[e] * r * (1.f + wf[e]) : wf[e] * rbf(x[e] * r);
    dst[c] = make_uint4(pack2(y[0], y[1]), pack2(y[2], y[3]), pack2(y[4], y[5]), pack2(y[6], y[7]));
  }
}

// act = bf16(bf16(silu(gate)) * up) (HF SiLU on a bf16 tensor, then the bf16 product), 8 values
// per thread; gate and up are the two halves of each [gate | up] projection row.
__global__ void __launch_bounds__(256) silu_mul_kernel(const bf16 *proj, bf16 *act, int I, int ld, int T) {
  const int n8 = I / 8;
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= (long long)T * n8) return;
  const long long t = i / n8;
  const int c = (int)(i % n8);
  const uint4 gv = reinterpret_cast<const uint4 *>(proj + t * ld)[c];
  const uint4 uv = reinterpret_cast<const uint4 *>(proj + t * ld + I)[c];
  float g[8], u[8], y[8];
  unpack8(gv, g);
  unpack8(uv, u);
#pragma unroll
  for (int e = 0; e < 8; ++e) y[e] = rbf(g[e] / (1.f + expf(-g[e]))) * u[e];
  reinterpret_cast<uint4 *>(act + t * I)[c] =
      make_uint4(pack2(y[0], y[1]), pack2(y[2], y[3]), pack2(y[4], y[5]), pack2(y[6], y[7]));
}

// The conv window after the last token: the last four inputs of [old window, tokens] for every
// channel (recurrent.py:43-52). Launched after every read of the old window, so in place is safe.
__global__ void conv_state_kernel(const bf16 *qkv, int ld, const bf16 *conv_in, bf16 *conv_out, int CH, int T) {
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= CH) return;
  bf16 w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int s = T - 4 + j;
    w[j] = s < 0 ? conv_in[(long long)ch * 4 + 4 + s] : qkv[(long long)s * ld + ch];
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) conv_out[(long long)ch * 4 + j] = w[j];
}

// ---- chunked gated delta rule ---------------------------------------------------------------
// The recurrence (recurrent.py:20-28), per value head with state S [dk, dv] fp32:
//   S_i = a_i S_{i-1} + k_i d_i^T,  d_i = b_i (v_i - a_i S_{i-1}^T k_i),  o_i = S_i^T q_i,
// evaluated 32 tokens at a time in the closed form of the reference's chunked path
// (chunked.py:17-160; chunk 64 there): with A_i = a_1 ... a_i inside the chunk,
//   (I + L) d = beta (v - A pk),  L_ij = beta_i (A_i / A_j) k_i.k_j  (j < i),  pk_i = k_i . S_0,
//   o_i = A_i q_i . S_0 + sum_{j<=i} (A_i / A_j) (q_i . k_j) d_j,
//   S_32 = A_32 S_0 + sum_j (A_32 / A_j) k_j d_j^T.
// A_i / A_j = exp(P_i - P_j) with P the in-order prefix sum of the log decays g. Tokens past the
// prompt are zero (g = 0, beta = 0, k = q = v = 0), which leaves S and every real token unchanged.
enum { REC_TINV = 0, REC_MO = kChunk * kChunk, REC_A = 2 * kChunk * kChunk, REC_BETA = REC_A + kChunk,
       REC_WS = REC_BETA + kChunk, REC_ALAST = REC_WS + kChunk };

// DeltaNet preparation (recurrent.py:32-58, 99-120; the long path's prepare_kernel,
// recurrent.py:127-189), one warp per (token, head part): part p < HK is query head p, p < 2 HK
// key head p - HK, else value head p - 2 HK. Lane l takes channels 4l..4l + 3 of the part: width-4
// causal conv over [old window, tokens] with fp32 FMAs in tap order, bf16, SiLU, bf16; q and k
// l2-normalised (q also scaled by dk^-0.5). The value-head warps also make beta = bf16(sigmoid(b))
// and the log decay g = -exp(A_log) * softplus(a + dt_bias), softplus threshold 20. Outputs fp32:
// q, k per key head [T, HK, 128], v per value head [T, HV, 128], beta and g [T, HV].
__global__ void __launch_bounds__(256) delta_prepare_kernel(
    const bf16 *qkv, const bf16 *bb, const bf16 *aa, int ld, const bf16 *conv_in, const bf16 *conv_w,
    const bf16 *a_log, const bf16 *dt_bias, float *qn, float *kn, float *vv, float *beta, float *glog, int HK,
    int HV, int T, float dk_scale) {
  constexpr int DK = 128;
  const int parts = 2 * HK + HV, lane = threadIdx.x & 31;
  const long long unit = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (unit >= (long long)T * parts) return;
  const int t = (int)(unit / parts), p = (int)(unit % parts);
  const int ch0 = p * DK + lane * 4;
  float w[4][4], x[4][4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint2 wv = *reinterpret_cast<const uint2 *>(conv_w + (long long)(ch0 + c) * 4);
    w[c][0] = bf_lo(wv.x); w[c][1] = bf_hi(wv.x); w[c][2] = bf_lo(wv.y); w[c][3] = bf_hi(wv.y);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int s = t - 3 + j;
    if (s < 0) {
#pragma unroll
      for (int c = 0; c < 4; ++c) x[j][c] = bf(conv_in[(long long)(ch0 + c) * 4 + 4 + s]);
    } else {
      const uint2 xv = *reinterpret_cast<const uint2 *>(qkv + (long long)s * ld + ch0);
      x[j][0] = bf_lo(xv.x); x[j][1] = bf_hi(xv.x); x[j][2] = bf_lo(xv.y); x[j][3] = bf_hi(xv.y);
    }
  }
  float y[4], ss = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float tot = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) tot = fmaf(x[j][c], w[c][j], tot);
    const float v = rbf(tot);
    y[c] = rbf(v * (1.f / (1.f + expf(-v))));
    ss = fmaf(y[c], y[c], ss);
  }
  float *dst;
  if (p < 2 * HK) {
    const float r = rsqrtf(warp_sum(ss) + 1e-6f) * (p < HK ? dk_scale : 1.f);
#pragma unroll
    for (int c = 0; c < 4; ++c) y[c] *= r;
    dst = (p < HK ? qn + ((long long)t * HK + p) * DK : kn + ((long long)t * HK + p - HK) * DK);
  } else {
    const int h = p - 2 * HK;
    dst = vv + ((long long)t * HV + h) * DK;
    if (lane == 0) {
      const float bv = bf(bb[(long long)t * ld + h]), av = bf(aa[(long long)t * ld + h]);
      beta[(long long)t * HV + h] = rbf(1.f / (1.f + expf(-bv)));
      const float xa = av + bf(dt_bias[h]);
      const float sp = xa > 20.f ? xa : log1pf(expf(xa));
      glog[(long long)t * HV + h] = -expf(bf(a_log[h])) * sp;
    }
  }
  *reinterpret_cast<float4 *>(dst + lane * 4) = make_float4(y[0], y[1], y[2], y[3]);
}

// The chunk-local matrices of one (chunk of 32 tokens, value head) (reference: _solve,
// chunked.py:17-44): P (in-order prefix sums of g), the Gram matrices k_i.k_j and q_i.k_j,
// T^-1 = (I + L)^-1 by forward substitution, M_ij = (A_i / A_j) q_i.k_j (j <= i), written as the
// chunk's record. Thread (a, b) of the 16 x 16 grid computes entries (i, j) in {a, a + 16} x
// {b, b + 16} of both Gram matrices, summing over d in order.
__global__ void __launch_bounds__(256) delta_chunk_prep_kernel(const float *qn, const float *kn, const float *glog,
                                                               const float *beta, float *rec, int HK, int HV, int T) {
  constexpr int DK = 128, LD = DK + 4;
  const int chunk = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = chunk * kChunk, kh = h / (HV / HK);
  __shared__ __align__(16) float ks[kChunk][LD], qs[kChunk][LD];
  __shared__ float P[kChunk], bt[kChunk], Lm[kChunk][kChunk + 1], Qm[kChunk][kChunk + 1];
  for (int idx = tid; idx < kChunk * DK / 4; idx += blockDim.x) {
    const int t = idx / (DK / 4), d4 = (idx % (DK / 4)) * 4, tok = t0 + t;
    const long long src = ((long long)tok * HK + kh) * DK + d4;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4 *>(&ks[t][d4]) = tok < T ? *reinterpret_cast<const float4 *>(kn + src) : z;
    *reinterpret_cast<float4 *>(&qs[t][d4]) = tok < T ? *reinterpret_cast<const float4 *>(qn + src) : z;
  }
  if (tid < kChunk) {
    const int tok = t0 + tid;
    P[tid] = tok < T ? glog[(long long)tok * HV + h] : 0.f;
    bt[tid] = tok < T ? beta[(long long)tok * HV + h] : 0.f;
  }
  __syncthreads();
  if (tid == 0) {
    float run = 0.f;
    for (int i = 0; i < kChunk; ++i) { run += P[i]; P[i] = run; }
  }
  const int a = tid >> 4, b = tid & 15;
  float g[2][2] = {{0.f, 0.f}, {0.f, 0.f}}, m[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll 4
  for (int d = 0; d < DK; d += 4) {
    const float4 ki0 = *reinterpret_cast<const float4 *>(&ks[a][d]);
    const float4 ki1 = *reinterpret_cast<const float4 *>(&ks[a + 16][d]);
    const float4 qi0 = *reinterpret_cast<const float4 *>(&qs[a][d]);
    const float4 qi1 = *reinterpret_cast<const float4 *>(&qs[a + 16][d]);
    const float4 kj0 = *reinterpret_cast<const float4 *>(&ks[b][d]);
    const float4 kj1 = *reinterpret_cast<const float4 *>(&ks[b + 16][d]);
    const float4 ki[2] = {ki0, ki1}, qi[2] = {qi0, qi1}, kj[2] = {kj0, kj1};
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        g[r][c] = fmaf(ki[r].w, kj[c].w, fmaf(ki[r].z, kj[c].z, fmaf(ki[r].y, kj[c].y, fmaf(ki[r].x, kj[c].x, g[r][c]))));
        m[r][c] = fmaf(qi[r].w, kj[c].w, fmaf(qi[r].z, kj[c].z, fmaf(qi[r].y, kj[c].y, fmaf(qi[r].x, kj[c].x, m[r][c]))));
      }
  }
  __syncthreads();  // P complete
  float *out = rec + ((long long)chunk * HV + h) * kRecFloats;
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int i = a + 16 * r, j = b + 16 * c;
      const float ratio = j <= i ? expf(P[i] - P[j]) : 0.f;
      Lm[i][j] = j < i ? bt[i] * ratio * g[r][c] : 0.f;
      Qm[i][j] = j <= i ? ratio * m[r][c] : 0.f;
    }
  __syncthreads();
  if (warp == 0) {
    // row i of X = (I + L)^-1: X_i = e_i - sum_{j<i} L_ij X_j; lane c keeps column c of X
    float X[kChunk];
#pragma unroll
    for (int i = 0; i < kChunk; ++i) {
      float x = lane == i ? 1.f : 0.f;
#pragma unroll
      for (int j = 0; j < i; ++j) x = fmaf(-Lm[i][j], X[j], x);
      X[i] = x;
    }
#pragma unroll
    for (int i = 0; i < kChunk; ++i) out[REC_TINV + lane * kChunk + i] = X[i];
  } else {
    for (int idx = tid - 32; idx < kChunk * kChunk; idx += blockDim.x - 32) {
      const int j = idx / kChunk, i = idx % kChunk;
      out[REC_MO + idx] = Qm[i][j];
    }
    if (tid >= 32 && tid < 32 + kChunk) {
      const int i = tid - 32;
      out[REC_A + i] = expf(P[i]);
      out[REC_BETA + i] = bt[i];
      out[REC_WS + i] = expf(P[kChunk - 1] - P[i]);
      if (i == 0) out[REC_ALAST] = expf(P[kChunk - 1]);
    }
  }
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// One CTA per (value head, 16 value columns); warp w owns columns 16 blockIdx.y + 2w and + 1, lane l
// rows 4l..4l + 3 of both (so every key and query row read from shared memory serves two
// columns). Per chunk (double-buffered in shared memory by cp.async): 32 key and query
// projections of S_0 per lane and column, summed across the warp by a transposing butterfly (lane i
// ends with token i's sums), then d = T^-1 rhs and o by broadcasts, then the state update.
constexpr int kScanCols = 16;
struct ChunkBuf {
  float k[kChunk][128];
  float q[kChunk][128];
  float v[kChunk][kScanCols];
  float rec[kRecFloats];
};
constexpr size_t kScanSmem = 2 * sizeof(ChunkBuf) + kChunk * kScanCols * sizeof(float);

__device__ __forceinline__ void transpose_sum(float (&v)[kChunk], int lane) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool up = lane & s;
#pragma unroll
    for (int j = 0; j < s; ++j) {
      const float send = up ? v[j] : v[j + s];
      const float keep = up ? v[j + s] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
}

// the 32 per-lane partial dot products of rows x_i (shared memory) with the lane's 4 state rows
// of two columns, summed over the warp: lane i returns token i's sums
__device__ __forceinline__ void project2(const float (*x)[128], int r0, const float (&S)[2][4], int lane,
                                         float &out0, float &out1) {
  float p0[kChunk], p1[kChunk];
#pragma unroll
  for (int i = 0; i < kChunk; ++i) {
    const float4 xv = *reinterpret_cast<const float4 *>(&x[i][r0]);
    p0[i] = fmaf(xv.w, S[0][3], fmaf(xv.z, S[0][2], fmaf(xv.y, S[0][1], xv.x * S[0][0])));
    p1[i] = fmaf(xv.w, S[1][3], fmaf(xv.z, S[1][2], fmaf(xv.y, S[1][1], xv.x * S[1][0])));
  }
  transpose_sum(p0, lane);
  transpose_sum(p1, lane);
  out0 = p0[0];
  out1 = p1[0];
}

__global__ void __launch_bounds__(256, 2) delta_chunk_scan_kernel(const float *qn, const float *kn, const float *vv,
                                                                  const float *rec, const float *rec_in,
                                                                  float *rec_out, bf16 *core, int HK, int HV, int T) {
  constexpr int DK = 128;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ChunkBuf *buf = reinterpret_cast<ChunkBuf *>(smem_raw);
  float(*obuf)[kScanCols] = reinterpret_cast<float(*)[kScanCols]>(smem_raw + 2 * sizeof(ChunkBuf));
  const int h = blockIdx.x, c0 = blockIdx.y * kScanCols, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cw = 2 * warp, r0 = lane * 4, kh = h / (HV / HK);
  const int nch = (T + kChunk - 1) / kChunk;
  auto issue = [&](int chunk, ChunkBuf &b) {
    const int t0 = chunk * kChunk;
    for (int idx = tid; idx < kChunk * DK / 4; idx += 256) {
      const int t = idx / (DK / 4), d4 = idx % (DK / 4), tok = t0 + t;
      const long long src = ((long long)min(tok, T - 1) * HK + kh) * DK + d4 * 4;
      cp_async16(&b.k[t][d4 * 4], kn + src, tok < T);
      cp_async16(&b.q[t][d4 * 4], qn + src, tok < T);
    }
    if (tid < kChunk * kScanCols / 4) {
      const int t = tid / (kScanCols / 4), part = tid % (kScanCols / 4), tok = t0 + t;
      cp_async16(&b.v[t][part * 4], vv + ((long long)min(tok, T - 1) * HV + h) * DK + c0 + part * 4, tok < T);
    }
    const float *src = rec + ((long long)chunk * HV + h) * kRecFloats;
    for (int idx = tid; idx < kRecFloats / 4; idx += 256) cp_async16(&b.rec[idx * 4], src + idx * 4, true);
    cp_async_commit();
  };
  const float *Si = rec_in + (long long)h * DK * DK;
  float S[2][4];
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int r = 0; r < 4; ++r) S[c][r] = Si[(long long)(r0 + r) * DK + c0 + cw + c];
  issue(0, buf[0]);
  for (int ch = 0; ch < nch; ++ch) {
    if (ch + 1 < nch) {
      issue(ch + 1, buf[(ch + 1) & 1]);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const ChunkBuf &b = buf[ch & 1];
    const float *R = b.rec;
    float pk0, pk1, pq0, pq1;
    project2(b.k, r0, S, lane, pk0, pk1);
    project2(b.q, r0, S, lane, pq0, pq1);
    const float A = R[REC_A + lane], beta = R[REC_BETA + lane];
    const float rhs0 = beta * (b.v[lane][cw] - A * pk0), rhs1 = beta * (b.v[lane][cw + 1] - A * pk1);
    float d0 = 0.f, d1 = 0.f;
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const float t = R[REC_TINV + j * kChunk + lane];
      d0 = fmaf(t, __shfl_sync(0xffffffffu, rhs0, j), d0);
      d1 = fmaf(t, __shfl_sync(0xffffffffu, rhs1, j), d1);
    }
    float o0 = A * pq0, o1 = A * pq1;
    const float alast = R[REC_ALAST];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      S[0][r] *= alast;
      S[1][r] *= alast;
    }
#pragma unroll 8
    for (int j = 0; j < kChunk; ++j) {
      const float dj0 = __shfl_sync(0xffffffffu, d0, j), dj1 = __shfl_sync(0xffffffffu, d1, j);
      const float m = R[REC_MO + j * kChunk + lane], ws = R[REC_WS + j];
      o0 = fmaf(m, dj0, o0);
      o1 = fmaf(m, dj1, o1);
      const float e0 = ws * dj0, e1 = ws * dj1;
      const float4 kv = *reinterpret_cast<const float4 *>(&b.k[j][r0]);
      S[0][0] = fmaf(kv.x, e0, S[0][0]);
      S[0][1] = fmaf(kv.y, e0, S[0][1]);
      S[0][2] = fmaf(kv.z, e0, S[0][2]);
      S[0][3] = fmaf(kv.w, e0, S[0][3]);
      S[1][0] = fmaf(kv.x, e1, S[1][0]);
      S[1][1] = fmaf(kv.y, e1, S[1][1]);
      S[1][2] = fmaf(kv.z, e1, S[1][2]);
      S[1][3] = fmaf(kv.w, e1, S[1][3]);
    }
    obuf[lane][cw] = o0;
    obuf[lane][cw + 1] = o1;
    __syncthreads();
    if (tid < kChunk * 2) {
      const int t = tid >> 1, half = tid & 1, tok = ch * kChunk + t;
      if (tok < T) {
        const float *ov = &obuf[t][half * 8];
        *reinterpret_cast<uint4 *>(core + ((long long)tok * HV + h) * DK + c0 + half * 8) =
            make_uint4(pack2(ov[0], ov[1]), pack2(ov[2], ov[3]), pack2(ov[4], ov[5]), pack2(ov[6], ov[7]));
      }
    }
    __syncthreads();
  }
  float *So = rec_out + (long long)h * DK * DK;
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int r = 0; r < 4; ++r) So[(long long)(r0 + r) * DK + c0 + cw + c] = S[c][r];
}

// Gated RMSNorm (HF Qwen3_5RMSNormGated): bf16(bf16(w * bf16(x r)) * silu(z)) over each head's
// 128 values, one warp per (token, head), lane l holding values 4l..4l + 3; the sum of squares is
// taken like the decode kernel's: per 16-value tile, then ((p0 + p1) + (p2 + p3)) + ((p4 + p5) +
// (p6 + p7)).
__global__ void __launch_bounds__(256) gated_norm_kernel(const bf16 *core, const bf16 *z, int ld, const bf16 *w,
                                                         bf16 *out, int HV, int T, float eps) {
  constexpr int DK = 128;
  const int lane = threadIdx.x & 31;
  const long long unit = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (unit >= (long long)T * HV) return;
  const long long t = unit / HV;
  const int h = (int)(unit % HV);
  const long long i = unit * DK + lane * 4;
  const uint2 xv = *reinterpret_cast<const uint2 *>(core + i);
  const uint2 zv = *reinterpret_cast<const uint2 *>(z + t * ld + h * DK + lane * 4);
  const uint2 wv = *reinterpret_cast<const uint2 *>(w + lane * 4);
  const float x[4] = {bf_lo(xv.x), bf_hi(xv.x), bf_lo(xv.y), bf_hi(xv.y)};
  const float zz[4] = {bf_lo(zv.x), bf_hi(zv.x), bf_lo(zv.y), bf_hi(zv.y)};
  const float wf[4] = {bf_lo(wv.x), bf_hi(wv.x), bf_lo(wv.y), bf_hi(wv.y)};
  float sq = fmaf(x[3], x[3], fmaf(x[2], x[2], fmaf(x[1], x[1], x[0] * x[0])));
  sq += __shfl_xor_sync(0xffffffffu, sq, 1);
  sq += __shfl_xor_sync(0xffffffffu, sq, 2);
  float p[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) p[k] = __shfl_sync(0xffffffffu, sq, 4 * k);
  const float tot = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
  const float r = rsqrtf(tot / (float)DK + eps);
  float y[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float n = rbf(wf[e] * rbf(x[e] * r));
    y[e] = n * (zz[e] / (1.f + expf(-zz[e])));
  }
  *reinterpret_cast<uint2 *>(out + i) = make_uint2(pack2(y[0], y[1]), pack2(y[2], y[3]));
}

// q/k RMSNorm over the head dim and RoPE (rotate-half over the first RD dims, bf16 cos/sin of
// fp32 angles, bf16 products and sum), as the decode kernel; one warp per (token, head). Heads
// [0, HQ) are query heads (written to qatt [HQ, T, D]); [HQ, HQ + HKV) keys and
// [HQ + HKV, HQ + 2 HKV) values, appended to the cache at position start + t.
__global__ void attn_prep_kernel(const bf16 *qo, const bf16 *ko, const bf16 *vo, int ld, const bf16 *qnorm,
                                 const bf16 *knorm, const float *inv_freq, bf16 *qatt, bf16 *kc, bf16 *vc,
                                 int HQ, int HKV, int D, int RD, int C, int T, long long start, float eps, int q35) {
  const int t = blockIdx.x, hh = blockIdx.y, lane = threadIdx.x, EPL = D / 32;
  const long long pos = start + t;
  if (hh >= HQ + HKV) {
    const int kvh = hh - HQ - HKV;
    for (int d = lane; d < D; d += 32)
      vc[((long long)kvh * C + pos) * D + d] = vo[(long long)t * ld + kvh * D + d];
    return;
  }
  const bool isk = hh >= HQ;
  const int hd = isk ? hh - HQ : hh;
  const bf16 *src = isk ? ko + (long long)t * ld + hd * D : qo + (long long)t * ld + hd * D * (q35 ? 2 : 1);
  const bf16 *nw = isk ? knorm : qnorm;
  float v[8], ss = 0.f;
  for (int e = 0; e < 8; ++e) {
    v[e] = e < EPL ? bf(src[lane * EPL + e]) : 0.f;
    ss = fmaf(v[e], v[e], ss);
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  __shared__ float nv[256];
  for (int e = 0; e < EPL; ++e) {
    const float wv = bf(nw[lane * EPL + e]);
    v[e] = q35 ? rbf(v[e] * r * (1.f + wv)) : rbf(wv * rbf(v[e] * r));
    nv[lane * EPL + e] = v[e];
  }
  __syncwarp();
  const int half = RD / 2;
  for (int e = 0; e < EPL; ++e) {
    const int d = lane * EPL + e;
    if (d < RD) {
      const int f = d < half ? d : d - half;
      const float ang = (float)pos * inv_freq[f];
      const float cs = rbf(cosf(ang)), sn = rbf(sinf(ang));
      const float rot = d < half ? -nv[d + half] : nv[d - half];
      v[e] = rbf(rbf(v[e] * cs) + rbf(rot * sn));
    }
  }
  bf16 *dst = isk ? kc + ((long long)hd * C + pos) * D : qatt + ((long long)hd * T + t) * D;
  for (int e = 0; e < EPL; ++e) dst[lane * EPL + e] = tobf(v[e]);
}

// Attention output rows [T, HQ * D] for o_proj: Qwen3.5 multiplies by bf16(sigmoid(gate)) and
// rounds (compiler/qwen35/adapters/attention.py:61-63); Qwen3 copies.
__global__ void attn_out_kernel(const bf16 *oatt, const bf16 *qo, int ld, bf16 *out, int HQ, int D, int T, int q35) {
  const int t = blockIdx.x, h = blockIdx.y;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float y = bf(oatt[((long long)h * T + t) * D + d]);
    if (q35) {
      const float g = bf(qo[(long long)t * ld + h * 2 * D + D + d]);
      y = rbf(y * rbf(1.f / (1.f + expf(-g))));
    }
    out[((long long)t * HQ + h) * D + d] = tobf(y);
  }
}

// torch.argmax of one bf16 row (first maximal index, NaN counts as the maximum) in two launches:
// each CTA reduces a contiguous range to one candidate, then one CTA reduces the candidates in
// range order.
__device__ __forceinline__ void block_argmax(float &bv, int &bi) {
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (argmax_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (argmax_better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
}

__global__ void __launch_bounds__(256) argmax_partial_kernel(const bf16 *row, int n, float *cand_v, int *cand_i) {
  const int per = (n + gridDim.x - 1) / gridDim.x, lo = blockIdx.x * per, hi = min(n, lo + per);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float v = bf(row[i]);
    if (argmax_better(v, i, bv, bi)) { bv = v; bi = i; }
  }
  block_argmax(bv, bi);
  if (threadIdx.x == 0) { cand_v[blockIdx.x] = bv; cand_i[blockIdx.x] = bi; }
}

__global__ void __launch_bounds__(256) argmax_final_kernel(const float *cand_v, const int *cand_i, int n, int64_t *token) {
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (argmax_better(cand_v[i], cand_i[i], bv, bi)) { bv = cand_v[i]; bi = cand_i[i]; }
  block_argmax(bv, bi);
  if (threadIdx.x == 0) *token = bi;
}

} // namespace xbpre

extern "C" int xb_gemm_bf16(int32_t m, int32_t n, int32_t k, const void *x, const void *w, void *out, void *stream);
extern "C" int xb_prefix_attention(const XbAttentionArgs *args, void *stream);

using namespace xbpre;

extern "C" int xb_prefill_workspace_bytes(const XbModel *model, int32_t max_tokens, size_t *bytes) {
  if (!model || !bytes) return xb::fail(XB_ERR_INVALID, "null argument");
  if (max_tokens < 1 || max_tokens > kMaxTokens) return xb::fail(XB_ERR_INVALID, "max_tokens must be 1..512");
  *bytes = layout(model->g, max_tokens).total;
  return XB_OK;
}

extern "C" int xb_prefill_step(const XbModel *model, const XbPrefillArgs *a, void *workspace,
                               size_t workspace_bytes, void *stream) {
  if (!model || !a || !workspace) return xb::fail(XB_ERR_INVALID, "null argument");
  const XbGeometry &g = model->g;
  const int T = a->tokens;
  if (T < 1 || T > kMaxTokens) return xb::fail(XB_ERR_INVALID, "prefill takes 1..512 tokens");
  if (!a->input_ids) return xb::fail(XB_ERR_INVALID, "input_ids are required");
  if (a->start_position < 0 || a->start_position + T > g.capacity)
    return xb::fail(XB_ERR_INVALID, "Context capacity exceeded");
  if (!a->logits) return xb::fail(XB_ERR_INVALID, "logits are required");
  const Layout L = layout(g, T);
  if (workspace_bytes < L.total) return xb::fail(XB_ERR_INVALID, "prefill workspace too small");
  for (int l = 0; l < g.num_layers; ++l) {
    const XbLayerState &s = a->layers[l];
    if (g.layer_kind[l] == XB_LAYER_DELTANET ? (!s.conv_in || !s.rec_in || !s.conv_out || !s.rec_out)
                                             : (!s.k_cache || !s.v_cache))
      return xb::fail(XB_ERR_INVALID, "missing state in layer " + std::to_string(l));
  }
  if (g.family == XB_FAMILY_QWEN35 && g.lin_head_dim != 128)
    return xb::fail(XB_ERR_UNSUPPORTED, "prefill needs DeltaNet heads of dimension 128");
  if (g.family == XB_FAMILY_QWEN35) {
    const cudaError_t e = cudaFuncSetAttribute(delta_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)kScanSmem);
    if (e != cudaSuccess) return xb::fail(XB_ERR_CUDA, std::string("prefill: ") + cudaGetErrorString(e));
  }
  cudaStream_t st = (cudaStream_t)stream;
  char *ws = (char *)workspace;
  auto P = [&](size_t off) { return (bf16 *)(ws + off); };
  auto F = [&](size_t off) { return (float *)(ws + off); };
  unsigned *err = (unsigned *)ws + 64;
  const bool q35 = g.family == XB_FAMILY_QWEN35;
  const int H = g.hidden, I = g.intermediate, HQ = g.num_q_heads, HKV = g.num_kv_heads, D = g.head_dim;
  const int HK = q35 ? g.lin_key_heads : 0, HV = q35 ? g.lin_value_heads : 0, DK = g.lin_head_dim;
  const int CH = q35 ? lin_channels(g) : 0;
  bf16 *h = P(L.h), *x = P(L.x), *x2 = P(L.x2), *out = P(L.out);
  int rc;
#define XB_TRY(call)                                                                                   \
  do {                                                                                               \
    rc = (call);                                                                                     \
    if (rc) return rc;                                                                               \
  } while (0)
#define XB_LAUNCHED()                                                                                  \
  do {                                                                                               \
    cudaError_t e_ = cudaGetLastError();                                                             \
    if (e_ != cudaSuccess) return xb::fail(XB_ERR_CUDA, std::string("prefill launch: ") + cudaGetErrorString(e_)); \
  } while (0)
  const int NP = proj_width(g);
  if (NP % 4) return xb::fail(XB_ERR_UNSUPPORTED, "prefill needs projection rows of a multiple of 4 elements");
  bf16 *proj = P(L.proj);
  // One GEMM per group of projections that read the same rows when their weights are adjacent
  // rows of one tensor (the reference's packed layout), else one GEMM per projection, each into
  // its columns of the projection rows.
  struct Part { const void *w; int rows; };
  auto group = [&](const bf16 *xin, int k, std::initializer_list<Part> parts) -> int {
    bool packed = true;
    int rows = 0;
    const Part *prev = nullptr;
    for (const Part &p : parts) {
      if (prev && (const char *)p.w != (const char *)prev->w + (size_t)prev->rows * k * 2) packed = false;
      rows += p.rows;
      prev = &p;
    }
    if (packed) return xb::gemm_bf16(T, rows, k, xin, parts.begin()->w, proj, NP, stream, err);
    int col = 0;
    for (const Part &p : parts) {
      const int rc = xb::gemm_bf16(T, p.rows, k, xin, p.w, proj + col, NP, stream, err);
      if (rc) return rc;
      col += p.rows;
    }
    return XB_OK;
  };
  const int rn = H / 8 <= 128 ? 128 : 256;  // threads per row of the add + RMSNorm kernel
  embed_kernel<<<T, 128, 0, st>>>(a->input_ids, (const bf16 *)model->w.embed, h, H, g.vocab, err);
  XB_LAUNCHED();
  add_rmsnorm_kernel<<<T, rn, 0, st>>>(h, nullptr, (const bf16 *)model->w.layers[0].input_norm, x, H, g.rms_eps,
                                        q35, 0);
  XB_LAUNCHED();
  for (int l = 0; l < g.num_layers; ++l) {
    const XbLayerWeights &w = model->w.layers[l];
    const XbLayerState &s = a->layers[l];
    if (g.layer_kind[l] == XB_LAYER_DELTANET) {
      const int HVD = HV * DK;
      XB_TRY(group(x, H, {{w.in_qkv, CH}, {w.in_z, HVD}, {w.in_b, HV}, {w.in_a, HV}}));
      const bf16 *qkv = proj, *z = proj + CH, *bb = proj + CH + HVD, *aa = proj + CH + HVD + HV;
      {
        const long long warps = (long long)T * (2 * HK + HV);
        delta_prepare_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(
            qkv, bb, aa, NP, (const bf16 *)s.conv_in, (const bf16 *)w.conv_w, (const bf16 *)w.a_log,
            (const bf16 *)w.dt_bias, F(L.qn), F(L.kn), F(L.vv), F(L.beta), F(L.glog), HK, HV, T,
            (float)(1.0 / std::sqrt((double)DK)));
        XB_LAUNCHED();
      }
      delta_chunk_prep_kernel<<<dim3((T + kChunk - 1) / kChunk, HV), 256, 0, st>>>(F(L.qn), F(L.kn), F(L.glog),
                                                                                F(L.beta), F(L.rec), HK, HV, T);
      XB_LAUNCHED();
      conv_state_kernel<<<(CH + 255) / 256, 256, 0, st>>>(qkv, NP, (const bf16 *)s.conv_in, (bf16 *)s.conv_out, CH, T);
      XB_LAUNCHED();
      delta_chunk_scan_kernel<<<dim3(HV, DK / kScanCols), 256, kScanSmem, st>>>(
          F(L.qn), F(L.kn), F(L.vv), F(L.rec), (const float *)s.rec_in, (float *)s.rec_out, P(L.core), HK, HV, T);
      XB_LAUNCHED();
      gated_norm_kernel<<<(unsigned)(((long long)T * HV + 7) / 8), 256, 0, st>>>(P(L.core), z, NP,
                                                                              (const bf16 *)w.gnorm, x2, HV, T,
                                                                              g.rms_eps);
      XB_LAUNCHED();
      XB_TRY(xb::gemm_bf16(T, H, HVD, x2, w.out_proj, out, H, stream, err));
    } else {
      const int qrows = HQ * D * (q35 ? 2 : 1);
      XB_TRY(group(x, H, {{w.q_proj, qrows}, {w.k_proj, HKV * D}, {w.v_proj, HKV * D}}));
      const bf16 *qo = proj, *ko = proj + qrows, *vo = proj + qrows + HKV * D;
      attn_prep_kernel<<<dim3(T, HQ + 2 * HKV), 32, 0, st>>>(
          qo, ko, vo, NP, (const bf16 *)w.q_norm, (const bf16 *)w.k_norm, model->d_inv_freq, P(L.qatt),
          (bf16 *)s.k_cache, (bf16 *)s.v_cache, HQ, HKV, D, g.rotary_dim, g.capacity, T, a->start_position,
          g.rms_eps, q35);
      XB_LAUNCHED();
      XbAttentionArgs at;
      std::memset(&at, 0, sizeof(at));
      at.q = P(L.qatt);
      at.k = s.k_cache;
      at.v = s.v_cache;
      at.out = P(L.oatt);
      const long long qs[3] = {(long long)HQ * T * D, (long long)T * D, D};
      const long long ks[3] = {(long long)HKV * g.capacity * D, (long long)g.capacity * D, D};
      for (int i = 0; i < 3; ++i) { at.strides[i] = qs[i]; at.strides[3 + i] = ks[i]; at.strides[6 + i] = ks[i]; }
      at.batch = 1; at.q_heads = HQ; at.kv_heads = HKV; at.head_dim = D; at.q_tokens = T;
      at.capacity = g.capacity;
      at.count = T;
      at.length = (int32_t)(a->start_position + T);
      at.scale = (float)(1.0 / std::sqrt((double)D));
      XB_TRY(xb_prefix_attention(&at, stream));
      attn_out_kernel<<<dim3(T, HQ), 128, 0, st>>>(P(L.oatt), qo, NP, x2, HQ, D, T, q35);
      XB_LAUNCHED();
      XB_TRY(xb::gemm_bf16(T, H, HQ * D, x2, w.o_proj, out, H, stream, err));
    }
    add_rmsnorm_kernel<<<T, rn, 0, st>>>(h, out, (const bf16 *)w.post_norm, x, H, g.rms_eps, q35, 0);
    XB_LAUNCHED();
    XB_TRY(group(x, H, {{w.gate, I}, {w.up, I}}));
    silu_mul_kernel<<<(unsigned)(((long long)T * (I / 8) + 255) / 256), 256, 0, st>>>(proj, x2, I, NP, T);
    XB_LAUNCHED();
    XB_TRY(xb::gemm_bf16(T, H, I, x2, w.down, out, H, stream, err));
    if (l + 1 < g.num_layers) {
      add_rmsnorm_kernel<<<T, rn, 0, st>>>(h, out, (const bf16 *)model->w.layers[l + 1].input_norm, x, H,
                                            g.rms_eps, q35, 0);
    } else {
      // the last token only: residual add, final norm (ModelStep's last-token gather, model.py:178-183)
      add_rmsnorm_kernel<<<1, rn, 0, st>>>(h, out, (const bf16 *)model->w.final_norm, P(L.xlast), H, g.rms_eps,
                                            q35, T - 1);
    }
    XB_LAUNCHED();
  }
  XB_TRY(xb::gemm_bf16(1, g.vocab, H, P(L.xlast), model->w.lm_head, a->logits, g.vocab, stream, err));
  if (a->next_token) {
    argmax_partial_kernel<<<kArgmaxBlocks, 256, 0, st>>>((const bf16 *)a->logits, g.vocab, F(L.amax),
                                                         (int *)(ws + L.amax) + kArgmaxBlocks);
    XB_LAUNCHED();
    argmax_final_kernel<<<1, 256, 0, st>>>(F(L.amax), (const int *)(ws + L.amax) + kArgmaxBlocks, kArgmaxBlocks,
                                           a->next_token);
    XB_LAUNCHED();
  }
#undef XB_TRY
#undef XB_LAUNCHED
  return XB_OK;
}
