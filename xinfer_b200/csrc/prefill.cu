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
// the prefill workspace starts with the decode workspace's control words, so that
// xb_workspace_check reads its error word (word 64) the same way
constexpr int kCtlBytes = 1024;
enum { PERR_TOKEN = 4 };

struct Layout {
  size_t h, x, x2, out, qkv, z, bb, aa, gate, up, qn, kn, vv, beta, decay, core, qatt, oatt, xlast, total;
};

static int lin_channels(const XbGeometry &g) { return (2 * g.lin_key_heads + g.lin_value_heads) * g.lin_head_dim; }

static Layout layout(const XbGeometry &g, int T) {
  Layout L{};
  const bool q35 = g.family == XB_FAMILY_QWEN35;
  const int HVD = q35 ? g.lin_value_heads * g.lin_head_dim : 0;
  const int qrows = g.num_q_heads * g.head_dim * (q35 ? 2 : 1);
  const int widest = std::max({g.hidden, g.intermediate, g.num_q_heads * g.head_dim, HVD});
  size_t off = kCtlBytes;
  auto take = [&](size_t bytes) { size_t o = off; off += (bytes + 255) & ~size_t(255); return o; };
  L.h = take((size_t)T * g.hidden * 2);
  L.x = take((size_t)T * widest * 2);
  L.x2 = take((size_t)T * widest * 2);
  L.out = take((size_t)T * g.hidden * 2);
  L.qkv = take((size_t)T * std::max(q35 ? lin_channels(g) : 0, qrows) * 2);
  L.z = take((size_t)T * std::max(HVD, g.num_kv_heads * g.head_dim) * 2);
  L.bb = take((size_t)T * std::max(q35 ? g.lin_value_heads : 8, g.num_kv_heads * g.head_dim) * 2);
  L.aa = take((size_t)T * std::max(q35 ? g.lin_value_heads : 8, 8) * 2);
  L.gate = take((size_t)T * g.intermediate * 2);
  L.up = take((size_t)T * g.intermediate * 2);
  const size_t vec = q35 ? (size_t)T * HVD * 4 : 256;
  L.qn = take(vec);
  L.kn = take(vec);
  L.vv = take(vec);
  L.beta = take(q35 ? (size_t)T * g.lin_value_heads * 4 : 256);
  L.decay = take(q35 ? (size_t)T * g.lin_value_heads * 4 : 256);
  L.core = take(q35 ? (size_t)T * HVD * 2 : 256);
  L.qatt = take((size_t)T * g.num_q_heads * g.head_dim * 2);
  L.oatt = take((size_t)T * g.num_q_heads * g.head_dim * 2);
  L.xlast = take((size_t)g.hidden * 2 + 16);
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

// RMSNorm of rows (HF Qwen3RMSNorm: w * bf16(x r); Qwen3_5RMSNorm: bf16(x r (1 + w))), 256
// threads per row, each summing the squares of its 8-element chunks c and c + 256 in order.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const bf16 *in, const bf16 *w, bf16 *out, int H,
                                                      float eps, int q35) {
  const int t = blockIdx.x, tid = threadIdx.x, nc = H / 8;
  const uint4 *row = reinterpret_cast<const uint4 *>(in + (long long)t * H);
  __shared__ float red[8];
  uint4 xv[2];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int c = tid + i * 256;
    xv[i] = c < nc ? row[c] : make_uint4(0, 0, 0, 0);
    float x[8];
    unpack8(xv[i], x);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)H + eps);
  uint4 *dst = reinterpret_cast<uint4 *>(out + (long long)t * H);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int c = tid + i * 256;
    if (c >= nc) continue;
    float x[8], wf[8], y[8];
    unpack8(xv[i], x);
    unpack8(reinterpret_cast<const uint4 *>(w)[c], wf);
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = q35 ? x[e] * r * (1.f + wf[e]) : wf[e] * rbf(x[e] * r);
    dst[c] = make_uint4(pack2(y[0], y[1]), pack2(y[2], y[3]), pack2(y[4], y[5]), pack2(y[6], y[7]));
  }
}

// h = bf16(h + o), the residual adds of the reference (both operands bf16).
__global__ void add_kernel(bf16 *h, const bf16 *o, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n / 2; i += (long long)gridDim.x * blockDim.x) {
    const uint32_t a = reinterpret_cast<uint32_t *>(h)[i], b = reinterpret_cast<const uint32_t *>(o)[i];
    reinterpret_cast<uint32_t *>(h)[i] = pack2(bf_lo(a) + bf_lo(b), bf_hi(a) + bf_hi(b));
  }
}

// act = bf16(bf16(silu(gate)) * up) (HF SiLU on a bf16 tensor, then the bf16 product).
__global__ void silu_mul_kernel(const bf16 *gate, const bf16 *up, bf16 *act, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float g = bf(gate[i]), u = bf(up[i]);
    const float s = rbf(g / (1.f + expf(-g)));
    act[i] = tobf(s * u);
  }
}

// DeltaNet preparation of token t, value head h (recurrent.py:32-58, 99-120 and the prepare step
// of the long path, recurrent.py:127-189): width-4 causal conv over [old window, tokens] with fp32
// FMAs in tap order, bf16, SiLU, bf16; q, k l2-normalised (q also scaled by dk^-0.5); beta =
// bf16(sigmoid(b)); decay = exp(-exp(A_log) * softplus(a + dt_bias)), softplus threshold 20.
__global__ void __launch_bounds__(256) delta_prepare_kernel(
    const bf16 *qkv, const bf16 *bb, const bf16 *aa, const bf16 *conv_in, const bf16 *conv_w,
    const bf16 *a_log, const bf16 *dt_bias, float *qn, float *kn, float *vv, float *beta, float *decay,
    int HK, int HV, int DK, float dk_scale) {
  const int t = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int CH = (2 * HK + HV) * DK, kh = h / (HV / HK);
  __shared__ float pn[8];
  auto conv = [&](int ch) -> float {
    float tot = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int s = t - 3 + j;
      const float in = s < 0 ? bf(conv_in[(long long)ch * 4 + 4 + s]) : bf(qkv[(long long)s * CH + ch]);
      tot = fmaf(in, bf(conv_w[(long long)ch * 4 + j]), tot);
    }
    const float v = rbf(tot);
    return rbf(v * (1.f / (1.f + expf(-v))));
  };
  const int chq = tid < DK ? kh * DK + tid : (HK + kh) * DK + (tid - DK);
  const float val = conv(chq);
  const float sq = warp_sum(val * val);
  if ((tid & 31) == 0) pn[tid >> 5] = sq;
  float vch = 0.f;
  if (tid < DK) vch = conv((2 * HK + h) * DK + tid);
  __syncthreads();
  const long long base = ((long long)t * HV + h) * DK;
  if (tid < DK) {
    const float qs = rsqrtf(pn[0] + pn[1] + pn[2] + pn[3] + 1e-6f);
    qn[base + tid] = val * qs * dk_scale;
    vv[base + tid] = vch;
  } else {
    const float ks = rsqrtf(pn[4] + pn[5] + pn[6] + pn[7] + 1e-6f);
    kn[base + tid - DK] = val * ks;
  }
  if (tid == 0) {
    const float b = bf(bb[(long long)t * HV + h]), a = bf(aa[(long long)t * HV + h]);
    beta[(long long)t * HV + h] = rbf(1.f / (1.f + expf(-b)));
    const float x = a + bf(dt_bias[h]);
    const float sp = x > 20.f ? x : log1pf(expf(x));
    decay[(long long)t * HV + h] = expf(-expf(bf(a_log[h])) * sp);
  }
}

// The conv window after the last token: the last four inputs of [old window, tokens] for every
// channel (recurrent.py:43-52). Launched after every read of the old window, so in place is safe.
__global__ void conv_state_kernel(const bf16 *qkv, const bf16 *conv_in, bf16 *conv_out, int CH, int T) {
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= CH) return;
  bf16 w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int s = T - 4 + j;
    w[j] = s < 0 ? conv_in[(long long)ch * 4 + 4 + s] : qkv[(long long)s * CH + ch];
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) conv_out[(long long)ch * 4 + j] = w[j];
}

// Gated delta rule over T tokens (recurrent.py:20-28) for one value head and 16 columns of its
// 128 x 128 fp32 state: warp w owns columns 2w, 2w + 1, lane l rows 4l..4l + 3. Per token:
// S *= decay; delta = (v - S^T k) * beta; S += k delta^T; out = S^T q (bf16). The next token's
// inputs are loaded while the current one is processed.
__global__ void __launch_bounds__(256) delta_scan_kernel(const float *qn, const float *kn, const float *vv,
                                                         const float *beta, const float *decay,
                                                         const float *rec_in, float *rec_out, bf16 *core,
                                                         int HV, int DK, int T) {
  const int h = blockIdx.x, tile = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = tile * 16 + 2 * warp, r0 = lane * 4;
  const float *Si = rec_in + (long long)h * DK * DK;
  float S[4][2];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    S[r][0] = Si[(long long)(r0 + r) * DK + c0];
    S[r][1] = Si[(long long)(r0 + r) * DK + c0 + 1];
  }
  auto load = [&](int t, float4 &k4, float4 &q4, float2 &v2, float &bt, float &dc) {
    const long long base = ((long long)t * HV + h) * DK;
    k4 = *reinterpret_cast<const float4 *>(kn + base + r0);
    q4 = *reinterpret_cast<const float4 *>(qn + base + r0);
    v2 = *reinterpret_cast<const float2 *>(vv + base + c0);
    bt = beta[(long long)t * HV + h];
    dc = decay[(long long)t * HV + h];
  };
  float4 k4, q4, nk4, nq4;
  float2 v2, nv2;
  float bt, dc, nbt, ndc;
  load(0, k4, q4, v2, bt, dc);
  for (int t = 0; t < T; ++t) {
    if (t + 1 < T) load(t + 1, nk4, nq4, nv2, nbt, ndc);
    const float k[4] = {k4.x, k4.y, k4.z, k4.w}, q[4] = {q4.x, q4.y, q4.z, q4.w};
    float p0 = 0.f, p1 = 0.f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      S[r][0] *= dc;
      S[r][1] *= dc;
      p0 = fmaf(S[r][0], k[r], p0);
      p1 = fmaf(S[r][1], k[r], p1);
    }
    p0 = warp_sum(p0);
    p1 = warp_sum(p1);
    const float d0 = (v2.x - p0) * bt, d1 = (v2.y - p1) * bt;
    float o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      S[r][0] = fmaf(k[r], d0, S[r][0]);
      S[r][1] = fmaf(k[r], d1, S[r][1]);
      o0 = fmaf(S[r][0], q[r], o0);
      o1 = fmaf(S[r][1], q[r], o1);
    }
    o0 = warp_sum(o0);
    o1 = warp_sum(o1);
    if (lane == 0)
      *reinterpret_cast<uint32_t *>(core + ((long long)t * HV + h) * DK + c0) = pack2(o0, o1);
    k4 = nk4; q4 = nq4; v2 = nv2; bt = nbt; dc = ndc;
  }
  float *So = rec_out + (long long)h * DK * DK;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    So[(long long)(r0 + r) * DK + c0] = S[r][0];
    So[(long long)(r0 + r) * DK + c0 + 1] = S[r][1];
  }
}

// Gated RMSNorm of token t, head h (HF Qwen3_5RMSNormGated): bf16(bf16(w * bf16(x r)) * silu(z)),
// the sum of squares taken like the decode kernel's: per 16-value tile, then
// ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7)).
__global__ void __launch_bounds__(128) gated_norm_kernel(const bf16 *core, const bf16 *z, const bf16 *w, bf16 *out,
                                                         int HV, int DK, float eps) {
  const int t = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const long long i = ((long long)t * HV + h) * DK + tid;
  __shared__ float part[8];
  const float x = bf(core[i]);
  float sq = x * x;
#pragma unroll
  for (int o = 8; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((tid & 15) == 0) part[tid >> 4] = sq;
  __syncthreads();
  const float tot = ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
  const float r = rsqrtf(tot / (float)DK + eps);
  const float n = rbf(bf(w[tid]) * rbf(x * r));
  const float zz = bf(z[i]);
  out[i] = tobf(n * (zz / (1.f + expf(-zz))));
}

// q/k RMSNorm over the head dim and RoPE (rotate-half over the first RD dims, bf16 cos/sin of
// fp32 angles, bf16 products and sum), as the decode kernel; one warp per (token, head). Heads
// [0, HQ) are query heads (written to qatt [HQ, T, D]); [HQ, HQ + HKV) keys and
// [HQ + HKV, HQ + 2 HKV) values, appended to the cache at position start + t.
__global__ void attn_prep_kernel(const bf16 *qo, const bf16 *ko, const bf16 *vo, const bf16 *qnorm,
                                 const bf16 *knorm, const float *inv_freq, bf16 *qatt, bf16 *kc, bf16 *vc,
                                 int HQ, int HKV, int D, int RD, int C, int T, long long start, float eps, int q35) {
  const int t = blockIdx.x, hh = blockIdx.y, lane = threadIdx.x, EPL = D / 32;
  const long long pos = start + t;
  if (hh >= HQ + HKV) {
    const int kvh = hh - HQ - HKV;
    for (int d = lane; d < D; d += 32)
      vc[((long long)kvh * C + pos) * D + d] = vo[((long long)t * HKV + kvh) * D + d];
    return;
  }
  const bool isk = hh >= HQ;
  const int hd = isk ? hh - HQ : hh;
  const bf16 *src = isk ? ko + ((long long)t * HKV + hd) * D : qo + ((long long)t * HQ + hd) * D * (q35 ? 2 : 1);
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
__global__ void attn_out_kernel(const bf16 *oatt, const bf16 *qo, bf16 *out, int HQ, int D, int T, int q35) {
  const int t = blockIdx.x, h = blockIdx.y;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float y = bf(oatt[((long long)h * T + t) * D + d]);
    if (q35) {
      const float g = bf(qo[((long long)t * HQ + h) * 2 * D + D + d]);
      y = rbf(y * rbf(1.f / (1.f + expf(-g))));
    }
    out[((long long)t * HQ + h) * D + d] = tobf(y);
  }
}

// torch.argmax of one bf16 row: first maximal index, NaN counts as the maximum.
__global__ void __launch_bounds__(1024) argmax_kernel(const bf16 *row, int n, int64_t *token) {
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = bf(row[i]);
    if (argmax_better(v, i, bv, bi)) { bv = v; bi = i; }
  }
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
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (argmax_better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
    *token = bi;
  }
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
  auto gemm = [&](int n, int k, const bf16 *xin, const void *w, bf16 *o) {
    return xb_gemm_bf16(T, n, k, xin, w, o, stream);
  };
  const long long nH = (long long)T * H;
  const int eb = 296;  // elementwise grid: 2 CTAs per SM
  embed_kernel<<<T, 128, 0, st>>>(a->input_ids, (const bf16 *)model->w.embed, h, H, g.vocab, err);
  XB_LAUNCHED();
  for (int l = 0; l < g.num_layers; ++l) {
    const XbLayerWeights &w = model->w.layers[l];
    const XbLayerState &s = a->layers[l];
    rmsnorm_kernel<<<T, 256, 0, st>>>(h, (const bf16 *)w.input_norm, x, H, g.rms_eps, q35);
    XB_LAUNCHED();
    if (g.layer_kind[l] == XB_LAYER_DELTANET) {
      XB_TRY(gemm(CH, H, x, w.in_qkv, P(L.qkv)));
      XB_TRY(gemm(HV * DK, H, x, w.in_z, P(L.z)));
      XB_TRY(gemm(HV, H, x, w.in_b, P(L.bb)));
      XB_TRY(gemm(HV, H, x, w.in_a, P(L.aa)));
      delta_prepare_kernel<<<dim3(T, HV), 256, 0, st>>>(
          P(L.qkv), P(L.bb), P(L.aa), (const bf16 *)s.conv_in, (const bf16 *)w.conv_w, (const bf16 *)w.a_log,
          (const bf16 *)w.dt_bias, F(L.qn), F(L.kn), F(L.vv), F(L.beta), F(L.decay), HK, HV, DK,
          (float)(1.0 / std::sqrt((double)DK)));
      XB_LAUNCHED();
      conv_state_kernel<<<(CH + 255) / 256, 256, 0, st>>>(P(L.qkv), (const bf16 *)s.conv_in, (bf16 *)s.conv_out, CH, T);
      XB_LAUNCHED();
      delta_scan_kernel<<<dim3(HV, DK / 16), 256, 0, st>>>(F(L.qn), F(L.kn), F(L.vv), F(L.beta), F(L.decay),
                                                           (const float *)s.rec_in, (float *)s.rec_out,
                                                           P(L.core), HV, DK, T);
      XB_LAUNCHED();
      gated_norm_kernel<<<dim3(T, HV), 128, 0, st>>>(P(L.core), P(L.z), (const bf16 *)w.gnorm, x2, HV, DK, g.rms_eps);
      XB_LAUNCHED();
      XB_TRY(gemm(H, HV * DK, x2, w.out_proj, out));
    } else {
      const int qrows = HQ * D * (q35 ? 2 : 1);
      bf16 *qo = P(L.qkv), *ko = P(L.z), *vo = P(L.bb);
      XB_TRY(gemm(qrows, H, x, w.q_proj, qo));
      XB_TRY(gemm(HKV * D, H, x, w.k_proj, ko));
      XB_TRY(gemm(HKV * D, H, x, w.v_proj, vo));
      attn_prep_kernel<<<dim3(T, HQ + 2 * HKV), 32, 0, st>>>(
          qo, ko, vo, (const bf16 *)w.q_norm, (const bf16 *)w.k_norm, model->d_inv_freq, P(L.qatt),
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
      attn_out_kernel<<<dim3(T, HQ), 128, 0, st>>>(P(L.oatt), qo, x2, HQ, D, T, q35);
      XB_LAUNCHED();
      XB_TRY(gemm(H, HQ * D, x2, w.o_proj, out));
    }
    add_kernel<<<eb, 256, 0, st>>>(h, out, nH);
    XB_LAUNCHED();
    rmsnorm_kernel<<<T, 256, 0, st>>>(h, (const bf16 *)w.post_norm, x, H, g.rms_eps, q35);
    XB_LAUNCHED();
    XB_TRY(gemm(I, H, x, w.gate, P(L.gate)));
    XB_TRY(gemm(I, H, x, w.up, P(L.up)));
    silu_mul_kernel<<<eb, 256, 0, st>>>(P(L.gate), P(L.up), x2, (long long)T * I);
    XB_LAUNCHED();
    XB_TRY(gemm(H, I, x2, w.down, out));
    add_kernel<<<eb, 256, 0, st>>>(h, out, nH);
    XB_LAUNCHED();
  }
  // the last token: final norm, lm_head, argmax (ModelStep's last-token gather, model.py:178-183)
  rmsnorm_kernel<<<1, 256, 0, st>>>(h + (long long)(T - 1) * H, (const bf16 *)model->w.final_norm, P(L.xlast), H,
                                    g.rms_eps, q35);
  XB_LAUNCHED();
  XB_TRY(xb_gemm_bf16(1, g.vocab, H, P(L.xlast), model->w.lm_head, a->logits, stream));
  if (a->next_token) {
    argmax_kernel<<<1, 1024, 0, st>>>((const bf16 *)a->logits, g.vocab, a->next_token);
    XB_LAUNCHED();
  }
#undef XB_TRY
#undef XB_LAUNCHED
  return XB_OK;
}
