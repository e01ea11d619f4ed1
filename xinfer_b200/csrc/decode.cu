// Host side of the decode megakernel: model plan, workspace, launches, C ABI (include/xinfer_b200.h).
// The kernels of batch rows 1 and 2 are compiled here; those of 4 and 8 in decode_tc.cu.

#include "decode_kernel.cuh"
#include "xb_host.h"

namespace xb {

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
thread_local std::string g_err;
static unsigned long long *g_trace = nullptr;  // xb_debug_trace

int fail(int code, const std::string &msg) {
  g_err = msg;
  return code;
}
#define XB_CUDA(call)                                                                          \
  do {                                                                                         \
    cudaError_t e_ = (call);                                                                   \
    if (e_ != cudaSuccess)                                                                     \
      return fail(XB_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));            \
  } while (0)

} // namespace xb

#ifndef XB_MIN_SPLIT_POSITIONS
#define XB_MIN_SPLIT_POSITIONS 4
#endif

namespace xb {

struct WsLayout {
  size_t ctrl, h, proj, core, ssq, att_o, att_ml, att_out, act, am_v, am_i, total;
  int pstride, max_splits;
};

static WsLayout ws_layout(const XbGeometry &g, int max_batch, int ncta) {
  WsLayout L{};
  const int B = max_batch;
  const bool q35 = g.family == XB_FAMILY_QWEN35;
  const int delta_rows = q35 ? (2 * g.lin_key_heads + 2 * g.lin_value_heads) * g.lin_head_dim +
                                   2 * g.lin_value_heads
                             : 0;
  const int attn_rows = g.num_q_heads * g.head_dim * (q35 ? 2 : 1) + 2 * g.num_kv_heads * g.head_dim;
  L.pstride = ((std::max(delta_rows, attn_rows) + 7) / 8) * 8;
  L.max_splits = ncta;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += (bytes + 255) & ~size_t(255); return o; };
  L.ctrl = take(CTL_TOTAL * 4);
  L.h = take((size_t)B * g.hidden * 4);
  L.proj = take((size_t)B * L.pstride * 4);
  const int vdim = q35 ? g.lin_value_heads * g.lin_head_dim : 8;
  L.core = take((size_t)B * vdim * 4);
  L.ssq = take((size_t)B * (q35 ? g.lin_value_heads : 1) * 8 * 8);
  L.att_o = take((size_t)B * g.num_q_heads * L.max_splits * g.head_dim * 8);
  L.att_ml = take((size_t)B * g.num_q_heads * L.max_splits * 16);  // (M, L) pairs
  L.att_out = take((size_t)B * g.num_q_heads * g.head_dim * 4);
  L.act = take((size_t)B * g.intermediate * 4);
  L.am_v = take((size_t)ncta * XB_MAX_BATCH * 4);
  L.am_i = take((size_t)ncta * XB_MAX_BATCH * 4);
  L.total = off;
  return L;
}

static int check_geometry(const XbGeometry &g) {
  const bool q35 = g.family == XB_FAMILY_QWEN35;
  if (g.family != XB_FAMILY_QWEN3 && !q35) return fail(XB_ERR_INVALID, "unknown model family");
  if (g.num_layers < 1 || g.num_layers > XB_MAX_LAYERS)
    return fail(XB_ERR_INVALID, "num_layers must be 1..64");
  if (g.hidden % 256 || g.intermediate % 8 || g.vocab < 1)
    return fail(XB_ERR_INVALID, "hidden must be a multiple of 256, intermediate of 8");
  if (g.num_kv_heads < 1 || g.num_q_heads % g.num_kv_heads)
    return fail(XB_ERR_INVALID, "query heads must be a positive multiple of KV heads");
  const int G = g.num_q_heads / g.num_kv_heads;
  if (G > 4) return fail(XB_ERR_UNSUPPORTED, "at most 4 query heads per KV head");
  if (g.head_dim != 128 && g.head_dim != 256)
    return fail(XB_ERR_UNSUPPORTED, "head_dim must be 128 or 256");
  if (g.rotary_dim < 2 || g.rotary_dim > g.head_dim || g.rotary_dim % 2 || g.rotary_dim > 2 * kRopeFreqs)
    return fail(XB_ERR_INVALID, "invalid rotary_dim (even, <= head_dim and <= 128)");
  if (g.capacity < 1) return fail(XB_ERR_INVALID, "capacity must be positive");
  if (g.state_rows < 1 || g.state_rows > XB_MAX_BATCH)
    return fail(XB_ERR_INVALID, "state_rows must be 1..8");
  for (int l = 0; l < g.num_layers; ++l) {
    const int k = g.layer_kind[l];
    if (k != XB_LAYER_ATTENTION && k != XB_LAYER_DELTANET)
      return fail(XB_ERR_INVALID, "invalid layer kind");
    if (k == XB_LAYER_DELTANET && !q35)
      return fail(XB_ERR_INVALID, "DeltaNet layers need the Qwen3.5 family");
  }
  if (q35) {
    if (g.lin_head_dim != 128 || g.lin_key_heads < 1 || g.lin_value_heads % g.lin_key_heads ||
        g.conv_width != 4)
      return fail(XB_ERR_UNSUPPORTED, "DeltaNet needs key/value dim 128, width-4 conv");
    if (g.lin_value_heads * g.lin_head_dim > 8192 || 2 * g.lin_head_dim > kCT)
      return fail(XB_ERR_UNSUPPORTED, "DeltaNet value width too large");
  }
  if (g.hidden > kResRows * 148)
    return fail(XB_ERR_UNSUPPORTED, "hidden size too large for the per-CTA residual rows");
  // every GEMV must fit at least one row (two for gate/up) into a 32 KB ring slot
  const int kmax = std::max(g.intermediate, std::max(g.hidden, g.num_q_heads * g.head_dim));
  if (kmax * 2 > kSlot || g.hidden * 4 > kSlot)
    return fail(XB_ERR_UNSUPPORTED, "GEMV input dimension too large for a ring slot");
  return XB_OK;
}

// Weight pointers: every tensor the geometry uses must be present, and the matrices the kernel
// streams with bulk copies (and lm_head) must be 16-byte aligned. Shared by xb_model_create and
// xb_decode_step_static.
static int check_weights(const XbGeometry &g, const XbModelWeights &weights) {
  auto aligned = [](const void *ptr) { return ((uintptr_t)ptr & 15) == 0; };
  if (!weights.embed || !weights.final_norm || !weights.lm_head)
    return fail(XB_ERR_INVALID, "embed, final_norm and lm_head are required");
  if (!aligned(weights.lm_head)) return fail(XB_ERR_INVALID, "lm_head must be 16-byte aligned");
  for (int l = 0; l < g.num_layers; ++l) {
    const XbLayerWeights &w = weights.layers[l];
    std::vector<const void *> need = {w.input_norm, w.post_norm, w.gate, w.up, w.down};
    std::vector<const void *> streamed = {w.gate, w.up, w.down};
    if (g.layer_kind[l] == XB_LAYER_DELTANET) {
      for (auto q : {w.in_qkv, w.in_z, w.in_b, w.in_a, w.conv_w, w.a_log, w.dt_bias, w.gnorm,
                     w.out_proj})
        need.push_back(q);
      for (auto q : {w.in_qkv, w.in_z, w.in_b, w.in_a, w.out_proj}) streamed.push_back(q);
    } else {
      for (auto q : {w.q_proj, w.k_proj, w.v_proj, w.o_proj, w.q_norm, w.k_norm}) need.push_back(q);
      for (auto q : {w.q_proj, w.k_proj, w.v_proj, w.o_proj}) streamed.push_back(q);
    }
    for (auto q : need)
      if (!q) return fail(XB_ERR_INVALID, "missing weight pointer in layer " + std::to_string(l));
    for (auto q : streamed)
      if (!aligned(q))
        return fail(XB_ERR_INVALID, "projection weights must be 16-byte aligned (layer " +
                                        std::to_string(l) + ")");
  }
  return XB_OK;
}

// The workspace layout is fixed by the workspace size: the largest batch whose layout fits, so
// the tagged words keep their addresses whatever batch size and split count a launch uses.
static int ws_layout_for(const XbGeometry &g, size_t workspace_bytes, int ncta, WsLayout &L, int &bcap) {
  for (int b = XB_MAX_BATCH; b >= 1; --b) {
    L = ws_layout(g, b, ncta);
    if (L.total <= workspace_bytes) { bcap = b; return XB_OK; }
  }
  bcap = 0;
  return fail(XB_ERR_INVALID, "workspace too small");
}

static size_t ubytes_for(const XbGeometry &g, int NB) {
  const bool q35 = g.family == XB_FAMILY_QWEN35;
  int kmax = std::max(g.hidden, g.intermediate);
  kmax = std::max(kmax, g.num_q_heads * g.head_dim);
  if (q35) kmax = std::max(kmax, g.lin_value_heads * g.lin_head_dim);
  const size_t act = (size_t)NB * (kmax * 2 + (NB >= 4 ? 16 : 0));  // padded rows at batch >= 4
  const int G = g.num_q_heads / g.num_kv_heads;
  const size_t att = ((size_t)G * g.head_dim + 2 * g.head_dim + (size_t)kWarps * (g.head_dim + 2)) * 4;
  const size_t u = std::max(act, att);
  return (u + 127) & ~size_t(127);
}

// Which long-context kernel serves a launch of one or two rows: 0 (the standard kernel) unless a
// split-KV item of an attention layer spans at least kAttBlockMin positions and the head geometry
// has a long-context kernel (1: head dimension 128, G <= 2; 2: head dimension 256, G <= 4).
static int long_attention_kind(const StepParams &p) {
  if (p.L <= 0 || p.delta_mask == (p.L >= 64 ? ~0ull : ((1ull << p.L) - 1))) return 0;
  int longest = 0;
  for (int b = 0; b < p.B; ++b)
    if (p.q_len[b] > 0) longest = std::max(longest, (p.kv_len[b] + p.splits - 1) / p.splits);
  if (longest < kAttBlockMin) return 0;
  const int G = p.HQ / p.HKV;
  if (p.D == 128 && G <= 2) return 1;
  if (p.D == 256 && G <= 4) return 2;
  return 0;
}

template <int NB>
static int launch(const StepParams &prm, size_t smem, int ncta, cudaStream_t stream) {
  const int kind = NB <= 2 ? long_attention_kind(prm) : 0;
  const bool wide = NB <= 2 && prm.H >= kWideHidden;
  cudaError_t e = NB >= 4 ? launch_tensor_tiles(NB, prm, smem, ncta, stream)
                  : wide && kind == 2 ? launch_wide_long(NB, prm, smem, ncta, stream)
                  : wide && kind == 0 ? launch_wide(NB, prm, smem, ncta, stream)
                  : kind ? launch_long_attention(NB, kind, prm, smem, ncta, stream)
                         : launch_decode<(NB >= 4 ? 1 : NB)>(prm, smem, ncta, stream);
  if (e != cudaSuccess) return fail(XB_ERR_CUDA, std::string("decode launch: ") + cudaGetErrorString(e));
  return XB_OK;
}

} // namespace xb

using namespace xb;

extern "C" {

const char *xb_last_error(void) { return g_err.c_str(); }
int xb_abi_version(void) { return XB_ABI_VERSION; }

int xb_debug_fault(int32_t withhold_stage, uint64_t wait_limit_ns) {
  const int stage = withhold_stage < 0 ? -1 : withhold_stage;
  const unsigned long long limit = wait_limit_ns ? wait_limit_ns : kWaitLimitNs;
  if (limit < 1000000ull) return fail(XB_ERR_INVALID, "wait limit below 1 ms");
  XB_CUDA(set_fault_constants(stage, limit));
  XB_CUDA(set_fault_tensor_tiles(stage, limit));
  XB_CUDA(set_fault_long_attention(stage, limit));
  XB_CUDA(set_fault_wide(stage, limit));
  XB_CUDA(set_fault_wide_long(stage, limit));
  return XB_OK;
}

int xb_debug_trace(void *device_buffer, size_t bytes) {
  const size_t need = (size_t)kTraceStride * 8 * 1024;
  if (device_buffer && bytes < need)
    return fail(XB_ERR_INVALID, "trace buffer needs " + std::to_string(need) + " bytes");
  g_trace = static_cast<unsigned long long *>(device_buffer);
  return XB_OK;
}

int xb_rope_inv_freq(float theta, int32_t rotary_dim, float *out) {
  if (!out || rotary_dim < 2 || rotary_dim % 2 || !(theta > 0.f))
    return fail(XB_ERR_INVALID, "invalid RoPE parameters");
  for (int i = 0; i < rotary_dim / 2; ++i) {
    const float expo = (float)(2 * i) / (float)rotary_dim;
    out[i] = 1.0f / powf(theta, expo);
  }
  return XB_OK;
}

int xb_model_create(const XbGeometry *geometry, const XbModelWeights *weights, XbModel **model) {
  if (!geometry || !weights || !model) return fail(XB_ERR_INVALID, "null argument");
  *model = nullptr;
  int rc = check_geometry(*geometry);
  if (rc) return rc;
  const XbGeometry &g = *geometry;
  rc = check_weights(g, *weights);
  if (rc) return rc;
  XbModel *m = new XbModel();
  m->g = g;
  m->w = *weights;
  cudaGetDevice(&m->device);
  cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, m->device);
  if (cudaMalloc(&m->d_layers, sizeof(XbLayerWeights) * g.num_layers) != cudaSuccess ||
      cudaMalloc(&m->d_inv_freq, sizeof(float) * (g.rotary_dim / 2)) != cudaSuccess) {
    cudaFree(m->d_layers);
    delete m;
    return fail(XB_ERR_CUDA, "cudaMalloc failed for the model plan");
  }
  // RoPE inverse frequencies as the HF default rope init: 1 / theta^(2i / dim), fp32.
  std::vector<float> inv(g.rotary_dim / 2);
  if (g.rope_inv_freq) {
    memcpy(inv.data(), g.rope_inv_freq, sizeof(float) * inv.size());
  } else {
    xb_rope_inv_freq(g.rope_theta, g.rotary_dim, inv.data());
  }
  cudaMemcpy(m->d_layers, weights->layers, sizeof(XbLayerWeights) * g.num_layers,
             cudaMemcpyHostToDevice);
  cudaMemcpy(m->d_inv_freq, inv.data(), sizeof(float) * inv.size(), cudaMemcpyHostToDevice);
  *model = m;
  return XB_OK;
}

int xb_model_destroy(XbModel *model) {
  if (!model) return XB_OK;
  cudaFree(model->d_layers);
  cudaFree(model->d_inv_freq);
  delete model;
  return XB_OK;
}

int xb_decode_workspace_bytes(const XbModel *model, int32_t max_batch, size_t *bytes) {
  if (!model || !bytes) return fail(XB_ERR_INVALID, "null argument");
  if (max_batch < 1 || max_batch > XB_MAX_BATCH) return fail(XB_ERR_INVALID, "max_batch 1..8");
  *bytes = ws_layout(model->g, max_batch, model->num_sms).total;
  return XB_OK;
}

int xb_workspace_init(void *workspace, size_t workspace_bytes, void *stream) {
  if (!workspace) return fail(XB_ERR_INVALID, "null workspace");
  XB_CUDA(cudaMemsetAsync(workspace, 0, workspace_bytes, (cudaStream_t)stream));
  return XB_OK;
}

int xb_workspace_check(void *workspace, void *stream, int32_t *device_error) {
  if (!workspace) return fail(XB_ERR_INVALID, "null workspace");
  unsigned err = 0;
  XB_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  XB_CUDA(cudaMemcpy(&err, (unsigned *)workspace + CTL_ERR, 4, cudaMemcpyDeviceToHost));
  if (device_error) *device_error = (int32_t)err;
  if (err) {
    // reset the control words so the workspace can be reused (the epoch word is kept)
    XB_CUDA(cudaMemset(workspace, 0, CTL_WORDS * 4));
    return fail(XB_ERR_DEVICE, "device-side error code " + std::to_string(err));
  }
  return XB_OK;
}

int xb_decode_step(const XbModel *model, const XbStepArgs *args, void *workspace,
                   size_t workspace_bytes, void *stream) {
  if (!model || !args || !workspace) return fail(XB_ERR_INVALID, "null argument");
  const XbGeometry &g = model->g;
  const int B = args->batch;
  if (B < 1 || B > XB_MAX_BATCH || B > g.state_rows)
    return fail(XB_ERR_INVALID, "batch must be 1..min(8, state_rows)");
  if (!args->logits) return fail(XB_ERR_INVALID, "logits are required");
  if (!args->input_ids != !args->cache_position)
    return fail(XB_ERR_INVALID, "pass both input_ids and cache_position on the device, or neither");
  int active = 0, max_kv = 1;
  for (int b = 0; b < B; ++b) {
    const int q = args->query_lengths[b], kv = args->kv_lengths[b];
    if (q != 0 && q != 1) return fail(XB_ERR_INVALID, "decode query lengths must be 0 or 1");
    if (kv < q || kv < 1 || kv > g.capacity) return fail(XB_ERR_INVALID, "Invalid query/KV lengths");
    active += q;
    max_kv = std::max(max_kv, kv);
  }
  if (!active) return fail(XB_ERR_INVALID, "at least one row must be active");
  for (int l = 0; l < g.num_layers; ++l) {
    const XbLayerState &s = args->layers[l];
    if (g.layer_kind[l] == XB_LAYER_DELTANET) {
      if (!s.conv_in || !s.rec_in || !s.conv_out || !s.rec_out)
        return fail(XB_ERR_INVALID, "missing DeltaNet state in layer " + std::to_string(l));
      // conv_out / rec_out either equal their input (update in place) or do not overlap it.
    } else if (!s.k_cache || !s.v_cache) {
      return fail(XB_ERR_INVALID, "missing KV cache in layer " + std::to_string(l));
    }
  }
  const int ncta = model->num_sms;
  WsLayout Lb;
  int bcap = 0;
  int lrc = ws_layout_for(g, workspace_bytes, ncta, Lb, bcap);
  if (lrc) return lrc;
  if (bcap < B)
    return fail(XB_ERR_INVALID, "workspace too small for batch " + std::to_string(B));
  if (((uintptr_t)workspace & 255) != 0) return fail(XB_ERR_INVALID, "workspace must be 256-byte aligned");

  StepParams p;
  memset(&p, 0, sizeof(p));
  const bool q35 = g.family == XB_FAMILY_QWEN35;
  p.family = g.family; p.L = g.num_layers; p.H = g.hidden; p.I = g.intermediate; p.V = g.vocab;
  p.HQ = g.num_q_heads; p.HKV = g.num_kv_heads; p.D = g.head_dim; p.RD = g.rotary_dim;
  p.HK = q35 ? g.lin_key_heads : 1; p.HV = q35 ? g.lin_value_heads : 1;
  p.DK = q35 ? g.lin_head_dim : 128; p.CW = q35 ? g.conv_width : 4; p.C = g.capacity;
  p.rows_alloc = g.state_rows; p.eps = g.rms_eps;
  // (float)(d ** -0.5) as the reference's Python constants: recurrent.py:23, attention scaling.
  p.dk_scale = (float)(1.0 / std::sqrt((double)p.DK));
  p.att_scale = (float)(1.0 / std::sqrt((double)g.head_dim));
  p.pstride = Lb.pstride;
  // split-KV: enough (row, kv head, split) items to cover every SM, but at least
  // XB_MIN_SPLIT_POSITIONS positions per split (fewer partials for the combine to merge)
  int splits = std::max(1, ncta / std::max(1, active * g.num_kv_heads));
  splits = std::min(splits, std::max(1, (max_kv + XB_MIN_SPLIT_POSITIONS - 1) / XB_MIN_SPLIT_POSITIONS));
  splits = std::min(splits, std::min(Lb.max_splits, 160));
  p.splits = splits;
  p.ncta = ncta;
  p.B = B;
  for (int b = 0; b < B; ++b) { p.kv_len[b] = args->kv_lengths[b]; p.q_len[b] = args->query_lengths[b]; }
  p.delta_mask = 0;
  for (int l = 0; l < g.num_layers; ++l)
    if (g.layer_kind[l] == XB_LAYER_DELTANET) p.delta_mask |= 1ull << l;
  p.layers = model->d_layers;
  p.embed = (const bf16 *)model->w.embed;
  p.final_norm = (const bf16 *)model->w.final_norm;
  p.lm_head = (const bf16 *)model->w.lm_head;
  p.inv_freq = model->d_inv_freq;
  p.ids = args->input_ids;
  p.pos = args->cache_position;
  for (int b = 0; b < B; ++b) {
    p.hid[b] = args->host_ids[b];
    p.hpos[b] = args->host_positions[b];
    if (!p.ids && (args->host_ids[b] < 0 || args->host_ids[b] >= g.vocab))
      return fail(XB_ERR_INVALID, "token id out of range");
  }
  for (int l = 0; l < g.num_layers; ++l) {
    const XbLayerState &s = args->layers[l];
    if (g.layer_kind[l] == XB_LAYER_DELTANET) {
      p.sa[l] = const_cast<void *>(s.conv_in);
      p.sb[l] = const_cast<void *>(s.rec_in);
      p.sc[l] = s.conv_out;
      p.sd[l] = s.rec_out;
    } else {
      p.sa[l] = s.k_cache;
      p.sb[l] = s.v_cache;
    }
  }
  p.logits = (bf16 *)args->logits;
  p.tokens = args->next_tokens;
  char *ws = (char *)workspace;
  p.ctrl = (unsigned *)(ws + Lb.ctrl);
  p.h = (unsigned *)(ws + Lb.h);
  p.proj = (unsigned *)(ws + Lb.proj);
  p.core = (unsigned *)(ws + Lb.core);
  p.ssq = (u64 *)(ws + Lb.ssq);
  p.att_o = (u64 *)(ws + Lb.att_o);
  p.att_ml = (u64 *)(ws + Lb.att_ml);
  p.att_out = (unsigned *)(ws + Lb.att_out);
  p.act = (unsigned *)(ws + Lb.act);
  p.am_v = (float *)(ws + Lb.am_v);
  p.am_i = (int *)(ws + Lb.am_i);
  // everything after the control words, up to the end of the workspace
  p.scrub_base = (uint4 *)(ws + Lb.h);
  p.scrub_chunks = (unsigned)((workspace_bytes - Lb.h) / 16);
  p.trace = g_trace;

  const int NB = B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : 8;
  p.ubytes = (int)ubytes_for(g, NB);
  const size_t fixed = kUOffset + (size_t)p.ubytes;
  int nslots = (int)((kSmemLimit - fixed) / kSlot);
  nslots = std::min(nslots, kMaxSlots);
  if (nslots < 2) return fail(XB_ERR_UNSUPPORTED, "not enough shared memory for the weight ring");
  p.nslots = nslots;
  const size_t smem = fixed + (size_t)nslots * kSlot;
  cudaStream_t st = (cudaStream_t)stream;
  switch (NB) {
  case 1: return launch<1>(p, smem, ncta, st);
  case 2: return launch<2>(p, smem, ncta, st);
  case 4: return launch<4>(p, smem, ncta, st);
  default: return launch<8>(p, smem, ncta, st);
  }
}

} // extern "C"

// ------------------------------------------------------------------------------------------
// Allocation-free variant of xb_decode_step.
//
// Some callers cannot allocate device memory at the moment they run a decode step: serving
// stacks that reserve (nearly) all of HBM for their own pool at start-up, so a later cudaMalloc
// fails or fragments that pool, and hosts with a fixed memory plan that forbids allocations
// after initialisation. This entry point needs neither an XbModel (whose
// creation allocates the weight table) nor a caller workspace: the per-layer weight table, the
// RoPE table and the kernel's scratch all live in one file-scope device array of
// XB_STATIC_SCRATCH_BYTES, which every GPU that loads this library keeps until the process exits.
// ------------------------------------------------------------------------------------------
namespace xb {

constexpr size_t kStaticScratchBytes = XB_STATIC_SCRATCH_BYTES;
constexpr size_t kStaticTableBytes = sizeof(XbLayerWeights) * XB_MAX_LAYERS;   // weight table
constexpr size_t kStaticRopeBytes = 4096;                                      // inv_freq floats
constexpr size_t kStaticWsOffset = ((kStaticTableBytes + kStaticRopeBytes) + 255) & ~size_t(255);
constexpr int kStaticMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

struct StaticDevice {
  bool ready = false;
  unsigned char *base = nullptr;  // device address of g_static_scratch on this device
  int num_sms = 0;
};

} // namespace xb

extern "C" int xb_decode_step_static(const XbGeometry *geometry, const XbModelWeights *weights,
                                     const XbStepArgs *args, void *stream,
                                     int32_t *device_error) {
  using namespace xb;
  static std::mutex mu;
  static StaticDevice devices[kStaticMaxDevices];
  if (!geometry || !weights || !args) return fail(XB_ERR_INVALID, "null argument");
  int rc = check_geometry(*geometry);
  if (rc) return rc;
  const XbGeometry &g = *geometry;
  const int B = args->batch;
  if (B < 1 || B > XB_MAX_BATCH) return fail(XB_ERR_INVALID, "batch must be 1..8");
  int dev = 0;
  XB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kStaticMaxDevices) return fail(XB_ERR_UNSUPPORTED, "device ordinal too large");
  StaticDevice sd;
  {
    // One-time set-up per device, with that device current: look up the device address of the
    // static array (host code may not use the symbol's host-side name as a device address).
    std::lock_guard<std::mutex> lock(mu);
    StaticDevice &d = devices[dev];
    if (!d.ready) {
      void *ptr = nullptr;
      XB_CUDA(cudaGetSymbolAddress(&ptr, g_static_scratch));
      int sms = 0;
      XB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
      d.base = static_cast<unsigned char *>(ptr);
      d.num_sms = sms;
      d.ready = true;
    }
    sd = d;
  }
  const size_t ws_bytes = ws_layout(g, B, sd.num_sms).total;
  const size_t ws_room = kStaticScratchBytes - kStaticWsOffset;
  if (ws_bytes > ws_room)
    return fail(XB_ERR_INVALID,
                "xb_decode_step_static: this model and batch need " + std::to_string(ws_bytes) +
                    " bytes of scratch, more than the " + std::to_string(ws_room) +
                    " bytes of the static array (use xb_decode_step with a workspace)");
  if ((size_t)(g.rotary_dim / 2) * sizeof(float) > kStaticRopeBytes)
    return fail(XB_ERR_INVALID, "rotary_dim too large for the static RoPE table");
  cudaStream_t st = (cudaStream_t)stream;
  unsigned char *table = sd.base;
  unsigned char *rope = sd.base + kStaticTableBytes;
  unsigned char *ws = sd.base + kStaticWsOffset;
  // The same weight-pointer rules as xb_model_create.
  rc = check_weights(g, *weights);
  if (rc) return rc;
  // Stage the weight table and RoPE frequencies into the static array (stream-ordered copies
  // from host memory; no allocation). Every call rewrites them.
  float inv[kStaticRopeBytes / sizeof(float)];
  if (g.rope_inv_freq) memcpy(inv, g.rope_inv_freq, sizeof(float) * (g.rotary_dim / 2));
  else xb_rope_inv_freq(g.rope_theta, g.rotary_dim, inv);
  XB_CUDA(cudaMemcpyAsync(table, weights->layers, sizeof(XbLayerWeights) * g.num_layers,
                          cudaMemcpyHostToDevice, st));
  XB_CUDA(cudaMemcpyAsync(rope, inv, sizeof(float) * (g.rotary_dim / 2), cudaMemcpyHostToDevice, st));
  // The array keeps the previous call's contents; the barrier / error / completion words must
  // start at zero, so clear them before every launch.
  XB_CUDA(cudaMemsetAsync(ws, 0, CTL_WORDS * 4, st));
  XbModel m;
  m.g = g;
  m.w = *weights;
  m.d_layers = reinterpret_cast<XbLayerWeights *>(table);
  m.d_inv_freq = reinterpret_cast<float *>(rope);
  m.device = dev;
  m.num_sms = sd.num_sms;
  // Same validation and launch as xb_decode_step; the model is a host-stack view. The scratch
  // is the whole rest of the array, so the kernel's periodic clear of its tagged words covers
  // what any earlier call (of any model) wrote there.
  rc = xb_decode_step(&m, args, ws, ws_room, stream);
  if (rc) return rc;
  if (device_error) {
    unsigned err = 0;
    XB_CUDA(cudaStreamSynchronize(st));
    XB_CUDA(cudaMemcpy(&err, ws + CTL_ERR * 4, 4, cudaMemcpyDeviceToHost));
    *device_error = (int32_t)err;
    if (err) return fail(XB_ERR_DEVICE, "device-side error code " + std::to_string(err));
  }
  return XB_OK;
}
