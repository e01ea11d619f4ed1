// Torch custom operators over the decode step of libxinfer_b200.so, and their AOTInductor C shims.
//
// This is the boundary the reference's export path binds (compiler/common/package.py:36-86 embeds
// native libraries and C shims into decode.pt2; compiler/common/kernels/attention_shim.cpp:5-32
// is the shim pattern): two operators in the `xinfer` namespace,
//
//   xinfer::qwen35_decode_step(Tensor input_ids, Tensor cache_position, Tensor(a!)[] state,
//                              Tensor kv_lengths, Tensor query_lengths, Tensor[] weights,
//                              int[] geometry, float[] params) -> Tensor[]
//   xinfer::qwen3_decode_step(...same arguments...) -> Tensor
//
// with the tensor contract of ModelStep.forward at T == 1 (compiler/qwen35/model.py:162-183,
// compiler/qwen3/model.py:70-95): input_ids / cache_position CUDA int64 [B, 1]; state in the
// reference's order (per layer key, value or conv, recurrent), views of the first B rows; KV
// caches are appended in place (hence the mutable annotation); kv_lengths / query_lengths CPU
// int32 [B]. qwen35_decode_step returns [logits, conv_0, recurrent_0, conv_1, ...]: bf16 logits
// [B, vocab] and, for every DeltaNet layer in order, fresh replacement conv / recurrent tensors
// (the inputs are not modified). qwen3_decode_step returns the logits. Outputs are allocated
// through ATen's caching allocator on the current CUDA stream, and the step runs on that stream.
//
// weights: the model's bf16 tensors in the order of xinfer_b200/torch_ops.py:weight_list
// (embed, final norm, lm_head, then per layer input norm, post norm, gate, up, down and the
// attention or DeltaNet tensors). geometry: XbGeometry's integer fields (family, layers, hidden,
// intermediate, vocab, q heads, KV heads, head dim, rotary dim, DeltaNet key heads, value heads,
// head dim, conv width, KV capacity, state rows) followed by one layer kind per layer; params:
// (rms_eps, rope_theta). The device plan (weight table, RoPE table, workspace) is built on the
// first call for a (device, stream, geometry, weight addresses) combination and kept for the
// life of the process.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/csrc/inductor/aoti_torch/utils.h>
#include <torch/library.h>

#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

#include "xinfer_b200.h"

namespace xinfer_b200 {

constexpr int kGeometryFields = 15;

struct Plan {
  std::vector<int64_t> key;
  XbModel *model = nullptr;
  at::Tensor workspace;
};

static std::mutex g_mu;
static std::vector<std::unique_ptr<Plan>> g_plans;

static void check_rc(int rc, const char *what) {
  TORCH_CHECK(rc == XB_OK, what, ": ", xb_last_error(), " (code ", rc, ")");
}

static XbGeometry parse_geometry(at::IntArrayRef geo, at::ArrayRef<double> params) {
  TORCH_CHECK(geo.size() >= (size_t)kGeometryFields, "geometry needs ", kGeometryFields,
              " fields plus one layer kind per layer");
  TORCH_CHECK(params.size() == 2, "params must be (rms_eps, rope_theta)");
  XbGeometry g;
  std::memset(&g, 0, sizeof(g));
  int32_t *f[kGeometryFields] = {&g.family, &g.num_layers, &g.hidden, &g.intermediate, &g.vocab,
                                 &g.num_q_heads, &g.num_kv_heads, &g.head_dim, &g.rotary_dim,
                                 &g.lin_key_heads, &g.lin_value_heads, &g.lin_head_dim,
                                 &g.conv_width, &g.capacity, &g.state_rows};
  for (int i = 0; i < kGeometryFields; ++i) *f[i] = (int32_t)geo[i];
  TORCH_CHECK(g.num_layers >= 1 && g.num_layers <= XB_MAX_LAYERS, "num_layers must be 1..64");
  TORCH_CHECK(geo.size() == (size_t)(kGeometryFields + g.num_layers),
              "geometry must end with one layer kind per layer");
  for (int l = 0; l < g.num_layers; ++l) g.layer_kind[l] = (int32_t)geo[kGeometryFields + l];
  g.rms_eps = (float)params[0];
  g.rope_theta = (float)params[1];
  g.rope_inv_freq = nullptr;  // the library computes the HF default frequencies
  return g;
}

static bool is_delta(const XbGeometry &g, int l) { return g.layer_kind[l] == XB_LAYER_DELTANET; }

static size_t weight_count(const XbGeometry &g) {
  size_t n = 3;
  for (int l = 0; l < g.num_layers; ++l) n += is_delta(g, l) ? 14 : 11;
  return n;
}

static XbModelWeights bind_weights(const XbGeometry &g, at::TensorList w, const at::Device &dev) {
  TORCH_CHECK(w.size() == weight_count(g), "expected ", weight_count(g), " weight tensors, got ",
              w.size());
  for (size_t i = 0; i < w.size(); ++i)
    TORCH_CHECK(w[i].device() == dev && w[i].scalar_type() == at::kBFloat16 && w[i].is_contiguous(),
                "weight ", i, " must be a contiguous bf16 tensor on ", dev);
  XbModelWeights m;
  std::memset(&m, 0, sizeof(m));
  size_t k = 0;
  auto next = [&]() { return w[k++].data_ptr(); };
  m.embed = next();
  m.final_norm = next();
  m.lm_head = next();
  for (int l = 0; l < g.num_layers; ++l) {
    XbLayerWeights &L = m.layers[l];
    L.input_norm = next();
    L.post_norm = next();
    L.gate = next();
    L.up = next();
    L.down = next();
    if (is_delta(g, l)) {
      L.in_qkv = next(); L.in_z = next(); L.in_b = next(); L.in_a = next(); L.conv_w = next();
      L.a_log = next(); L.dt_bias = next(); L.gnorm = next(); L.out_proj = next();
    } else {
      L.q_proj = next(); L.k_proj = next(); L.v_proj = next(); L.o_proj = next();
      L.q_norm = next(); L.k_norm = next();
    }
  }
  return m;
}

// The device plan of one (device, stream, geometry, weights) combination.
static Plan &plan_for(const XbGeometry &g, const XbModelWeights &w, at::TensorList weights,
                      at::IntArrayRef geo, at::ArrayRef<double> params, const at::Device &dev,
                      cudaStream_t stream) {
  std::vector<int64_t> key = {dev.index(), (int64_t)(uintptr_t)stream};
  key.insert(key.end(), geo.begin(), geo.end());
  for (double v : params) {
    int64_t bits;
    std::memcpy(&bits, &v, sizeof(bits));
    key.push_back(bits);
  }
  for (const auto &t : weights) key.push_back((int64_t)(uintptr_t)t.data_ptr());
  std::lock_guard<std::mutex> lock(g_mu);
  for (auto &p : g_plans)
    if (p->key == key) return *p;
  auto plan = std::make_unique<Plan>();
  plan->key = std::move(key);
  check_rc(xb_model_create(&g, &w, &plan->model), "xb_model_create");
  size_t bytes = 0;
  check_rc(xb_decode_workspace_bytes(plan->model, XB_MAX_BATCH, &bytes), "xb_decode_workspace_bytes");
  // zeroed once on this stream; it then carries the launch epoch from step to step
  plan->workspace = at::zeros({(int64_t)bytes}, at::TensorOptions().dtype(at::kByte).device(dev));
  g_plans.push_back(std::move(plan));
  return *g_plans.back();
}

// One decode step; returns [logits, fresh conv / recurrent tensors of the DeltaNet layers].
static std::vector<at::Tensor> decode_step(int family, const at::Tensor &input_ids,
                                           const at::Tensor &cache_position, at::TensorList state,
                                           const at::Tensor &kv_lengths,
                                           const at::Tensor &query_lengths, at::TensorList weights,
                                           at::IntArrayRef geometry, at::ArrayRef<double> params) {
  const XbGeometry g = parse_geometry(geometry, params);
  TORCH_CHECK(g.family == family, family == XB_FAMILY_QWEN35
                                      ? "qwen35_decode_step needs a Qwen3.5 geometry"
                                      : "qwen3_decode_step needs a Qwen3 geometry");
  TORCH_CHECK(input_ids.is_cuda() && input_ids.scalar_type() == at::kLong && input_ids.dim() == 2 &&
                  input_ids.size(1) == 1,
              "decode expects input_ids CUDA int64 [B, 1]");
  const int64_t B = input_ids.size(0);
  TORCH_CHECK(B >= 1 && B <= XB_MAX_BATCH && B <= g.state_rows, "batch must be 1..8");
  const at::Device dev = input_ids.device();
  TORCH_CHECK(cache_position.device() == dev && cache_position.scalar_type() == at::kLong &&
                  cache_position.sizes() == input_ids.sizes(),
              "cache_position must be CUDA int64 [B, 1] on the device of input_ids");
  for (const at::Tensor *t : {&kv_lengths, &query_lengths})
    TORCH_CHECK(t->device().is_cpu() && t->scalar_type() == at::kInt && t->dim() == 1 &&
                    t->size(0) == B,
                "kv_lengths / query_lengths must be CPU int32 [B]");
  TORCH_CHECK(state.size() == (size_t)(2 * g.num_layers), "incorrect state count");
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev.index()).stream();
  const XbModelWeights w = bind_weights(g, weights, dev);
  Plan &plan = plan_for(g, w, weights, geometry, params, dev, stream);

  XbStepArgs a;
  std::memset(&a, 0, sizeof(a));
  a.batch = (int32_t)B;
  const at::Tensor ids = input_ids.contiguous(), pos = cache_position.contiguous();
  a.input_ids = ids.data_ptr<int64_t>();
  a.cache_position = pos.data_ptr<int64_t>();
  const at::Tensor kv_c = kv_lengths.contiguous(), q_c = query_lengths.contiguous();
  const int32_t *kv = kv_c.data_ptr<int32_t>();
  const int32_t *q = q_c.data_ptr<int32_t>();
  for (int64_t b = 0; b < B; ++b) {
    a.kv_lengths[b] = kv[b];
    a.query_lengths[b] = q[b];
  }
  auto opts = at::TensorOptions().device(dev);
  std::vector<at::Tensor> out;
  out.push_back(at::empty({B, (int64_t)g.vocab}, opts.dtype(at::kBFloat16)));
  for (int l = 0; l < g.num_layers; ++l) {
    const at::Tensor &s0 = state[2 * l], &s1 = state[2 * l + 1];
    std::vector<int64_t> shape0, shape1;
    at::ScalarType t1;
    if (is_delta(g, l)) {
      const int64_t ch = (2 * g.lin_key_heads + g.lin_value_heads) * (int64_t)g.lin_head_dim;
      shape0 = {B, ch, g.conv_width};
      shape1 = {B, g.lin_value_heads, g.lin_head_dim, g.lin_head_dim};
      t1 = at::kFloat;
    } else {
      shape0 = shape1 = {B, g.num_kv_heads, g.capacity, g.head_dim};
      t1 = at::kBFloat16;
    }
    TORCH_CHECK(s0.device() == dev && s0.scalar_type() == at::kBFloat16 && s0.sizes() == shape0 &&
                    s0.is_contiguous() && s1.device() == dev && s1.scalar_type() == t1 &&
                    s1.sizes() == shape1 && s1.is_contiguous(),
                "incorrect state shape/dtype/device/layout in layer ", l);
    XbLayerState &ls = a.layers[l];
    if (is_delta(g, l)) {
      at::Tensor c = at::empty_like(s0), r = at::empty_like(s1);
      ls.conv_in = s0.data_ptr();
      ls.rec_in = s1.data_ptr();
      ls.conv_out = c.data_ptr();
      ls.rec_out = r.data_ptr();
      out.push_back(c);
      out.push_back(r);
    } else {
      ls.k_cache = s0.data_ptr();
      ls.v_cache = s1.data_ptr();
    }
  }
  a.logits = out[0].data_ptr();
  a.next_tokens = nullptr;
  check_rc(xb_decode_step(plan.model, &a, plan.workspace.data_ptr(), (size_t)plan.workspace.numel(),
                          stream),
           "xb_decode_step");
  return out;
}

std::vector<at::Tensor> qwen35_decode_step(const at::Tensor &input_ids, const at::Tensor &cache_position,
                                           at::TensorList state, const at::Tensor &kv_lengths,
                                           const at::Tensor &query_lengths, at::TensorList weights,
                                           at::IntArrayRef geometry, at::ArrayRef<double> params) {
  return decode_step(XB_FAMILY_QWEN35, input_ids, cache_position, state, kv_lengths, query_lengths,
                     weights, geometry, params);
}

at::Tensor qwen3_decode_step(const at::Tensor &input_ids, const at::Tensor &cache_position,
                             at::TensorList state, const at::Tensor &kv_lengths,
                             const at::Tensor &query_lengths, at::TensorList weights,
                             at::IntArrayRef geometry, at::ArrayRef<double> params) {
  return decode_step(XB_FAMILY_QWEN3, input_ids, cache_position, state, kv_lengths, query_lengths,
                     weights, geometry, params)[0];
}

// ---- xinfer_attention_ops: the reference's attention operators on libxinfer_b200's kernel ----
// Same schemas, checks and contract as compiler/common/kernels/attention.cpp:14-140: fresh
// contiguous outputs that never alias the inputs, inputs never modified, inference only.

// A view the kernel can read directly: unit feature stride, 8-element strides, 16-byte aligned.
static at::Tensor kernel_view(const at::Tensor &t) {
  bool ok = t.stride(3) == 1 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0;
  for (int i = 0; i < 3; ++i) ok = ok && t.stride(i) % 8 == 0;
  return ok ? t : t.contiguous();
}

static at::Tensor run_attention(const at::Tensor &q, const at::Tensor &k, const at::Tensor &v,
                                const int32_t *cu, int32_t count, int32_t length,
                                const at::Tensor *blocks, double scale) {
  c10::cuda::CUDAGuard guard(q.device());
  const at::Tensor query = kernel_view(q), key = kernel_view(k), value = kernel_view(v);
  at::Tensor out = at::empty(q.sizes(), q.options().memory_format(at::MemoryFormat::Contiguous));
  XbAttentionArgs a;
  std::memset(&a, 0, sizeof(a));
  a.q = query.data_ptr();
  a.k = key.data_ptr();
  a.v = value.data_ptr();
  a.out = out.data_ptr();
  const at::Tensor *t[3] = {&query, &key, &value};
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) a.strides[3 * i + j] = t[i]->stride(j);
  a.batch = (int32_t)q.size(0);
  a.q_heads = (int32_t)q.size(1);
  a.kv_heads = (int32_t)k.size(1);
  a.head_dim = (int32_t)q.size(3);
  a.q_tokens = (int32_t)q.size(2);
  a.capacity = (int32_t)k.size(2);
  a.cu_offsets = cu;
  a.count = count;
  a.length = length;
  a.scale = (float)scale;
  if (blocks) {
    a.blocks = blocks->data_ptr<int32_t>();
    a.blocks_stride = blocks->stride(0);
  }
  check_rc(xb_prefix_attention(&a, at::cuda::getCurrentCUDAStream(q.device().index()).stream()),
           "xb_prefix_attention");
  return out;
}

static void check_qkv_common(const at::Tensor &q, const at::Tensor &k, const at::Tensor &v, double scale) {
  TORCH_CHECK(q.size(1) > 0 && k.size(1) > 0 && q.size(1) % k.size(1) == 0,
              "Query heads must be a positive multiple of KV heads");
  TORCH_CHECK(q.size(3) >= 8 && q.size(3) <= 256 && q.size(3) % 8 == 0,
              "Flash head dimension must be a multiple of 8 in 8..256");
  TORCH_CHECK(std::isfinite(scale) && scale > 0, "Attention scale must be finite and positive");
  TORCH_CHECK(!q.requires_grad() && !k.requires_grad() && !v.requires_grad(),
              "xinfer attention supports inference only");
}

at::Tensor flash_attention(const at::Tensor &q, const at::Tensor &k, const at::Tensor &v,
                           const at::Tensor &extent, double scale) {
  TORCH_CHECK(q.is_cuda() && k.device() == q.device() && v.device() == q.device(),
              "xinfer attention requires Q/K/V on the same CUDA device");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 &&
                  v.scalar_type() == at::kBFloat16,
              "xinfer attention requires BF16");
  TORCH_CHECK(q.dim() == 4 && q.size(0) > 0 && q.size(2) >= 1 && q.size(2) <= 512, "Unsupported Q shape");
  TORCH_CHECK(k.dim() == 4 && v.dim() == 4 && k.size(0) == q.size(0) && k.size(2) > 0 &&
                  k.size(3) == q.size(3) && v.sizes() == k.sizes(),
              "Expected matching full-capacity K/V inputs [batch,kv_heads,capacity,head_dim]");
  check_qkv_common(q, k, v, scale);
  TORCH_CHECK(extent.device().is_cpu() && extent.scalar_type() == at::kByte && extent.dim() == 1,
              "Expected a CPU uint8 extent vector");
  const int64_t length = extent.size(0) - 1;  // metadata only; the extent's data is never read
  TORCH_CHECK(length >= q.size(2) && length <= k.size(2), "Invalid valid-prefix length");
  return run_attention(q, k, v, nullptr, (int32_t)q.size(2), (int32_t)length, nullptr, scale);
}

at::Tensor batched_flash_attention(const at::Tensor &q, const at::Tensor &k, const at::Tensor &v,
                                   const at::Tensor &offsets, const at::Tensor &cuda_offsets,
                                   const at::Tensor &blocks, double scale) {
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.sizes() == k.sizes() && k.size(0) == q.size(0) &&
                  k.size(3) == q.size(3),
              "Invalid Q/K/V shapes");
  TORCH_CHECK(q.is_cuda() && k.device() == q.device() && v.device() == q.device() &&
                  q.scalar_type() == at::kBFloat16 && k.scalar_type() == q.scalar_type() &&
                  v.scalar_type() == q.scalar_type(),
              "Expected colocated CUDA BF16 Q/K/V");
  TORCH_CHECK(q.size(2) >= 1 && q.size(2) <= 512, "Unsupported Q shape");
  check_qkv_common(q, k, v, scale);
  const int64_t batch = q.size(0);
  TORCH_CHECK(offsets.device().is_cpu() && offsets.scalar_type() == at::kInt && offsets.is_contiguous() &&
                  offsets.sizes() == at::IntArrayRef({2, batch + 1}),
              "Expected CPU int32 cumulative query/KV lengths [2,B+1]");
  TORCH_CHECK(cuda_offsets.device() == q.device() && cuda_offsets.scalar_type() == at::kInt &&
                  cuda_offsets.sizes() == offsets.sizes() && cuda_offsets.is_contiguous() &&
                  blocks.device() == q.device() && blocks.scalar_type() == at::kInt &&
                  blocks.sizes() == at::IntArrayRef({batch, 1}),
              "Invalid CUDA attention metadata");
  const int32_t *cuq = offsets.const_data_ptr<int32_t>(), *cuk = cuq + batch + 1;
  TORCH_CHECK(cuq[0] == 0 && cuk[0] == 0, "Cumulative lengths must start at zero");
  for (int64_t row = 0; row < batch; ++row) {
    const int64_t count = cuq[row + 1] - cuq[row], length = cuk[row + 1] - cuk[row];
    TORCH_CHECK(count >= 0 && count <= q.size(2) && length >= count && length >= 1 && length <= k.size(2),
                "Invalid query/KV lengths");
  }
  return run_attention(q, k, v, cuda_offsets.data_ptr<int32_t>(), 0, 0, &blocks, scale);
}

} // namespace xinfer_b200

TORCH_LIBRARY_FRAGMENT(xinfer, m) {
  m.def("batched_flash_attention(Tensor q, Tensor k, Tensor v, Tensor offsets, "
        "Tensor cuda_offsets, Tensor blocks, float scale) -> Tensor",
        {at::Tag::flexible_layout});
  m.def("flash_attention(Tensor q, Tensor k, Tensor v, Tensor kv_extent, float scale) -> Tensor",
        {at::Tag::flexible_layout});
  m.def("qwen35_decode_step(Tensor input_ids, Tensor cache_position, Tensor(a!)[] state, "
        "Tensor kv_lengths, Tensor query_lengths, Tensor[] weights, int[] geometry, "
        "float[] params) -> Tensor[]");
  m.def("qwen3_decode_step(Tensor input_ids, Tensor cache_position, Tensor(a!)[] state, "
        "Tensor kv_lengths, Tensor query_lengths, Tensor[] weights, int[] geometry, "
        "float[] params) -> Tensor");
}

TORCH_LIBRARY_IMPL(xinfer, CUDA, m) {
  m.impl("qwen35_decode_step", TORCH_FN(xinfer_b200::qwen35_decode_step));
  m.impl("qwen3_decode_step", TORCH_FN(xinfer_b200::qwen3_decode_step));
  m.impl("batched_flash_attention", TORCH_FN(xinfer_b200::batched_flash_attention));
  m.impl("flash_attention", TORCH_FN(xinfer_b200::flash_attention));
}

// AOTInductor C shims (the pattern of compiler/common/kernels/attention_shim.cpp:5-32): borrowed
// handles in, new handles out, C++ exceptions converted to AOTITorchError. A list argument is a
// handle array and its length; the qwen35 outputs are written to `outputs`, whose length must be
// 1 + 2 * (number of DeltaNet layers).
extern "C" AOTI_TORCH_EXPORT AOTITorchError aoti_torch_cuda_qwen35_decode_step(
    AtenTensorHandle input_ids, AtenTensorHandle cache_position, const AtenTensorHandle *state,
    int64_t state_len_, AtenTensorHandle kv_lengths, AtenTensorHandle query_lengths,
    const AtenTensorHandle *weights, int64_t weights_len_, const int64_t *geometry,
    int64_t geometry_len_, const double *params, int64_t params_len_, AtenTensorHandle *outputs,
    int64_t outputs_len_) {
  AOTI_TORCH_CONVERT_EXCEPTION_TO_ERROR_CODE({
    namespace ai = torch::aot_inductor;
    auto result = xinfer_b200::qwen35_decode_step(
        ai::resolve_tensor_dispatch_flags(input_ids), ai::resolve_tensor_dispatch_flags(cache_position),
        ai::resolve_tensor_list_dispatch_flags(state, state_len_),
        ai::resolve_tensor_dispatch_flags(kv_lengths), ai::resolve_tensor_dispatch_flags(query_lengths),
        ai::resolve_tensor_list_dispatch_flags(weights, weights_len_),
        at::IntArrayRef(geometry, (size_t)geometry_len_), at::ArrayRef<double>(params, (size_t)params_len_));
    TORCH_CHECK((int64_t)result.size() == outputs_len_, "expected ", result.size(), " output handles");
    for (size_t i = 0; i < result.size(); ++i) outputs[i] = ai::new_tensor_handle(std::move(result[i]));
  });
}

extern "C" AOTI_TORCH_EXPORT AOTITorchError aoti_torch_cuda_qwen3_decode_step(
    AtenTensorHandle input_ids, AtenTensorHandle cache_position, const AtenTensorHandle *state,
    int64_t state_len_, AtenTensorHandle kv_lengths, AtenTensorHandle query_lengths,
    const AtenTensorHandle *weights, int64_t weights_len_, const int64_t *geometry,
    int64_t geometry_len_, const double *params, int64_t params_len_, AtenTensorHandle *output) {
  AOTI_TORCH_CONVERT_EXCEPTION_TO_ERROR_CODE({
    namespace ai = torch::aot_inductor;
    auto result = xinfer_b200::qwen3_decode_step(
        ai::resolve_tensor_dispatch_flags(input_ids), ai::resolve_tensor_dispatch_flags(cache_position),
        ai::resolve_tensor_list_dispatch_flags(state, state_len_),
        ai::resolve_tensor_dispatch_flags(kv_lengths), ai::resolve_tensor_dispatch_flags(query_lengths),
        ai::resolve_tensor_list_dispatch_flags(weights, weights_len_),
        at::IntArrayRef(geometry, (size_t)geometry_len_), at::ArrayRef<double>(params, (size_t)params_len_));
    *output = ai::new_tensor_handle(std::move(result));
  });
}

// The attention operators' shims, with the reference's signatures
// (compiler/common/attention.py:10-16).
extern "C" AOTI_TORCH_EXPORT AOTITorchError aoti_torch_cuda_batched_flash_attention(
    AtenTensorHandle q, AtenTensorHandle k, AtenTensorHandle v, AtenTensorHandle offsets,
    AtenTensorHandle cuda_offsets, AtenTensorHandle blocks, double scale, AtenTensorHandle *output) {
  AOTI_TORCH_CONVERT_EXCEPTION_TO_ERROR_CODE({
    namespace ai = torch::aot_inductor;
    auto result = xinfer_b200::batched_flash_attention(
        ai::resolve_tensor_dispatch_flags(q), ai::resolve_tensor_dispatch_flags(k),
        ai::resolve_tensor_dispatch_flags(v), ai::resolve_tensor_dispatch_flags(offsets),
        ai::resolve_tensor_dispatch_flags(cuda_offsets), ai::resolve_tensor_dispatch_flags(blocks), scale);
    *output = ai::new_tensor_handle(std::move(result));
  });
}

extern "C" AOTI_TORCH_EXPORT AOTITorchError aoti_torch_cuda_flash_attention(
    AtenTensorHandle q, AtenTensorHandle k, AtenTensorHandle v, AtenTensorHandle extent, double scale,
    AtenTensorHandle *output) {
  AOTI_TORCH_CONVERT_EXCEPTION_TO_ERROR_CODE({
    namespace ai = torch::aot_inductor;
    auto result = xinfer_b200::flash_attention(
        ai::resolve_tensor_dispatch_flags(q), ai::resolve_tensor_dispatch_flags(k),
        ai::resolve_tensor_dispatch_flags(v), ai::resolve_tensor_dispatch_flags(extent), scale);
    *output = ai::new_tensor_handle(std::move(result));
  });
}
