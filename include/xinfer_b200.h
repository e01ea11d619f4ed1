/*
 * xinfer_b200 — C ABI of the B200 (sm_100a) decode step for the Qwen3 and Qwen3.5 families.
 *
 * Plain C: device pointers, sizes and an opaque stream; no torch types. Every entry point
 * returns 0 on success and a nonzero XB_ERR_* code on failure; xb_last_error() gives the
 * message of the calling thread's most recent failure.
 *
 * The entry points replace the following reference interfaces (paths inside tqxia/xinfer):
 *   xb_decode_step          compiler/qwen35/model.py:162-183 (ModelStep.forward, T == 1) and
 *                           compiler/qwen3/model.py:70-95, as run from decode.pt2 by
 *                           runtime/common/runner.h:30-78 (Runner::step_batch / run_inputs).
 *                           Also fuses the argmax of runtime/common/generation.h:39.
 *
 * Memory layout of every tensor is the reference's (contiguous, row-major):
 *   KV cache       bf16 [rows, kv_heads, capacity, head_dim]     updated in place
 *   conv state     bf16 [rows, conv_channels, conv_width]        replaced (read in, write out)
 *   recurrent      fp32 [rows, value_heads, key_dim, value_dim]  replaced (read in, write out)
 *   logits         bf16 [B, vocab]
 */
#ifndef XINFER_B200_H
#define XINFER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XB_ABI_VERSION 1

#define XB_MAX_LAYERS 64
#define XB_MAX_BATCH 8

enum {
  XB_OK = 0,
  XB_ERR_INVALID = 1,   /* bad argument, geometry or size */
  XB_ERR_CUDA = 2,      /* a CUDA runtime call failed */
  XB_ERR_DEVICE = 3,    /* the kernel reported a device-side error (bounded wait expired) */
  XB_ERR_UNSUPPORTED = 4
};

enum { XB_FAMILY_QWEN3 = 1, XB_FAMILY_QWEN35 = 2 };
enum { XB_LAYER_ATTENTION = 0, XB_LAYER_DELTANET = 1 };

/* Model geometry. Field meaning follows the HF configs that the reference loads
 * (compiler/qwen3/model.py:16-26, compiler/qwen35/model.py:21-42). */
typedef struct XbGeometry {
  int32_t family;            /* XB_FAMILY_* */
  int32_t num_layers;
  int32_t hidden;
  int32_t intermediate;
  int32_t vocab;
  int32_t num_q_heads;       /* full-attention layers */
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t rotary_dim;        /* head_dim for Qwen3; head_dim * partial_rotary_factor for Qwen3.5 */
  int32_t lin_key_heads;     /* DeltaNet layers (Qwen3.5 only) */
  int32_t lin_value_heads;
  int32_t lin_head_dim;      /* key dim == value dim == 128 */
  int32_t conv_width;        /* 4 */
  int32_t capacity;          /* KV slots per row */
  int32_t state_rows;        /* allocated rows of every state tensor (8 in the reference) */
  float rms_eps;
  float rope_theta;
  const float *rope_inv_freq;        /* host, rotary_dim/2 values, or NULL: xb_rope_inv_freq() */
  int32_t layer_kind[XB_MAX_LAYERS]; /* XB_LAYER_* */
} XbGeometry;

/* Per-layer device pointers to bf16 weights in the HF layout ([out, in] for linears). */
typedef struct XbLayerWeights {
  const void *input_norm, *post_norm;
  /* full attention */
  const void *q_proj, *k_proj, *v_proj, *o_proj, *q_norm, *k_norm;
  /* Gated DeltaNet (the reference's packed in_proj 8224 rows may be passed as four views) */
  const void *in_qkv, *in_z, *in_b, *in_a, *conv_w, *a_log, *dt_bias, *gnorm, *out_proj;
  /* SwiGLU MLP */
  const void *gate, *up, *down;
} XbLayerWeights;

typedef struct XbModelWeights {
  const void *embed;       /* [vocab, hidden] */
  const void *final_norm;  /* [hidden] */
  const void *lm_head;     /* [vocab, hidden]; == embed when tied */
  XbLayerWeights layers[XB_MAX_LAYERS];
} XbModelWeights;

/* Per-layer state pointers for one step. Attention layers use k_cache / v_cache; DeltaNet
 * layers use conv_in / rec_in (read) and conv_out / rec_out (written). An output either is a
 * distinct buffer (the reference's "replace" contract: inputs stay unmodified) or equals its
 * input pointer exactly (update in place); partial overlap is invalid. Pointers address row 0;
 * rows [0, B) are read and written, rows >= B are never touched. */
typedef struct XbLayerState {
  void *k_cache, *v_cache;
  const void *conv_in, *rec_in;
  void *conv_out, *rec_out;
} XbLayerState;

typedef struct XbStepArgs {
  int32_t batch;                      /* B, 1..8 */
  const int64_t *input_ids;           /* device [B], or NULL to pass host_ids by value */
  const int64_t *cache_position;      /* device [B], or NULL to pass host_positions by value */
  int64_t host_ids[XB_MAX_BATCH];     /* used when input_ids == NULL (launch parameters, no copy) */
  int64_t host_positions[XB_MAX_BATCH];
  int32_t kv_lengths[XB_MAX_BATCH];   /* host values: populated length after this call */
  int32_t query_lengths[XB_MAX_BATCH];/* host values: 0 (empty row) or 1 */
  XbLayerState layers[XB_MAX_LAYERS];
  void *logits;                       /* device bf16 [B, vocab] */
  int64_t *next_tokens;               /* device int64 [B] or NULL: argmax of each logits row */
} XbStepArgs;

typedef struct XbModel XbModel;

/* Build a device-side plan for one model: validates geometry, uploads the pointer table and
 * the RoPE inverse frequencies (computed exactly as the HF rotary embedding does). */
int xb_model_create(const XbGeometry *geometry, const XbModelWeights *weights, XbModel **model);
int xb_model_destroy(XbModel *model);

/* Bytes of device scratch one xb_decode_step of up to max_batch rows needs. */
int xb_decode_workspace_bytes(const XbModel *model, int32_t max_batch, size_t *bytes);

/* One decode step (T == 1) of B rows, one persistent kernel launch on `stream`.
 * `workspace` must be zeroed once before first use (xb_workspace_init) and not shared by
 * steps that overlap on the GPU. */
int xb_workspace_init(void *workspace, size_t workspace_bytes, void *stream);
int xb_decode_step(const XbModel *model, const XbStepArgs *args, void *workspace,
                   size_t workspace_bytes, void *stream);

/* Synchronises `stream` and returns XB_ERR_DEVICE if a kernel using `workspace` reported a
 * device-side error since the last call (and clears it). */
int xb_workspace_check(void *workspace, void *stream, int32_t *device_error);

/* Allocation-free decode step. No counterpart in the reference: this entry point exists for
 * callers that cannot allocate device memory when they step the model (a serving runtime that
 * reserved HBM for its own pool at start-up, a host with a fixed memory plan that forbids
 * allocations after initialisation). It takes the geometry and weight pointers directly (no
 * XbModel, whose creation allocates) and no workspace: the weight table, RoPE table and the
 * kernel's scratch live in one static device array of XB_STATIC_SCRATCH_BYTES, held by every
 * GPU that loads this library until the process exits. Steps whose scratch would not fit
 * (large batch or many heads) fail with XB_ERR_INVALID and a message; use xb_decode_step.
 * It calls no cudaMalloc / cudaFree. The first call on each device does a one-time set-up
 * (a symbol address lookup, no allocation); make that first call before any stream capture.
 * All calls on a device share the array, which keeps the previous call's contents: each call
 * rewrites the tables and clears the control words, so calls that overlap on the GPU (other
 * streams, other threads) race and must be serialised by the caller. If device_error is not
 * NULL the call synchronises the stream and reports the kernel's device-side error word.
 * Weight pointers follow xb_model_create's rules. */
#define XB_STATIC_SCRATCH_BYTES (4u << 20)
int xb_decode_step_static(const XbGeometry *geometry, const XbModelWeights *weights,
                          const XbStepArgs *args, void *stream, int32_t *device_error);

/* Prefix attention of up to 512 queries per row over a KV cache: the computation behind the
 * reference's xinfer::flash_attention and xinfer::batched_flash_attention operators
 * (compiler/common/kernels/attention.cpp:14-79 batched, :82-124 single extent), which call ATen's
 * FlashAttention-2 there. Query t < count_b of row b sits at position length_b - count_b + t and
 * attends to KV slots 0..length_b - count_b + t (lower-right causal); query head h reads KV head
 * h / (q_heads / kv_heads); queries t >= count_b get zeros. bf16 tensors with unit feature stride:
 *   q   [batch, q_heads, q_tokens, head_dim]   strides[0..2] = batch, head, token strides
 *   k,v [batch, kv_heads, capacity, head_dim]  strides[3..5] (k) and [6..8] (v)
 *   out [batch, q_heads, q_tokens, head_dim]   contiguous, fully written
 * Per-row extents come from cu_offsets (device int32 [2, batch + 1]: cumulative query counts, then
 * cumulative KV lengths, as batched_attention_metadata builds them, compiler/common/attention.py
 * :27-40) or, when cu_offsets is NULL, are the same (count, length) for every row. Strides must be
 * multiples of 8 elements and tensors 16-byte aligned. `blocks` is the one-block-per-row page
 * table of the batched operator (attention.cpp:58-63). Errors: XB_ERR_INVALID with the
 * reference's messages ("Query heads must be a positive multiple of KV heads", "Flash head
 * dimension must be a multiple of 8 in 8..256", "Invalid valid-prefix length"). */
typedef struct XbAttentionArgs {
  const void *q, *k, *v;
  void *out;
  long long strides[9];
  int32_t batch, q_heads, kv_heads, head_dim, q_tokens, capacity;
  const int32_t *cu_offsets;
  int32_t count, length;
  float scale;
  const int32_t *blocks;     /* device int32: row b reads cache row blocks[b * blocks_stride], or NULL: b */
  long long blocks_stride;
} XbAttentionArgs;
int xb_prefix_attention(const XbAttentionArgs *args, void *stream);

/* Prefill of one row: ModelStep.forward with T > 1 tokens (compiler/qwen35/model.py:162-183,
 * compiler/qwen3/model.py:70-95, exported as prefill.pt2 by compiler/qwen35/export.py:43-57, run by
 * runtime/common/runner.h:30-78 for prompts). T tokens (1..512) at cache positions
 * start_position .. start_position + T - 1 of state row 0: K/V appended in place, the DeltaNet
 * conv window and recurrent state read from *_in and written to *_out (equal pointers update in
 * place), the logits of the last token written to `logits` (bf16 [vocab]) and its argmax to
 * `next_token` (or skipped when NULL). The projections run on the tensor cores (xb_gemm_bf16);
 * the DeltaNet recurrence is scanned over the tokens. The workspace (xb_prefill_workspace_bytes)
 * starts with the decode workspace's control words: token ids out of range are reported by
 * xb_workspace_check. Calls that overlap on the GPU must not share a workspace. */
typedef struct XbPrefillArgs {
  int32_t tokens;
  const int64_t *input_ids;           /* device int64 [T] */
  int64_t start_position;
  XbLayerState layers[XB_MAX_LAYERS]; /* row 0 of every state tensor */
  void *logits;                       /* device bf16 [vocab] */
  int64_t *next_token;                /* device int64 [1], or NULL */
} XbPrefillArgs;
int xb_prefill_workspace_bytes(const XbModel *model, int32_t max_tokens, size_t *bytes);
int xb_prefill_step(const XbModel *model, const XbPrefillArgs *args, void *workspace,
                    size_t workspace_bytes, void *stream);

/* out[m, n] = x[m, k] . w[n, k]^T in bf16 with fp32 accumulation and one rounding: the bf16
 * nn.Linear of the reference's prefill graph (cuBLAS through Inductor there), on the sm_100a
 * tensor cores. n and k multiples of 8, all pointers 16-byte aligned, row-major and packed. */
int xb_gemm_bf16(int32_t m, int32_t n, int32_t k, const void *x, const void *w, void *out, void *stream);

/* Host-only helper: the HF default RoPE inverse frequencies 1 / theta^(2i / rotary_dim) in fp32
 * (transformers Qwen3_5TextRotaryEmbedding.compute_default_rope_parameters, as loaded by
 * compiler/qwen35/model.py:41 and compiler/qwen3/model.py:16-26). */
int xb_rope_inv_freq(float theta, int32_t rotary_dim, float *out);

/* Stage trace for performance work (the reference has no in-process tracer; it profiles with
 * external tools). While a device buffer is set, every xb_decode_step launch writes, per CTA,
 * (3 * 512 + 8) u64 words: %globaltimer at each stage's barrier arrival, release and end of
 * prologue, then the kernel end time, the consumers' total ring-slot wait, the stage count, the
 * producer's busy time, its total wait for free slots and the number of tiles it issued. Pass NULL to switch tracing off. The buffer must hold 1024 CTAs' worth. */
int xb_debug_trace(void *device_buffer, size_t bytes);

/* Fault injection for tests of the bounded waits (the reference's failure handling is the
 * runner's exception path, runtime/common/runner.h, with no device-side counterpart). For the
 * launches that follow on the current device: CTA 0 does not publish the outputs of GEMV stage
 * `withhold_stage` (index in the step's stage order; negative: none), and every wait gives up
 * after `wait_limit_ns` (0: the default 2 s; at least 1 ms). A withheld stage makes the stages
 * that read it time out: the launch ends, every CTA returns, and xb_workspace_check reports
 * XB_ERR_DEVICE with DERR_WAIT (1). xb_debug_fault(-1, 0) restores normal operation. Not for
 * use while other launches of this library run. */
int xb_debug_fault(int32_t withhold_stage, uint64_t wait_limit_ns);

const char *xb_last_error(void);
int xb_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* XINFER_B200_H */
