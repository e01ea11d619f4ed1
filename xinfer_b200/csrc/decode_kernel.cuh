// Persistent sm_100a decode megakernel for the Qwen3 / Qwen3.5 decode step (T == 1, B <= 8).
//
// One cooperative launch per step, one CTA per SM. Each CTA runs two roles:
//   * a producer warp that streams this CTA's share of every weight matrix of the step, in
//     consumption order, through a ring of 32 KB shared-memory slots with 1-D bulk copies (TMA,
//     cp.async.bulk, completion on mbarriers). Weights do not depend on activations, so the
//     producer runs ahead across stage boundaries and keeps HBM busy while the consumers wait
//     for the previous stage's outputs;
//   * eight consumer warps that run the stages of the layer loop:
//       DeltaNet layer : in_proj GEMV -> conv/delta-rule -> gated norm + out_proj -> gate/up -> down
//       attention layer: q/k/v GEMV -> norm/RoPE/KV append/split-KV partials -> combine
//                        -> o_proj -> gate/up -> down
//       final          : final norm + lm_head GEMV with fused argmax.
//     Stages hand values on through tagged words (value and a per-launch tag in one word), which
//     consumers poll with bounded spins; there is no grid barrier. RMSNorms are recomputed by
//     every CTA from the residual stream in its stage prologue; SiLU*mul and residual adds are
//     fused into GEMV epilogues.
// This file is compiled twice: with XB_TENSOR_TILES 0 (batch rows 1 and 2, FMA GEMV tiles) and
// with XB_TENSOR_TILES 1 (batch rows 4 and 8, tensor-core GEMV tiles), so that each kernel's code
// contains only its own tile path.
// Rounding points follow the reference step (bf16 tensors between ops, fp32 inside each op):
//   compiler/qwen35/model.py:162-183, compiler/qwen35/adapters/{attention.py:39-63,delta.py:32-49},
//   compiler/qwen35/kernels/recurrent.py:20-124, compiler/qwen3/model.py:70-95,
//   compiler/qwen3/adapters/attention.py:41-62, compiler/common/kernels/kv_cache.py:8-42,
//   compiler/common/kernels/attention.cpp:14-79.

#pragma once
#ifndef XB_TENSOR_TILES
#define XB_TENSOR_TILES 0
#endif

#include "xb_device.cuh"
#include "xinfer_b200.h"

#include <cuda.h>
#include <cstdio>
#include <cstring>
#include <cmath>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

namespace xb {

constexpr int kWarps = 8;                 // consumer warps
constexpr int kCT = kWarps * 32;          // consumer threads
constexpr int kThreads = kCT + 32;        // + producer warp
constexpr int kSlot = 32768;              // ring slot bytes
constexpr int kMaxSlots = 8;
constexpr int kHdrBytes = 512;
constexpr int kResRows = 32;                           // residual rows a CTA owns (<= 32)
constexpr int kResBytes = XB_MAX_BATCH * kResRows * 4;
constexpr int kRedFloats = 1024;
// Long-context kernels (AG > 0) run the attention items in position blocks when an item spans at
// least this many positions (the host picks the kernel per launch).
#ifndef XB_ATT_BLOCK_MIN
#define XB_ATT_BLOCK_MIN 128
#endif
constexpr int kAttBlockMin = XB_ATT_BLOCK_MIN;
// RoPE cos/sin of every row's position (bf16 pair per frequency), computed once per launch:
// the positions are the same for every attention layer of the step.
constexpr int kRopeFreqs = 64;  // rotary_dim / 2 <= 64
constexpr int kRopeBytes = XB_MAX_BATCH * kRopeFreqs * 4;
constexpr int kUOffset = kHdrBytes + kResBytes + kRedFloats * 4 + kRopeBytes;  // 7680, 128-aligned
constexpr int kSmemLimit = 232448;                     // 227 KB opt-in per CTA
// layout of the per-CTA float scratch `red` during GEMV stages
constexpr int RED_PART = 512;   // [2][kWarps][2][NB][2] split-K partials (batch 1 tiles)

// control words in the workspace (each on its own 128-byte line)
// Words [0, CTL_WORDS) are cleared whenever a workspace is reset; the launch epoch (which
// stamps every inter-stage value with a tag) and the epoch of the last clear of the tagged
// buffers live after them.
enum {
  CTL_SCRUB_BAR = 32, CTL_ERR = 64, CTL_DONE = 96, CTL_WORDS = 128, CTL_EPOCH = 128,
  CTL_SCRUBBED = 160, CTL_TOTAL = 192
};
// device error codes
enum { DERR_WAIT = 1, DERR_RING_FULL = 2, DERR_RING_EMPTY = 3, DERR_TOKEN = 4, DERR_DRAIN = 5 };

// Fault injection for tests of the bounded waits (xb_debug_fault): the wait limit, and a stage
// (index in the step's stage order) whose outputs CTA 0 does not publish. Defaults: 2 s, none.
static __constant__ unsigned long long c_wait_limit_ns = kWaitLimitNs;
static __constant__ int c_withhold_stage = -1;

enum Stage {
  ST_IN_DELTA = 0, ST_OUT_DELTA, ST_QKV, ST_O, ST_GATEUP, ST_DOWN, ST_LMHEAD
};
enum Epi { EPI_STORE = 0, EPI_RESID, EPI_GATEUP, EPI_LOGITS };

struct StepParams {
  int family, L, H, I, V, HQ, HKV, D, RD, HK, HV, DK, CW, C, rows_alloc;
  float eps, dk_scale, att_scale;
  int pstride, splits, ncta, nslots, ubytes, B;
  int kv_len[XB_MAX_BATCH], q_len[XB_MAX_BATCH];
  unsigned long long delta_mask;
  const XbLayerWeights *layers;
  const bf16 *embed, *final_norm, *lm_head;
  const float *inv_freq;
  const int64_t *ids, *pos;  // device arrays, or NULL: use hid / hpos
  long long hid[XB_MAX_BATCH], hpos[XB_MAX_BATCH];
  void *sa[XB_MAX_LAYERS], *sb[XB_MAX_LAYERS], *sc[XB_MAX_LAYERS], *sd[XB_MAX_LAYERS];
  bf16 *logits;
  int64_t *tokens;
  unsigned *ctrl;
  // inter-stage buffers of tagged words: (bf16 bits | tag << 16) or {fp32 bits, tag}
  unsigned *h, *proj, *core, *att_out, *act;
  u64 *ssq, *att_o, *att_ml;  // {fp32, tag} words; att_ml holds (M, L) pairs
  // the tagged buffers as one range [scrub_base, scrub_base + 16 * scrub_chunks), cleared by
  // the launches that start kScrubInterval or more epochs after the previous clear
  uint4 *scrub_base;
  unsigned scrub_chunks;
  float *am_v;
  int *am_i;
  // Optional stage trace (see xb_debug_trace): per CTA kTraceStages x {arrive, release} stamps
  // of %globaltimer plus ring-wait totals; NULL when tracing is off.
  unsigned long long *trace;
};
constexpr int kTraceStages = 512;
constexpr int kTraceStride = 3 * kTraceStages + 8;  // u64 words per CTA

struct SmemHdr {
  uint64_t full[kMaxSlots];
  uint64_t empty[kMaxSlots];
  long long ids[XB_MAX_BATCH];
  long long pos[XB_MAX_BATCH];
  int abort;
  int is_last;
  int scrub;  // this launch clears the tagged buffers before any stage runs
  unsigned epoch;
};
static_assert(sizeof(SmemHdr) <= kHdrBytes, "header");

// One GEMV stage: logical rows [0, N) over up to four row segments (concatenated), or a
// gate/up pair (paired: logical row i is row i of seg[0] and row i of seg[1]).
struct Gemv {
  const bf16 *seg[4];
  int seg_rows[4];
  int nseg;
  int K, N;
  bool paired;
  int stage;
};

__device__ __forceinline__ long long token_id(const StepParams &p, int b) {
  return p.ids ? (long long)p.ids[b] : p.hid[b];
}
__device__ __forceinline__ long long position(const StepParams &p, int b) {
  return p.pos ? (long long)p.pos[b] : p.hpos[b];
}

__device__ __forceinline__ bool is_delta(const StepParams &p, int l) {
  return (p.delta_mask >> l) & 1ull;
}
// Stage [src, src + bytes) from global memory into L2 (16-byte aligned, multiple of 16 bytes).
__device__ __forceinline__ void prefetch_l2(const void *src, size_t bytes) {
  for (size_t o = 0; o < bytes; o += 65536)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"((const char *)src + o),
                 "r"((unsigned)(bytes - o < 65536 ? bytes - o : 65536))
                 : "memory");
}

__device__ __forceinline__ Gemv make_gemv(const StepParams &p, int l, int stage) {
  Gemv g;
  g.nseg = 1;
  g.paired = false;
  g.stage = stage;
  for (int i = 0; i < 4; ++i) { g.seg[i] = nullptr; g.seg_rows[i] = 0; }
  if (stage == ST_LMHEAD) {
    g.seg[0] = p.lm_head; g.seg_rows[0] = p.V; g.K = p.H; g.N = p.V;
    return g;
  }
  const XbLayerWeights &w = p.layers[l];
  switch (stage) {
  case ST_IN_DELTA: {
    const int key = p.HK * p.DK, val = p.HV * p.DK;
    g.nseg = 4;
    g.seg[0] = (const bf16 *)w.in_qkv; g.seg_rows[0] = 2 * key + val;
    g.seg[1] = (const bf16 *)w.in_z;   g.seg_rows[1] = val;
    g.seg[2] = (const bf16 *)w.in_b;   g.seg_rows[2] = p.HV;
    g.seg[3] = (const bf16 *)w.in_a;   g.seg_rows[3] = p.HV;
    g.K = p.H;
    break;
  }
  case ST_OUT_DELTA:
    g.seg[0] = (const bf16 *)w.out_proj; g.seg_rows[0] = p.H; g.K = p.HV * p.DK;
    break;
  case ST_QKV: {
    const int qrows = p.HQ * p.D * (p.family == XB_FAMILY_QWEN35 ? 2 : 1);
    g.nseg = 3;
    g.seg[0] = (const bf16 *)w.q_proj; g.seg_rows[0] = qrows;
    g.seg[1] = (const bf16 *)w.k_proj; g.seg_rows[1] = p.HKV * p.D;
    g.seg[2] = (const bf16 *)w.v_proj; g.seg_rows[2] = p.HKV * p.D;
    g.K = p.H;
    break;
  }
  case ST_O:
    g.seg[0] = (const bf16 *)w.o_proj; g.seg_rows[0] = p.H; g.K = p.HQ * p.D;
    break;
  case ST_GATEUP:
    g.nseg = 2; g.paired = true;
    g.seg[0] = (const bf16 *)w.gate; g.seg_rows[0] = p.I;
    g.seg[1] = (const bf16 *)w.up;   g.seg_rows[1] = p.I;
    g.K = p.H;
    g.N = p.I;
    return g;
  case ST_DOWN:
    g.seg[0] = (const bf16 *)w.down; g.seg_rows[0] = p.H; g.K = p.I;
    break;
  }
  g.N = 0;
  for (int i = 0; i < g.nseg; ++i) g.N += g.seg_rows[i];
  return g;
}

__device__ __forceinline__ int tile_rows(const Gemv &g) {
  return kSlot / (g.K * 2 * (g.paired ? 2 : 1));
}
#if XB_TENSOR_TILES
// Rows of a padded ring tile (batch >= 4, tensor-core tiles of 16 rows): every row occupies
// K * 2 + 16 bytes so that the 8 rows one MMA fragment reads fall in different banks.
__device__ __forceinline__ int tile_rows_padded(const Gemv &g) {
  const int r = kSlot / ((g.K * 2 + 16) * (g.paired ? 2 : 1));
  return min(r, g.paired ? 8 : 16);
}
#endif
__device__ __forceinline__ void cta_range(int N, int cta, int ncta, int &lo, int &hi) {
  lo = (int)(((long long)N * cta) / ncta);
  hi = (int)(((long long)N * (cta + 1)) / ncta);
}

// ------------------------------------------------------------------------------------------
// Producer role: lane 0 of the last warp issues every weight tile of this CTA, in order.
// ------------------------------------------------------------------------------------------
struct Producer {
  const StepParams &p;
  SmemHdr *hdr;
  char *ring;
  uint64_t policy;
  int slot = 0;
  unsigned phase = 0;
  int issued = 0;
  bool stop = false;
  unsigned long long empty_wait = 0;  // ns waiting for free slots (trace)

  __device__ Producer(const StepParams &p_, SmemHdr *h, char *r) : p(p_), hdr(h), ring(r) {
    policy = policy_evict_first();
  }

  __device__ bool acquire() {
    // Wait until the consumers released this slot AND the previous copy into it has landed
    // (the second condition only matters after an abort, when consumers release unread slots).
    uint64_t t0 = 0;
    unsigned spins = 0;
    const uint64_t tw = p.trace ? globaltimer() : 0;
    struct Acc {
      const StepParams &p; unsigned long long &acc; uint64_t tw;
      __device__ ~Acc() { if (p.trace) acc += globaltimer() - tw; }
    } acc_guard{p, empty_wait, tw};
    while (!mbar_try_wait(&hdr->empty[slot], phase ^ 1u) ||
           (issued >= p.nslots && !mbar_try_wait(&hdr->full[slot], phase ^ 1u))) {
      if ((++spins & 63u) == 0) {
        const uint64_t t = globaltimer();
        if (t0 == 0) t0 = t;
        else if (t - t0 > kSlowWaitNs) {
          if (ld_volatile(p.ctrl + CTL_ERR)) return false;
          if (t - t0 > 2 * c_wait_limit_ns) {
            atomicCAS(p.ctrl + CTL_ERR, 0u, (unsigned)DERR_RING_EMPTY);
            return false;
          }
        }
      }
    }
    return true;
  }

  __device__ void gemv(int l, int stage) {
    if (stop) return;
    const Gemv g = make_gemv(p, l, stage);
    int lo, hi;
    cta_range(g.N, blockIdx.x, p.ncta, lo, hi);
#if XB_TENSOR_TILES
    const int R = tile_rows_padded(g);
#else
    const int R = tile_rows(g);
#endif
    const unsigned rowb = (unsigned)g.K * 2u;
    for (int r0 = lo; r0 < hi; r0 += R) {
      const int n = min(R, hi - r0);
      if (!acquire()) { stop = true; return; }
      char *dst = ring + (size_t)slot * kSlot;
      uint64_t *bar = &hdr->full[slot];
#if XB_TENSOR_TILES
      {
        // one copy per row into a padded row slot: gate/up tiles hold n gate rows, then n up rows
        const unsigned pitch = rowb + 16u;
        mbar_arrive_expect_tx(bar, (unsigned)n * rowb * (g.paired ? 2u : 1u));
        if (g.paired) {
          for (int r = 0; r < n; ++r) {
            bulk_g2s(dst + (size_t)r * pitch, g.seg[0] + (size_t)(r0 + r) * g.K, rowb, bar, policy);
            bulk_g2s(dst + (size_t)(n + r) * pitch, g.seg[1] + (size_t)(r0 + r) * g.K, rowb, bar, policy);
          }
        } else {
          int sg = 0, base = 0;
          for (int r = 0; r < n; ++r) {
            while (sg + 1 < g.nseg && r0 + r >= base + g.seg_rows[sg]) base += g.seg_rows[sg++];
            bulk_g2s(dst + (size_t)r * pitch, g.seg[sg] + (size_t)(r0 + r - base) * g.K, rowb, bar, policy);
          }
        }
      }
#else
      if (g.paired) {
        const unsigned bytes = (unsigned)n * rowb;
        mbar_arrive_expect_tx(bar, 2u * bytes);
        bulk_g2s(dst, g.seg[0] + (size_t)r0 * g.K, bytes, bar, policy);
        bulk_g2s(dst + bytes, g.seg[1] + (size_t)r0 * g.K, bytes, bar, policy);
      } else {
        mbar_arrive_expect_tx(bar, (unsigned)n * rowb);
        int base = 0;
        for (int s = 0; s < g.nseg; ++s) {
          const int a = max(r0, base), b = min(r0 + n, base + g.seg_rows[s]);
          if (a < b)
            bulk_g2s(dst + (size_t)(a - r0) * rowb, g.seg[s] + (size_t)(a - base) * g.K,
                     (unsigned)(b - a) * rowb, bar, policy);
          base += g.seg_rows[s];
        }
      }
#endif
      ++issued;
      if (++slot == p.nslots) { slot = 0; phase ^= 1u; }
    }
  }
  __device__ void delta(int) {}
  __device__ void attn(int) {}
  __device__ void comb(int) {}
};


// One warp's share of a GEMV tile: rows A and B (and, for gate/up tiles, their up rows) dotted
// with the NB activation rows over K chunks [cb, ce), reduced over the warp. Returns, for lane
// b (< NB) the row-A result of batch row b and for lane 16 + b the row-B result (.y = up row).
// Kept out of line so that its code is generated independently of the surrounding megakernel.
template <bool PAIRED, int NB>
__device__ __forceinline__ float2 gemv_pair(const uint4 *__restrict__ wA, const uint4 *__restrict__ wB,
                                         const uint4 *__restrict__ uA, const uint4 *__restrict__ uB,
                                         const uint4 *__restrict__ act4, int n8, int cb, int ce) {
  const int lane = threadIdx.x & 31;
  float a0[NB], c0[NB], a1[NB], c1[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) { a0[b] = c0[b] = a1[b] = c1[b] = 0.f; }
  if (PAIRED) {
#pragma unroll 2
    for (int j = cb + lane; j < ce; j += 32) {
      const uint4 wa = wA[j], wb = wB[j], ua = uA[j], ub = uB[j];
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const uint4 x = act4[b * n8 + j];
        a0[b] = dot8_bf16(wa, x, a0[b]);
        c0[b] = dot8_bf16(wb, x, c0[b]);
        a1[b] = dot8_bf16(ua, x, a1[b]);
        c1[b] = dot8_bf16(ub, x, c1[b]);
      }
    }
  } else {
#pragma unroll 4
    for (int j = cb + lane; j < ce; j += 32) {
      const uint4 wa = wA[j], wb = wB[j];
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const uint4 x = act4[b * n8 + j];
        a0[b] = dot8_bf16(wa, x, a0[b]);
        c0[b] = dot8_bf16(wb, x, c0[b]);
      }
    }
  }
  const int bsel = lane & 15;
  const bool second = lane >= 16;
  float2 r = make_float2(0.f, 0.f);
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const float sa = warp_sum(a0[b]), sc = warp_sum(c0[b]);
    float ta = 0.f, tc = 0.f;
    if (PAIRED) { ta = warp_sum(a1[b]); tc = warp_sum(c1[b]); }
    if (bsel == b) r = second ? make_float2(sc, tc) : make_float2(sa, ta);
  }
  return r;
}


#if XB_TENSOR_TILES
// D += A (16 x 16, row-major) * B (16 x 8, column-major), bf16 inputs, fp32 accumulation.
__device__ __forceinline__ void mma_16816(float (&d)[4], unsigned a0, unsigned a1, unsigned a2,
                                          unsigned a3, unsigned b0, unsigned b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
#endif

#ifndef XB_POLL_NS
#define XB_POLL_NS 0
#endif
// Pause between two polls of a word that was not ready yet (0: poll back to back).
__device__ __forceinline__ void poll_pause() {
  if (XB_POLL_NS) __nanosleep(XB_POLL_NS);
}

// ---- waits (free functions: the consumer object must never have its address taken, so that
// its state stays in registers) -------------------------------------------------------------
// True when a wait must end: this CTA aborted, or (only after kSlowWaitNs of waiting, so that the
// hot hand-offs never pay for a global load) the grid reported an error or the limit passed.
__device__ __forceinline__ bool wait_give_up(volatile int *abort_flag, unsigned *ctrl, uint64_t &t0) {
  if (*abort_flag) return true;
  const uint64_t t = globaltimer();
  if (t0 == 0) { t0 = t; return false; }
  if (t - t0 < kSlowWaitNs) return false;
  if (ld_volatile(ctrl + CTL_ERR)) { *abort_flag = 1; return true; }
  if (t - t0 > c_wait_limit_ns) {
    atomicCAS(ctrl + CTL_ERR, 0u, (unsigned)DERR_WAIT);
    *abort_flag = 1;
    return true;
  }
  return false;
}
static __device__ __noinline__ uint4 repoll4(const unsigned *w, unsigned tg, volatile int *abort_flag,
                                      unsigned *ctrl) {
  uint4 v;
  uint64_t t0 = 0;
  for (unsigned spins = 1;; ++spins) {
    poll_pause();
    v = ld_poll_u4(w);
    if (tag4_ok(v, tg)) break;
    if ((spins & 15u) == 0 && wait_give_up(abort_flag, ctrl, t0)) break;
  }
  return v;
}
static __device__ __noinline__ unsigned repoll1(const unsigned *w, unsigned tg, volatile int *abort_flag,
                                         unsigned *ctrl) {
  unsigned v;
  uint64_t t0 = 0;
  for (unsigned spins = 1;; ++spins) {
    poll_pause();
    v = ld_poll_u32(w);
    if ((v >> 16) == tg) break;
    if ((spins & 15u) == 0 && wait_give_up(abort_flag, ctrl, t0)) break;
  }
  return v;
}
static __device__ __noinline__ ulonglong2 repoll2f(const u64 *w, unsigned tg, volatile int *abort_flag,
                                             unsigned *ctrl) {
  ulonglong2 v;
  uint64_t t0 = 0;
  for (unsigned spins = 1;; ++spins) {
    poll_pause();
    v = ld_poll_u64x2(w);
    if (ftag_tag(v.x) == tg && ftag_tag(v.y) == tg) break;
    if ((spins & 15u) == 0 && wait_give_up(abort_flag, ctrl, t0)) break;
  }
  return v;
}
static __device__ __noinline__ float repoll1f(const u64 *w, unsigned tg, volatile int *abort_flag,
                                       unsigned *ctrl) {
  u64 v;
  uint64_t t0 = 0;
  for (unsigned spins = 1;; ++spins) {
    poll_pause();
    v = ld_poll_u64(w);
    if (ftag_tag(v) == tg) break;
    if ((spins & 15u) == 0 && wait_give_up(abort_flag, ctrl, t0)) break;
  }
  return ftag_val(v);
}

// ------------------------------------------------------------------------------------------
// Consumer role
// ------------------------------------------------------------------------------------------
template <int NB, int AG = 0, int AE = 0, int LK = 0> struct Consumer {
#if XB_TENSOR_TILES
  static constexpr int kPad = 1;  // padded activation rows (tensor-core tiles)
#else
  static constexpr int kPad = 0;
#endif
  const StepParams &p;
  SmemHdr *hdr;
  float *red;     // kRedFloats scratch, reused stage by stage
  unsigned *rope; // [XB_MAX_BATCH][kRopeFreqs] bf16 (cos | sin << 16) of each row's position
  float *hres;    // [NB][kResRows] this CTA's rows of the residual stream, kept across stages
  char *U;        // union region: GEMV activations / attention scratch
  char *ring;
  int tid, warp, lane;
  int slot = 0;
  unsigned phase = 0;
  bool h_ready = false;   // residual stream published (false: still the embedding rows)
  int sidx = 0;           // stage counter (trace)
  bool withhold = false;  // fault injection (xb_debug_fault)
  unsigned epoch;
  unsigned long long full_wait = 0;  // ns waiting for ring slots (trace, tid 0)
  unsigned long long poll_wait = 0;  // ns waiting for tagged inputs (trace, tid 0)
  // running argmax for the lm_head stage (lane b / 16 + b keeps batch row b)
  float am_v = -INFINITY;
  int am_i = 0x7fffffff;
#if XB_TENSOR_TILES
  int am_b = -1;  // batch row whose logits this thread reduced
#endif

  __device__ Consumer(const StepParams &p_, SmemHdr *h, float *r, unsigned *rp, float *hr, char *u,
                      char *rg)
      : p(p_), hdr(h), red(r), rope(rp), hres(hr), U(u), ring(rg) {
    tid = threadIdx.x;
    warp = tid >> 5;
    lane = tid & 31;
    epoch = hdr->epoch;
  }

  // cos/sin of (float)pos * inv_freq[f] for every row and frequency, rounded to bf16 as the
  // reference's rotary tables (same fp32 angle and functions as a per-layer evaluation).
  __device__ void rope_table() {
    const int nf = p.RD / 2;
    for (int i = tid; i < p.B * nf; i += kCT) {
      const int b = i / nf, f = i % nf;
      const float ang = (float)hdr->pos[b] * p.inv_freq[f];
      rope[b * kRopeFreqs + f] = pack2(cosf(ang), sinf(ang));
    }
    csync();
  }

  __device__ __forceinline__ void csync() { named_sync<kCT>(1); }
  __device__ __forceinline__ unsigned tag(int l, int k) const { return tag_of(epoch, l, k); }

  // Abort rules: every consumer thread always executes the same sequence of named barriers.
  // An abort (device error word set anywhere in the grid) only makes waits give up.
  __device__ __forceinline__ bool aborted() const {
    return *reinterpret_cast<volatile int *>(&hdr->abort) != 0;
  }
  __device__ void set_abort(unsigned code) {
    atomicCAS(p.ctrl + CTL_ERR, 0u, code);
    *reinterpret_cast<volatile int *>(&hdr->abort) = 1;
  }
  __device__ __forceinline__ volatile int *abort_flag() const {
    return reinterpret_cast<volatile int *>(&hdr->abort);
  }
  __device__ __forceinline__ bool give_up(uint64_t &t0) const {
    return wait_give_up(abort_flag(), p.ctrl, t0);
  }

  // ---- tagged inputs -----------------------------------------------------------------------
  // Callers load first (plain L2 loads, all issued together) and only fall into the
  // non-inlined slow paths for words whose tag is not there yet.
  __device__ __forceinline__ uint4 poll4(const unsigned *w, unsigned tg) const {
    const uint4 v = ldcg_u4(w);
    return tag4_ok(v, tg) ? v : repoll4(w, tg, abort_flag(), p.ctrl);
  }
  __device__ __forceinline__ uint4 check4(const unsigned *w, uint4 v, unsigned tg) const {
    return tag4_ok(v, tg) ? v : repoll4(w, tg, abort_flag(), p.ctrl);
  }
  __device__ __forceinline__ unsigned poll1(const unsigned *w, unsigned tg) const {
    const unsigned v = ld_poll_u32(w);
    return (v >> 16) == tg ? v : repoll1(w, tg, abort_flag(), p.ctrl);
  }
  __device__ __forceinline__ ulonglong2 poll2f(const u64 *w, unsigned tg) const {
    const ulonglong2 v = ldcg_u64x2(w);
    return (ftag_tag(v.x) == tg && ftag_tag(v.y) == tg) ? v : repoll2f(w, tg, abort_flag(), p.ctrl);
  }

  // Completes a batch of tagged loads: words v[i] with want(i) that are not ok() yet are loaded
  // again, all of them back to back, until every one is ready, so a late batch costs one L2
  // round trip per round instead of one per word. addr(i) is word i's address.
  template <int N, class Addr, class Want, class Ok>
  __device__ __forceinline__ void settle(uint4 (&v)[N], Addr addr, Want want, Ok ok) const {
    bool late = false;
#pragma unroll
    for (int i = 0; i < N; ++i) late |= want(i) && !ok(v[i]);
    uint64_t t0 = 0;
    for (unsigned round = 1; late; ++round) {
      poll_pause();
#pragma unroll
      for (int i = 0; i < N; ++i)
        if (want(i) && !ok(v[i])) v[i] = ld_poll_u4(addr(i));
      late = false;
#pragma unroll
      for (int i = 0; i < N; ++i) late |= want(i) && !ok(v[i]);
      if (late && (round & 15u) == 0 && give_up(t0)) break;
    }
  }
  template <int N, class Addr, class Want>
  __device__ __forceinline__ void settle1(unsigned (&v)[N], Addr addr, Want want, unsigned tg) const {
    bool late = false;
#pragma unroll
    for (int i = 0; i < N; ++i) late |= want(i) && (v[i] >> 16) != tg;
    uint64_t t0 = 0;
    for (unsigned round = 1; late; ++round) {
      poll_pause();
#pragma unroll
      for (int i = 0; i < N; ++i)
        if (want(i) && (v[i] >> 16) != tg) v[i] = ld_poll_u32(addr(i));
      late = false;
#pragma unroll
      for (int i = 0; i < N; ++i) late |= want(i) && (v[i] >> 16) != tg;
      if (late && (round & 15u) == 0 && give_up(t0)) break;
    }
  }

  // settle() for vectors of two {fp32, tag} words.
  template <int N, class Addr, class Want>
  __device__ __forceinline__ void settle64(ulonglong2 (&v)[N], Addr addr, Want want, unsigned tg) const {
    auto ok = [&](const ulonglong2 &w) { return ftag_tag(w.x) == tg && ftag_tag(w.y) == tg; };
    bool late = false;
#pragma unroll
    for (int i = 0; i < N; ++i) late |= want(i) && !ok(v[i]);
    uint64_t t0 = 0;
    for (unsigned round = 1; late; ++round) {
      poll_pause();
#pragma unroll
      for (int i = 0; i < N; ++i)
        if (want(i) && !ok(v[i])) v[i] = ld_poll_u64x2(addr(i));
      late = false;
#pragma unroll
      for (int i = 0; i < N; ++i) late |= want(i) && !ok(v[i]);
      if (late && (round & 15u) == 0 && give_up(t0)) break;
    }
  }

  __device__ void stage_begin() {
    unsigned long long *tr = p.trace ? p.trace + (size_t)blockIdx.x * kTraceStride : nullptr;
    const int si = sidx < kTraceStages ? sidx : kTraceStages - 1;
    if (tr && tid == 0) tr[3 * si] = tr[3 * si + 1] = tr[3 * si + 2] = globaltimer();
    withhold = blockIdx.x == 0 && sidx == c_withhold_stage;
    ++sidx;
  }
  // Stamps of the current stage: [0] begin, [1] inputs ready (end of a GEMV prologue),
  // [2] weight tiles done.
  __device__ void trace_mark(int k) {
    if (p.trace && tid == 0) {
      const int si = (sidx - 1) < kTraceStages ? sidx - 1 : kTraceStages - 1;
      unsigned long long *tr = p.trace + (size_t)blockIdx.x * kTraceStride + 3 * si;
      const unsigned long long t = globaltimer();
      tr[2] = t;
      if (k == 1) tr[1] = t;
    }
  }
  __device__ void trace_end() {
    if (p.trace && tid == 0) {
      unsigned long long *tr = p.trace + (size_t)blockIdx.x * kTraceStride;
      tr[3 * kTraceStages] = globaltimer();
      tr[3 * kTraceStages + 1] = full_wait;
      tr[3 * kTraceStages + 2] = (unsigned long long)sidx;
      tr[3 * kTraceStages + 6] = poll_wait;
    }
  }

  __device__ const char *wait_full() {
    if (aborted()) return nullptr;
    uint64_t t0 = 0;
    unsigned spins = 0;
    const uint64_t tw = (p.trace && tid == 0) ? globaltimer() : 0;
    while (!mbar_try_wait(&hdr->full[slot], phase)) {
      if ((++spins & 63u) == 0 && give_up(t0)) return nullptr;
    }
    if (p.trace && tid == 0) full_wait += globaltimer() - tw;
    return ring + (size_t)slot * kSlot;
  }
  __device__ void release() {
    __syncwarp();
    if (lane == 0) mbar_arrive(&hdr->empty[slot]);
    if (++slot == p.nslots) { slot = 0; phase ^= 1u; }
  }

  // 16 bytes (8 bf16) of residual-stream row b at element e: the embedding row before layer 0's
  // first residual update, afterwards the tagged stream written by the RESID epilogues.
  __device__ __forceinline__ uint4 pack_words(const uint4 &a, const uint4 &c) {
    return make_uint4((a.x & 0xffffu) | (a.y << 16), (a.z & 0xffffu) | (a.w << 16),
                      (c.x & 0xffffu) | (c.y << 16), (c.z & 0xffffu) | (c.w << 16));
  }

#if !XB_TENSOR_TILES
  // RMSNorm of the residual stream into the activation buffer (bf16 [NB][H]).
  //  Qwen3   : w * bf16(x * rsqrt(mean(x^2) + eps))        (HF Qwen3RMSNorm)
  //  Qwen3.5 : bf16(x * rsqrt(mean(x^2) + eps) * (1 + w))   (HF Qwen3_5RMSNorm)
  __device__ void norm_prologue(const bf16 *w, unsigned tg) {
    uint4 *act = reinterpret_cast<uint4 *>(U);
    const int H = p.H, nc = H / 8;
    constexpr int MAXC = 2;  // H <= 2 * 256 * 8
    uint4 xv[NB][MAXC], wv[MAXC];
    if (!h_ready) {
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kCT;
        wv[i] = c < nc ? ldnc_u4(w + c * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int b = 0; b < NB; ++b)
          xv[b][i] = (c < nc && b < p.B) ? ldnc_u4(p.embed + (size_t)hdr->ids[b] * H + c * 8)
                                          : make_uint4(0, 0, 0, 0);
      }
    } else {
      uint4 lo4[NB][MAXC], hi4[NB][MAXC];
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kCT;
        wv[i] = c < nc ? ldnc_u4(w + c * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const bool ok = c < nc && b < p.B;
          lo4[b][i] = ok ? ldcg_u4(p.h + (size_t)b * H + c * 8) : make_uint4(0, 0, 0, 0);
          hi4[b][i] = ok ? ldcg_u4(p.h + (size_t)b * H + c * 8 + 4) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kCT;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          if (c < nc && b < p.B) {
            const uint4 a = check4(p.h + (size_t)b * H + c * 8, lo4[b][i], tg);
            const uint4 d = check4(p.h + (size_t)b * H + c * 8 + 4, hi4[b][i], tg);
            xv[b][i] = pack_words(a, d);
          } else {
            xv[b][i] = make_uint4(0, 0, 0, 0);
          }
        }
      }
    }
    float ss[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      ss[b] = 0.f;
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        float x[8];
        unpack8(xv[b][i], x);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss[b] = fmaf(x[e], x[e], ss[b]);
      }
      ss[b] = warp_sum(ss[b]);
    }
    if (lane == 0)
#pragma unroll
      for (int b = 0; b < NB; ++b) red[warp * NB + b] = ss[b];
    csync();
    const bool q35 = p.family == XB_FAMILY_QWEN35;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < kWarps; ++i) tot += red[i * NB + b];
      const float r = rsqrtf(tot / (float)H + p.eps);
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kCT;
        if (c >= nc) continue;
        float x[8], wf[8], y[8];
        unpack8(xv[b][i], x);
        unpack8(wv[i], wf);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          y[e] = (b < p.B) ? (q35 ? x[e] * r * (1.f + wf[e]) : wf[e] * rbf(x[e] * r)) : 0.f;
        act[b * (nc + kPad) + c] = make_uint4(pack2(y[0], y[1]), pack2(y[2], y[3]), pack2(y[4], y[5]),
                                     pack2(y[6], y[7]));
      }
    }
  }
#else
  // RMSNorm of the residual stream for batch rows 4..8 (same formula and summation order as the
  // small-batch version): two rows' tagged words per round trip, the raw bf16 rows staged in the
  // (padded) activation rows and normalised there in place.
  __device__ void norm_prologue(const bf16 *w, unsigned tg) {
    uint4 *act = reinterpret_cast<uint4 *>(U);
    const int H = p.H, nc = H / 8, ap = nc + 1;
    constexpr int MAXC = 2;  // H <= 2 * 256 * 8
    uint4 wv[MAXC];
    float ss[NB];
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * kCT;
      wv[i] = c < nc ? ldnc_u4(w + c * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) ss[b] = 0.f;
    auto sumsq = [&](const uint4 &xv, float acc) {
      float x[8];
      unpack8(xv, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(x[e], x[e], acc);
      return acc;
    };
#pragma unroll
    for (int b0 = 0; b0 < NB; b0 += 2) {
      if (!h_ready) {
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int i = 0; i < MAXC; ++i) {
            const int c = tid + i * kCT, b = b0 + j;
            if (c >= nc) continue;
            const uint4 xv = b < p.B ? ldnc_u4(p.embed + (size_t)hdr->ids[b] * H + c * 8) : make_uint4(0, 0, 0, 0);
            act[b * ap + c] = xv;
            ss[b] = sumsq(xv, ss[b]);
          }
      } else {
        uint4 u[2 * MAXC * 2];  // (row j, chunk i, half)
        auto addr = [&](int k) {
          const int j = k / (2 * MAXC), i = (k / 2) % MAXC;
          return p.h + (size_t)(b0 + j) * H + (tid + i * kCT) * 8 + (k & 1) * 4;
        };
        auto want = [&](int k) {
          const int j = k / (2 * MAXC), i = (k / 2) % MAXC;
          return tid + i * kCT < nc && b0 + j < p.B;
        };
#pragma unroll
        for (int k = 0; k < 2 * MAXC * 2; ++k) u[k] = want(k) ? ldcg_u4(addr(k)) : make_uint4(0, 0, 0, 0);
        settle(u, addr, want, [&](const uint4 &v) { return tag4_ok(v, tg); });
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int i = 0; i < MAXC; ++i) {
            const int c = tid + i * kCT, b = b0 + j, k = (j * MAXC + i) * 2;
            if (c >= nc) continue;
            const uint4 xv = b < p.B ? pack_words(u[k], u[k + 1]) : make_uint4(0, 0, 0, 0);
            act[b * ap + c] = xv;
            ss[b] = sumsq(xv, ss[b]);
          }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const float t = warp_sum(ss[b]);
      if (lane == 0) red[warp * NB + b] = t;
    }
    csync();
    const bool q35 = p.family == XB_FAMILY_QWEN35;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < kWarps; ++i) tot += red[i * NB + b];
      const float r = rsqrtf(tot / (float)H + p.eps);
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kCT;
        if (c >= nc) continue;
        float x[8], wf[8], y[8];
        unpack8(act[b * ap + c], x);
        unpack8(wv[i], wf);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          y[e] = (b < p.B) ? (q35 ? x[e] * r * (1.f + wf[e]) : wf[e] * rbf(x[e] * r)) : 0.f;
        act[b * ap + c] = make_uint4(pack2(y[0], y[1]), pack2(y[2], y[3]), pack2(y[4], y[5]),
                                     pack2(y[6], y[7]));
      }
    }
  }

#endif

#if !XB_TENSOR_TILES
  // Tagged bf16 vector [B][K] (row stride ld words) into the activations.
  __device__ void copy_prologue(const unsigned *src, int K, int ld, unsigned tg) {
    uint2 *act = reinterpret_cast<uint2 *>(U);  // 4 bf16 per uint2
    const int nq = K / 4;
    constexpr int MAXC = 10;  // K <= 10 * 256 * 4
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      uint4 v[MAXC];
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kCT;
        v[i] = (c < nq && b < p.B) ? ldcg_u4(src + (size_t)b * ld + c * 4) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kCT;
        if (c >= nq) continue;
        uint2 o = make_uint2(0, 0);
        if (b < p.B) {
          const uint4 q = check4(src + (size_t)b * ld + c * 4, v[i], tg);
          o = make_uint2((q.x & 0xffffu) | (q.y << 16), (q.z & 0xffffu) | (q.w << 16));
        }
        act[b * (nq + 2 * kPad) + c] = o;
      }
    }
  }
#else
  // Tagged bf16 vectors [B][K] (row stride ld words) into the padded activation rows, batch
  // rows 4..8: all words of a row in one round trip.
  __device__ void copy_prologue(const unsigned *src, int K, int ld, unsigned tg) {
    uint2 *act = reinterpret_cast<uint2 *>(U);  // 4 bf16 per uint2
    const int nq = K / 4, aq = nq + 2;
    constexpr int MAXC = 10;  // K <= 10 * 256 * 4
#pragma unroll 1
    for (int b = 0; b < NB; ++b) {
      uint4 v[MAXC];
      auto addr = [&](int i) { return src + (size_t)b * ld + (tid + i * kCT) * 4; };
      auto want = [&](int i) { return tid + i * kCT < nq && b < p.B; };
#pragma unroll
      for (int i = 0; i < MAXC; ++i) v[i] = want(i) ? ldcg_u4(addr(i)) : make_uint4(0, 0, 0, 0);
      settle(v, addr, want, [&](const uint4 &q) { return tag4_ok(q, tg); });
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kCT;
        if (c >= nq) continue;
        const uint4 q = v[i];
        act[b * aq + c] = b < p.B ? make_uint2((q.x & 0xffffu) | (q.y << 16), (q.z & 0xffffu) | (q.w << 16))
                                  : make_uint2(0, 0);
      }
    }
  }

#endif

#if !XB_TENSOR_TILES
  // Gated RMSNorm of the DeltaNet core output (HF Qwen3_5RMSNormGated, as called in
  // compiler/qwen35/adapters/delta.py:46-47): y = bf16( bf16(w * bf16(x * r)) * silu(z) ).
  // One warp covers one head (32 lanes x 4 values) per chunk index; lanes 0..3 load the head's
  // eight per-tile sums of squares (two per lane) and the warp reduces them as
  // ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7)). All loads of a row are issued together
  // and only late words are loaded again.
  __device__ void gated_norm_prologue(const bf16 *w, unsigned tg) {
    uint2 *act = reinterpret_cast<uint2 *>(U);
    const int K = p.HV * p.DK, nq = K / 4, DK = p.DK;
    const int zoff = 2 * p.HK * p.DK + p.HV * p.DK;
    constexpr int MAXC = 4;  // K <= 4 * 256 * 4
    uint2 wq[MAXC];
#pragma unroll
    for (int i = 0; i < MAXC; ++i)
      wq[i] = tid + i * kCT < nq ? *reinterpret_cast<const uint2 *>(w + ((tid + i * kCT) * 4) % DK)
                                 : make_uint2(0, 0);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      uint4 xz[2 * MAXC];  // core chunks, then gate (z) chunks
      ulonglong2 sv[MAXC];
      auto addr = [&](int k) {
        const int c = tid + (k % MAXC) * kCT;
        return k < MAXC ? p.core + (size_t)b * K + c * 4 : p.proj + (size_t)b * p.pstride + zoff + c * 4;
      };
      auto want = [&](int k) { return tid + (k % MAXC) * kCT < nq && b < p.B; };
      auto saddr = [&](int i) {
        const int h = ((tid + i * kCT) * 4) / DK;
        return p.ssq + ((size_t)b * p.HV + h) * 8 + 2 * (lane & 3);
      };
      auto swant = [&](int i) { return tid + i * kCT < nq && b < p.B && lane < 4; };
#pragma unroll
      for (int k = 0; k < 2 * MAXC; ++k) xz[k] = want(k) ? ldcg_u4(addr(k)) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int i = 0; i < MAXC; ++i) sv[i] = swant(i) ? ldcg_u64x2(saddr(i)) : make_ulonglong2(0, 0);
      settle(xz, addr, want, [&](const uint4 &v) { return tag4_ok(v, tg); });
      settle64(sv, saddr, swant, tg);
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kCT;
        float part = lane < 4 ? ftag_val(sv[i].x) + ftag_val(sv[i].y) : 0.f;
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        const float tot = __shfl_sync(0xffffffffu, part, 0);
        if (c >= nq) continue;
        uint2 o = make_uint2(0, 0);
        if (b < p.B) {
          const float r = rsqrtf(tot / (float)DK + p.eps);
          const uint4 xv = xz[i], zv = xz[MAXC + i];
          const uint2 wv = wq[i];
          const float x[4] = {bf_lo(xv.x), bf_lo(xv.y), bf_lo(xv.z), bf_lo(xv.w)};
          const float z[4] = {bf_lo(zv.x), bf_lo(zv.y), bf_lo(zv.z), bf_lo(zv.w)};
          const float wf[4] = {bf_lo(wv.x), bf_hi(wv.x), bf_lo(wv.y), bf_hi(wv.y)};
          float y[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float n = rbf(wf[e] * rbf(x[e] * r));
            y[e] = n * (z[e] / (1.f + expf(-z[e])));
          }
          o = make_uint2(pack2(y[0], y[1]), pack2(y[2], y[3]));
        }
        act[b * (nq + 2 * kPad) + c] = o;
      }
    }
  }
#else
  // Gated RMSNorm of the DeltaNet core output for batch rows 4..8 (same formula as the
  // small-batch version): the per-tile sums of squares of every (row, head) in one round trip,
  // reduced by four lanes each ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7)); then each row's
  // core and gate words in one round trip.
  __device__ void gated_norm_prologue(const bf16 *w, unsigned tg) {
    uint2 *act = reinterpret_cast<uint2 *>(U);
    const int HV = p.HV, DK = p.DK, K = HV * DK, nq = K / 4, aq = nq + 2;
    const int zoff = 2 * p.HK * p.DK + p.HV * p.DK;
    float *rr = red;          // [NB][HV] 1 / rms
    constexpr int MAXC = 4;   // K <= 4 * 256 * 4
    constexpr int MAXS = 4;   // B * HV * 4 <= 4 * 256 (16-byte words of partials)
    const int nsq = p.B * HV * 4;
    {
      ulonglong2 sv[MAXS];
      auto saddr = [&](int i) { return p.ssq + (size_t)(tid + i * kCT) * 2; };
      auto swant = [&](int i) { return tid + i * kCT < nsq; };
#pragma unroll
      for (int i = 0; i < MAXS; ++i) sv[i] = swant(i) ? ldcg_u64x2(saddr(i)) : make_ulonglong2(0, 0);
      settle64(sv, saddr, swant, tg);
#pragma unroll
      for (int i = 0; i < MAXS; ++i) {
        float part = swant(i) ? ftag_val(sv[i].x) + ftag_val(sv[i].y) : 0.f;
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        const int k = tid + i * kCT;
        if ((k & 3) == 0 && k < nsq) rr[k >> 2] = rsqrtf(part / (float)DK + p.eps);
      }
    }
    uint2 wq[MAXC];
#pragma unroll
    for (int i = 0; i < MAXC; ++i)
      wq[i] = tid + i * kCT < nq ? *reinterpret_cast<const uint2 *>(w + ((tid + i * kCT) * 4) % DK)
                                 : make_uint2(0, 0);
    csync();
#pragma unroll 1
    for (int b = 0; b < NB; ++b) {
      uint4 xz[2 * MAXC];  // core chunks, then gate (z) chunks
      auto addr = [&](int k) {
        const int c = tid + (k % MAXC) * kCT;
        return k < MAXC ? p.core + (size_t)b * K + c * 4 : p.proj + (size_t)b * p.pstride + zoff + c * 4;
      };
      auto want = [&](int k) { return tid + (k % MAXC) * kCT < nq && b < p.B; };
#pragma unroll
      for (int k = 0; k < 2 * MAXC; ++k) xz[k] = want(k) ? ldcg_u4(addr(k)) : make_uint4(0, 0, 0, 0);
      settle(xz, addr, want, [&](const uint4 &v) { return tag4_ok(v, tg); });
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kCT;
        if (c >= nq) continue;
        uint2 o = make_uint2(0, 0);
        if (b < p.B) {
          const uint4 xv = xz[i], zv = xz[MAXC + i];
          const uint2 wv = wq[i];
          const float r = rr[b * HV + (c * 4) / DK];
          const float x[4] = {bf_lo(xv.x), bf_lo(xv.y), bf_lo(xv.z), bf_lo(xv.w)};
          const float z[4] = {bf_lo(zv.x), bf_lo(zv.y), bf_lo(zv.z), bf_lo(zv.w)};
          const float wf[4] = {bf_lo(wv.x), bf_hi(wv.x), bf_lo(wv.y), bf_hi(wv.y)};
          float y[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float n = rbf(wf[e] * rbf(x[e] * r));
            y[e] = n * (z[e] / (1.f + expf(-z[e])));
          }
          o = make_uint2(pack2(y[0], y[1]), pack2(y[2], y[3]));
        }
        act[b * aq + c] = o;
      }
    }
  }

#endif

  // Next conv window per channel: [conv[1], conv[2], conv[3], x] for active rows, unchanged for
  // empty rows (recurrent.py:43-52). Runs in the out_proj stage after its prologue has seen
  // every head's core output, i.e. after every DeltaNet item has read the old windows.
  __device__ void conv_state_update(int l, unsigned tg) {
    const int CH = (2 * p.HK + p.HV) * p.DK;
    const uint2 *cin = reinterpret_cast<const uint2 *>(p.sa[l]);
    uint2 *cout = reinterpret_cast<uint2 *>(p.sc[l]);
    int lo, hi;
    cta_range(p.B * CH, blockIdx.x, p.ncta, lo, hi);
    for (int i = lo + tid; i < hi; i += kCT) {
      const int b = i / CH, ch = i % CH;
      const uint2 old = cin[i];
      uint2 nw = old;
      if (p.q_len[b] > 0) {
        const unsigned xw = poll1(p.proj + (size_t)b * p.pstride + ch, tg);
        nw.x = (old.x >> 16) | (old.y << 16);
        nw.y = (old.y >> 16) | ((xw & 0xffffu) << 16);
      }
      cout[i] = nw;
    }
  }

  // This CTA's residual rows from the embedding (before layer 0's first residual update).
  __device__ void hres_from_embedding(int lo, int hi) {
    const int n = hi - lo;
    for (int i = tid; i < NB * n; i += kCT) {
      const int b = i / n, r = i % n;
      hres[b * kResRows + r] = b < p.B ? bf(p.embed[(size_t)hdr->ids[b] * p.H + lo + r]) : 0.f;
    }
  }

  // ---- GEMV tile loop ----------------------------------------------------------------------
  // A warp handles a pair of rows of the tile (two independent FMA chains; gate/up tiles carry
  // four), over all of K or, when the tile has fewer than 16 rows, over 1/S of K with the S
  // partial sums combined through shared memory. Lanes 0..NB-1 run the epilogue of the first
  // row for batch rows 0..NB-1, lanes 16..16+NB-1 that of the second row.
  __device__ __forceinline__ void gemv(int l, int stage) {
    stage_begin();
    const Gemv g = make_gemv(p, l, stage);
    const XbLayerWeights *w = (stage == ST_LMHEAD) ? nullptr : &p.layers[l];
    int lo, hi;
    cta_range(g.N, blockIdx.x, p.ncta, lo, hi);
    int epi = EPI_STORE;
    unsigned otag = 0;  // tag of this stage's outputs
    switch (stage) {
    case ST_IN_DELTA:
    case ST_QKV:
      norm_prologue((const bf16 *)w->input_norm, l > 0 ? tag(l - 1, 1) : 0u);
      otag = tag(l, 0);
      break;
    case ST_OUT_DELTA:
      if (!h_ready) hres_from_embedding(lo, hi);
      gated_norm_prologue((const bf16 *)w->gnorm, tag(l, 0));
      epi = EPI_RESID;
      otag = tag(l, 0);
      break;
    case ST_O:
      if (!h_ready) hres_from_embedding(lo, hi);
      copy_prologue(p.att_out, g.K, p.HQ * p.D, tag(l, 0));
      epi = EPI_RESID;
      otag = tag(l, 0);
      break;
    case ST_GATEUP:
      norm_prologue((const bf16 *)w->post_norm, tag(l, 0));
      epi = EPI_GATEUP;
      otag = tag(l, 0);
      break;
    case ST_DOWN:
      copy_prologue(p.act, g.K, p.I, tag(l, 0));
      epi = EPI_RESID;
      otag = tag(l, 1);
      break;
    case ST_LMHEAD:
      norm_prologue(p.final_norm, tag(p.L - 1, 1));
      epi = EPI_LOGITS;
      break;
    }
    csync();
    // The conv windows may be updated in place only once no DeltaNet item of this layer can
    // still read them: after the csync above, this CTA has observed every head's core output,
    // which each item writes after its last read of the old window.
    if (stage == ST_OUT_DELTA) conv_state_update(l, tag(l, 0));
    trace_mark(1);
    switch (epi) {
    case EPI_STORE: tile_loop<false, EPI_STORE>(g, lo, hi, otag); break;
    case EPI_RESID: tile_loop<false, EPI_RESID>(g, lo, hi, otag); break;
    case EPI_GATEUP: tile_loop<true, EPI_GATEUP>(g, lo, hi, otag); break;
    default: tile_loop<false, EPI_LOGITS>(g, lo, hi, otag); break;
    }
    trace_mark(2);
    if (epi == EPI_RESID) h_ready = true;
    if (epi == EPI_LOGITS) {
      if (p.trace && tid == 0) p.trace[(size_t)blockIdx.x * kTraceStride + 3 * kTraceStages + 7] = globaltimer();
      argmax_finish();
    }
  }

  // Tiles of this CTA's rows [lo, hi) as they arrive in the ring. Full tiles with at least 16
  // rows take the fast path (one pair of rows per warp per pass, all of K); smaller tiles split K
  // over S warps per pair and combine the partial sums in shared memory.
#if XB_TENSOR_TILES
  template <bool PAIRED, int EPI>
  __device__ __forceinline__ void tile_loop(const Gemv &g, int lo, int hi, unsigned otag) {
    tile_loop_mma<PAIRED>(g, lo, hi, otag, EPI);
  }

  // Batch rows 4..8: tensor-core tiles. A tile's rows (gate/up tiles: n gate rows, then n up
  // rows) form one 16-row block; warp w multiplies it by the activations over the w-th eighth of
  // K with m16n8k16 MMAs (rows as M, batch rows as N, missing rows and batch rows as zeros) and
  // the eight partial blocks are summed in a fixed order through shared memory. Rows in shared
  // memory are padded to K * 2 + 16 bytes, so the fragment loads are free of bank conflicts. The
  // K order inside a block is permuted identically for A and B (lane t of a row group reads the
  // four contiguous values 4t..4t+3), which leaves each dot product unchanged.
  template <bool PAIRED>
  __device__ __forceinline__ void tile_loop_mma(const Gemv &g, int lo, int hi, unsigned otag, int epi) {
    const int pitch = g.K * 2 + 16;
    const int R = tile_rows_padded(g);
    const int nkb = g.K / 16;
    const int kb0 = nkb * warp / kWarps, kb1 = nkb * (warp + 1) / kWarps;
    const int gq = lane >> 2, t4 = lane & 3;
    const char *xrow = U + (size_t)gq * pitch;  // activations of batch row gq
    const bool xok = gq < NB;
    for (int r0 = lo; r0 < hi; r0 += R) {
      const int n = min(R, hi - r0);
      const int rows = PAIRED ? 2 * n : n;
      const char *slotp = wait_full();
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      if (slotp) {
        const bool okA = gq < rows, okB = gq + 8 < rows;
        const char *pa = slotp + (size_t)gq * pitch, *pb = slotp + (size_t)(gq + 8) * pitch;
        for (int kb = kb0; kb < kb1; ++kb) {
          const int ko = kb * 32 + t4 * 8;
          const uint2 a = okA ? *reinterpret_cast<const uint2 *>(pa + ko) : make_uint2(0, 0);
          const uint2 c = okB ? *reinterpret_cast<const uint2 *>(pb + ko) : make_uint2(0, 0);
          const uint2 x = xok ? *reinterpret_cast<const uint2 *>(xrow + ko) : make_uint2(0, 0);
          mma_16816(d, a.x, c.x, a.y, c.y, x.x, x.y);
        }
      }
      float *pw = red + warp * 128;  // [16 rows][8 batch rows]
      pw[gq * 8 + 2 * t4] = d[0];
      pw[gq * 8 + 2 * t4 + 1] = d[1];
      pw[(gq + 8) * 8 + 2 * t4] = d[2];
      pw[(gq + 8) * 8 + 2 * t4 + 1] = d[3];
      release();
      csync();
      if (slotp && tid < 128) {
        const int r = tid >> 3, b = tid & 7;
        if (r < n && b < p.B) {
          float v = 0.f, v2 = 0.f;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) v += red[w * 128 + r * 8 + b];
          if (PAIRED)
#pragma unroll
            for (int w = 0; w < kWarps; ++w) v2 += red[w * 128 + (n + r) * 8 + b];
          epilogue(epi, b, r0 + r, v, v2, lo, otag);
        }
      }
      csync();  // partial sums consumed before the next tile writes them
    }
  }
#else
  template <bool PAIRED, int EPI>
  __device__ __forceinline__ void tile_loop(const Gemv &g, int lo, int hi, unsigned otag) {
    tile_loop_fma<PAIRED, EPI>(g, lo, hi, otag);
  }
#endif

  template <bool PAIRED, int EPI>
  __device__ __forceinline__ void tile_loop_fma(const Gemv &g, int lo, int hi, unsigned otag) {
    const uint4 *act4 = reinterpret_cast<const uint4 *>(U);
    const int R = tile_rows(g);
    const int K = g.K, n8 = K / 8;
    const size_t rowb = (size_t)K * 2;
    const int bsel = lane & 15;
    const bool second = lane >= 16;
    // Kernels for wide models (LK): with few rows per ring slot and at least one tile per warp,
    // tile t belongs to warp t % kWarps, which runs all its rows over all of K; no partial sums, no
    // CTA barrier. Every warp still waits for and releases every slot, in order, as in the other
    // paths.
    if (LK && (R + 1) / 2 < kWarps && (hi - lo + R - 1) / R >= kWarps) {
      int t = 0;
      for (int r0 = lo; r0 < hi; r0 += R, ++t) {
        const int n = min(R, hi - r0);
        const char *slotp = wait_full();
        if (slotp && t % kWarps == warp) {
          for (int pair = 0; pair < (n + 1) / 2; ++pair) {
            const int rA = 2 * pair, rB = min(rA + 1, n - 1);
            const uint4 *wA = reinterpret_cast<const uint4 *>(slotp + rA * rowb);
            const uint4 *wB = reinterpret_cast<const uint4 *>(slotp + rB * rowb);
            const uint4 *uA = reinterpret_cast<const uint4 *>(slotp + (n + rA) * rowb);
            const uint4 *uB = reinterpret_cast<const uint4 *>(slotp + (n + rB) * rowb);
            const float2 r = gemv_pair<PAIRED, NB>(wA, wB, uA, uB, act4, n8, 0, n8);
            const int row = rA + (second ? 1 : 0);
            if (bsel < NB && bsel < p.B && row < n) epilogue(EPI, bsel, r0 + row, r.x, r.y, lo, otag);
          }
        }
        release();
      }
      return;
    }
    int parity = 0;
    for (int r0 = lo; r0 < hi; r0 += R, parity ^= 1) {
      const int n = min(R, hi - r0);
      const int pairs = (n + 1) >> 1;
      const char *slotp = wait_full();
      if (pairs >= kWarps) {
        // fast path
        for (int pair = warp; slotp && pair < pairs; pair += kWarps) {
          const int rA = 2 * pair, rB = min(rA + 1, n - 1);
          const uint4 *wA = reinterpret_cast<const uint4 *>(slotp + rA * rowb);
          const uint4 *wB = reinterpret_cast<const uint4 *>(slotp + rB * rowb);
          const uint4 *uA = reinterpret_cast<const uint4 *>(slotp + (n + rA) * rowb);
          const uint4 *uB = reinterpret_cast<const uint4 *>(slotp + (n + rB) * rowb);
          const float2 r = gemv_pair<PAIRED, NB>(wA, wB, uA, uB, act4, n8, 0, n8);
          const int row = rA + (second ? 1 : 0);
          if (bsel < NB && bsel < p.B && row < n) epilogue(EPI, bsel, r0 + row, r.x, r.y, lo, otag);
        }
        release();
        continue;
      }
      int S = 1;
      while (S < kWarps && pairs * S * 2 <= kWarps) S <<= 1;
      const int seg = warp % S;
      const int pair = warp / S;
      const bool active = slotp != nullptr && pair < pairs;
      float a0[NB], a1[NB], c0[NB], c1[NB];
#pragma unroll
      for (int b = 0; b < NB; ++b) { a0[b] = a1[b] = c0[b] = c1[b] = 0.f; }
      if (active) {
        const int rA = 2 * pair, rB = min(rA + 1, n - 1);
        const uint4 *wA = reinterpret_cast<const uint4 *>(slotp + rA * rowb);
        const uint4 *wB = reinterpret_cast<const uint4 *>(slotp + rB * rowb);
        const uint4 *uA = reinterpret_cast<const uint4 *>(slotp + (n + rA) * rowb);
        const uint4 *uB = reinterpret_cast<const uint4 *>(slotp + (n + rB) * rowb);
        const int cb = (n8 * seg) / S, ce = (n8 * (seg + 1)) / S;
#pragma unroll 2
        for (int j = cb + lane; j < ce; j += 32) {
          const uint4 wa = wA[j], wb = wB[j];
          uint4 ua = make_uint4(0, 0, 0, 0), ub = ua;
          if (PAIRED) { ua = uA[j]; ub = uB[j]; }
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            const uint4 x = act4[b * n8 + j];
            a0[b] = dot8_bf16(wa, x, a0[b]);
            c0[b] = dot8_bf16(wb, x, c0[b]);
            if (PAIRED) {
              a1[b] = dot8_bf16(ua, x, a1[b]);
              c1[b] = dot8_bf16(ub, x, c1[b]);
            }
          }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          a0[b] = warp_sum(a0[b]);
          c0[b] = warp_sum(c0[b]);
          if (PAIRED) { a1[b] = warp_sum(a1[b]); c1[b] = warp_sum(c1[b]); }
        }
      }
      float v = 0.f, v2 = 0.f;
#pragma unroll
      for (int b = 0; b < NB; ++b)
        if (bsel == b) { v = second ? c0[b] : a0[b]; v2 = second ? c1[b] : a1[b]; }
      float *part = red + RED_PART + parity * 256;  // [warp][2 rows][NB][2]
      if (active && bsel < NB) {
        float *q = part + ((warp * 2 + (second ? 1 : 0)) * NB + bsel) * 2;
        q[0] = v;
        q[1] = v2;
      }
      csync();
      if (active && seg == 0 && bsel < NB) {
        v = v2 = 0.f;
        for (int sgi = 0; sgi < S; ++sgi) {
          const float *q = part + (((pair * S + sgi) * 2 + (second ? 1 : 0)) * NB + bsel) * 2;
          v += q[0];
          v2 += q[1];
        }
        const int row = 2 * pair + (second ? 1 : 0);
        if (bsel < p.B && row < n) epilogue(EPI, bsel, r0 + row, v, v2, lo, otag);
      }
      release();
    }
  }

  __device__ __forceinline__ void epilogue(int epi, int b, int row, float v, float v2, int lo,
                                           unsigned tg) {
    if (withhold) return;  // fault injection: this stage's outputs of CTA 0 never appear
    switch (epi) {
    case EPI_STORE:
      p.proj[(size_t)b * p.pstride + row] = tagged(v, tg);
      break;
    case EPI_RESID: {
      float *hr = hres + b * kResRows + (row - lo);
      const float hv = rbf(*hr + rbf(v));
      *hr = hv;
      p.h[(size_t)b * p.H + row] = tagged(hv, tg);
      break;
    }
    case EPI_GATEUP: {
      const float gt = rbf(v), up = rbf(v2);
      const float s = rbf(gt / (1.f + expf(-gt)));
      p.act[(size_t)b * p.I + row] = tagged(s * up, tg);
      break;
    }
    case EPI_LOGITS: {
      const float y = p.q_len[b] > 0 ? rbf(v) : 0.f;
      p.logits[(size_t)b * p.V + row] = tobf(y);
#if XB_TENSOR_TILES
      am_b = b;
#endif
      if (argmax_better(y, row, am_v, am_i)) { am_v = y; am_i = row; }
      break;
    }
    }
  }

  // Per-CTA argmax -> workspace; the last CTA to finish reduces all CTAs, writes the tokens,
  // advances the launch epoch and resets its own ticket for the next launch.
  // Batch rows below 4: the epilogue lanes b and 16 + b of each warp hold batch row b.
  __device__ void argmax_lanes() {
    float *sv = red;                                  // [kWarps][2][NB]
    int *si = reinterpret_cast<int *>(red + 2 * kWarps * NB);
    const int bsel = lane & 15;
    if (bsel < NB) {
      const int k = (warp * 2 + (lane >= 16 ? 1 : 0)) * NB + bsel;
      sv[k] = am_v;
      si[k] = am_i;
    }
    csync();
    if (tid < NB && tid < p.B) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int k = 0; k < 2 * kWarps; ++k)
        if (argmax_better(sv[k * NB + tid], si[k * NB + tid], bv, bi)) {
          bv = sv[k * NB + tid];
          bi = si[k * NB + tid];
        }
      p.am_v[blockIdx.x * XB_MAX_BATCH + tid] = bv;
      p.am_i[blockIdx.x * XB_MAX_BATCH + tid] = bi;
    }
  }

  __device__ void argmax_finish() {
#if XB_TENSOR_TILES
    {
      // every thread of the tensor-core epilogue may hold candidates of any batch row
      float *sv = red;
      int *si = reinterpret_cast<int *>(red + kCT);
      int *sb = reinterpret_cast<int *>(red + 2 * kCT);
      csync();  // the lm_head tiles' scratch in red has been consumed
      sv[tid] = am_v;
      si[tid] = am_i;
      sb[tid] = am_b;
      csync();
      if (tid < NB && tid < p.B) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int k = 0; k < kCT; ++k)
          if (sb[k] == tid && argmax_better(sv[k], si[k], bv, bi)) {
            bv = sv[k];
            bi = si[k];
          }
        p.am_v[blockIdx.x * XB_MAX_BATCH + tid] = bv;
        p.am_i[blockIdx.x * XB_MAX_BATCH + tid] = bi;
      }
    }
#else
    argmax_lanes();
#endif
    csync();
    if (tid == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(p.ctrl + CTL_DONE, 1u);
      hdr->is_last = prev == (unsigned)p.ncta - 1u;
    }
    csync();
    if (hdr->is_last) {
      __threadfence();
      // warp b reduces batch row b over all CTAs: lanes load candidates in parallel
      if (warp < p.B && warp < NB && p.tokens) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int c = lane; c < p.ncta; c += 32) {
          const float v = ldcg_f(p.am_v + c * XB_MAX_BATCH + warp);
          const int i = __ldcg(p.am_i + c * XB_MAX_BATCH + warp);
          if (argmax_better(v, i, bv, bi)) { bv = v; bi = i; }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (argmax_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) p.tokens[warp] = bi;
      }
      if (tid == 0) {
        // every CTA has consumed all tagged inputs of this launch before taking a ticket
        p.ctrl[CTL_EPOCH] = epoch + 1u;  // also after an abort: stale tags never match again
        if (hdr->scrub) {
          p.ctrl[CTL_SCRUBBED] = epoch;
          p.ctrl[CTL_SCRUB_BAR] = 0u;
        }
        atomicExch(p.ctrl + CTL_DONE, 0u);
      }
    }
  }

  // ---- Gated DeltaNet recurrent step (compiler/qwen35/kernels/recurrent.py:20-124) ---------
  // Work item = (row b, value head h, 16-column tile t of the 128x128 state). The state slice,
  // conv windows and taps are loaded up front; the projections of this head are polled.
  // ---- Gated DeltaNet, four or more batch rows: one work item per (row, value head) ---------
  // The q/k conv and l2-norms run once per head instead of once per 16-column tile. The head's
  // 128 x 128 fp32 state is updated in four passes of 32 columns: thread t keeps column t & 31 of
  // the pass, rows 16 (t >> 5) .. + 15, and the eight row groups are added in shared memory.
  // Outputs as the per-tile items: the core values, the per-16-column sums of squares for the
  // gated norm, the updated state.
  __device__ __forceinline__ void delta_heads(int l) {
    stage_begin();
    const XbLayerWeights &w = p.layers[l];
    const unsigned tg = tag(l, 0);
    const int HK = p.HK, HV = p.HV, DK = p.DK;
    const int CH = (2 * HK + HV) * DK, CW = p.CW;
    const int group = HV / HK;
    const int items = p.B * HV;
    const bf16 *cw = (const bf16 *)w.conv_w;
    float *qk = red;          // [2 DK]  (q | k)
    float *vv = red + 256;    // [DK]
    float *pn = red + 384;    // [kWarps] norm partials
    float *gt = red + 392;    // beta, decay
    float *pp = red + 400;    // [8][32] prediction partials
    float *po = red + 656;    // [8][32] output partials
    const bf16 *conv_in_all = (const bf16 *)p.sa[l];
    const float *rec_in_all = (const float *)p.sb[l];
    float *rec_out_all = (float *)p.sd[l];
    const int c32 = tid & 31, rg = tid >> 5, r0 = rg * 16;
    for (int item = blockIdx.x; item < items; item += p.ncta) {
      const int b = item / HV;
      const int h = item % HV;
      const int kh = h / group;
      const float *S_in = rec_in_all + (((size_t)b * HV + h) * DK) * DK;
      float *S_out = rec_out_all + (((size_t)b * HV + h) * DK) * DK;
      unsigned *core = p.core + (size_t)b * HV * DK + h * DK;
      u64 *ssq = p.ssq + ((size_t)b * HV + h) * 8;
      if (p.q_len[b] == 0) {
        // Empty row: replacement state equals the input state (a no-op when in place).
        for (int i = tid; i < DK * DK; i += kCT) S_out[i] = S_in[i];
        if (tid < DK) core[tid] = tagged(0.f, tg);
        if (tid < 8) st_u64(ssq + tid, ftag(0.f, tg));
        continue;
      }
      const bf16 *cin = conv_in_all + (size_t)b * CH * CW;
      const unsigned *x = p.proj + (size_t)b * p.pstride;
      // conv channels: q (tid < 128) or k (tid >= 128) of key head kh; v channel tid (< 128)
      const int chq = tid < DK ? kh * DK + tid : (HK + kh) * DK + (tid - DK);
      const int chv = (2 * HK + h) * DK + (tid & 127);
      const uint2 cq = *reinterpret_cast<const uint2 *>(cin + (size_t)chq * CW);
      const uint2 wq = *reinterpret_cast<const uint2 *>(cw + (size_t)chq * CW);
      uint2 cv = make_uint2(0, 0), wvv = make_uint2(0, 0);
      if (tid < DK) {
        cv = *reinterpret_cast<const uint2 *>(cin + (size_t)chv * CW);
        wvv = *reinterpret_cast<const uint2 *>(cw + (size_t)chv * CW);
      }
      float gsc = 0.f;
      if (warp == 0) {
        if (lane == 2) gsc = bf(((const bf16 *)w.dt_bias)[h]);
        else if (lane == 3) gsc = bf(((const bf16 *)w.a_log)[h]);
      }
      // q/k channel, v channel (tid < 128), then b and a (warp 0, lanes 0 and 1), polled together
      unsigned xw[3];
      auto xaddr = [&](int k) { return k == 0 ? x + chq : k == 1 ? x + chv : x + CH + HV * DK + lane * HV + h; };
      auto xwant = [&](int k) { return k == 0 || (k == 1 && tid < DK) || (k == 2 && warp == 0 && lane < 2); };
#pragma unroll
      for (int k = 0; k < 3; ++k) xw[k] = xwant(k) ? ld_poll_u32(xaddr(k)) : 0u;
      settle1(xw, xaddr, xwant, tg);
      trace_mark(1);
      const float xq = bf_lo(xw[0]);
      const float xv = tid < DK ? bf_lo(xw[1]) : 0.f;
      if (warp == 0 && lane < 2) gsc = bf_lo(xw[2]);  // b, a
      // causal conv (width 4) over [conv[1..3], x] + SiLU, rounded as recurrent.py:32-58
      auto conv = [](uint2 cs, uint2 ws, float xx) -> float {
        float tot = 0.f;
        tot = fmaf(bf_hi(cs.x), bf_lo(ws.x), tot);
        tot = fmaf(bf_lo(cs.y), bf_hi(ws.x), tot);
        tot = fmaf(bf_hi(cs.y), bf_lo(ws.y), tot);
        tot = fmaf(xx, bf_hi(ws.y), tot);
        const float v = rbf(tot);
        return rbf(v * (1.f / (1.f + expf(-v))));
      };
      const float qkv_val = conv(cq, wq, xq);
      qk[tid] = qkv_val;
      if (tid < DK) vv[tid] = conv(cv, wvv, xv);
      if (warp == 0) {
        const float bb = __shfl_sync(0xffffffffu, gsc, 0);
        const float aa = __shfl_sync(0xffffffffu, gsc, 1);
        const float dt = __shfl_sync(0xffffffffu, gsc, 2);
        const float al = __shfl_sync(0xffffffffu, gsc, 3);
        if (lane == 0) {
          gt[0] = rbf(1.f / (1.f + expf(-bb)));  // beta
          const float xx = aa + dt;
          const float sp = xx > 20.f ? xx : log1pf(expf(xx));
          gt[1] = expf(-expf(al) * sp);          // decay = exp(g)
        }
      }
      {
        const float sq = warp_sum(qkv_val * qkv_val);
        if (lane == 0) pn[warp] = sq;
      }
      csync();
      const float qs = rsqrtf(pn[0] + pn[1] + pn[2] + pn[3] + 1e-6f);
      const float ks = rsqrtf(pn[4] + pn[5] + pn[6] + pn[7] + 1e-6f);
      const float beta = gt[0], decay = gt[1];
#pragma unroll 1
      for (int pass = 0; pass < 4; ++pass) {
        const int col = pass * 32 + c32;
        float S[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) S[i] = S_in[(size_t)(r0 + i) * DK + col];
        float pr = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          S[i] *= decay;
          pr = fmaf(S[i], qk[DK + r0 + i] * ks, pr);
        }
        pp[rg * 32 + c32] = pr;
        csync();
        float pred = 0.f;
#pragma unroll
        for (int g = 0; g < 8; ++g) pred += pp[g * 32 + c32];
        const float delta_c = (vv[col] - pred) * beta;
        float o = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          S[i] = fmaf(qk[DK + r0 + i] * ks, delta_c, S[i]);
          o = fmaf(S[i], qk[r0 + i] * qs * p.dk_scale, o);
          S_out[(size_t)(r0 + i) * DK + col] = S[i];
        }
        po[rg * 32 + c32] = o;
        csync();
        if (tid < 32) {
          float out = 0.f;
#pragma unroll
          for (int g = 0; g < 8; ++g) out += po[g * 32 + tid];
          const float ob = rbf(out);
          core[pass * 32 + tid] = tagged(ob, tg);
          float sq = ob * ob;
#pragma unroll
          for (int o2 = 8; o2; o2 >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o2);
          if ((tid & 15) == 0) st_u64(ssq + pass * 2 + (tid >> 4), ftag(sq, tg));
        }
      }
    }
  }
  // ---- Gated DeltaNet, one or two batch rows: one item per (row, value head, 16-column tile) --
  __device__ __forceinline__ void delta_tiles(int l) {
    stage_begin();
    const XbLayerWeights &w = p.layers[l];
    const unsigned tg = tag(l, 0);
    const int HK = p.HK, HV = p.HV, DK = p.DK;
    const int CH = (2 * HK + HV) * DK, CW = p.CW;
    const int group = HV / HK;
    const int tiles = DK / 16;
    const int items = p.B * HV * tiles;
    const bf16 *cw = (const bf16 *)w.conv_w;
    float *qk = red;               // [2*DK]  (q | k)
    float *vv = red + 256;         // [16]
    float *pn = red + 272;         // [kWarps] norm partials
    float *gt = red + 280;         // beta, decay
    float *pp = red + 288;         // [kWarps][16] prediction partials
    float *po = red + 416;         // [kWarps][16] output partials
    const bf16 *conv_in_all = (const bf16 *)p.sa[l];
    const float *rec_in_all = (const float *)p.sb[l];
    float *rec_out_all = (float *)p.sd[l];
    const int c = lane & 15;
    const int rbase = warp * 16 + (lane >> 4) * 8;
    for (int item = blockIdx.x; item < items; item += p.ncta) {
      const int b = item / (HV * tiles);
      const int h = (item / tiles) % HV;
      const int t = item % tiles;
      const int kh = h / group;
      const float *S_in = rec_in_all + (((size_t)b * HV + h) * DK) * DK;
      float *S_out = rec_out_all + (((size_t)b * HV + h) * DK) * DK;
      const int col = t * 16 + c;
      float S[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) S[i] = S_in[(size_t)(rbase + i) * DK + col];
      unsigned *core = p.core + (size_t)b * HV * DK + h * DK + t * 16;
      u64 *ssq = p.ssq + ((size_t)b * HV + h) * 8 + t;
      if (p.q_len[b] == 0) {
        // Empty row: replacement state equals the input state (a no-op when in place).
#pragma unroll
        for (int i = 0; i < 8; ++i) S_out[(size_t)(rbase + i) * DK + col] = S[i];
        if (tid < 16) core[tid] = tagged(0.f, tg);
        if (tid == 0) st_u64(ssq, ftag(0.f, tg));
        continue;
      }
      const bf16 *cin = conv_in_all + (size_t)b * CH * CW;
      const unsigned *x = p.proj + (size_t)b * p.pstride;
      // conv channels: q (tid < 128) or k (tid >= 128) of key head kh; v channel for tid < 16
      const int chq = tid < DK ? kh * DK + tid : (HK + kh) * DK + (tid - DK);
      const int chv = (2 * HK + h) * DK + t * 16 + (tid & 15);
      const uint2 cq = *reinterpret_cast<const uint2 *>(cin + (size_t)chq * CW);
      const uint2 wq = *reinterpret_cast<const uint2 *>(cw + (size_t)chq * CW);
      uint2 cv = make_uint2(0, 0), wvv = make_uint2(0, 0);
      if (tid < 16) {
        cv = *reinterpret_cast<const uint2 *>(cin + (size_t)chv * CW);
        wvv = *reinterpret_cast<const uint2 *>(cw + (size_t)chv * CW);
      }
      float gsc = 0.f;
      if (warp == 0) {
        if (lane == 2) gsc = bf(((const bf16 *)w.dt_bias)[h]);
        else if (lane == 3) gsc = bf(((const bf16 *)w.a_log)[h]);
      }
      // q/k channel, v channel (tid < 16), then b and a (warp 0, lanes 0 and 1), polled together
      unsigned xw[3];
      auto xaddr = [&](int k) { return k == 0 ? x + chq : k == 1 ? x + chv : x + CH + HV * DK + lane * HV + h; };
      auto xwant = [&](int k) { return k == 0 || (k == 1 && tid < 16) || (k == 2 && warp == 0 && lane < 2); };
#pragma unroll
      for (int k = 0; k < 3; ++k) xw[k] = xwant(k) ? ld_poll_u32(xaddr(k)) : 0u;
      settle1(xw, xaddr, xwant, tg);
      trace_mark(1);
      const float xq = bf_lo(xw[0]);
      const float xv = tid < 16 ? bf_lo(xw[1]) : 0.f;
      if (warp == 0 && lane < 2) gsc = bf_lo(xw[2]);  // b, a
      // causal conv (width 4) over [conv[1..3], x] + SiLU, rounded as recurrent.py:32-58
      auto conv = [](uint2 cs, uint2 ws, float xx) -> float {
        float tot = 0.f;
        tot = fmaf(bf_hi(cs.x), bf_lo(ws.x), tot);
        tot = fmaf(bf_lo(cs.y), bf_hi(ws.x), tot);
        tot = fmaf(bf_hi(cs.y), bf_lo(ws.y), tot);
        tot = fmaf(xx, bf_hi(ws.y), tot);
        const float v = rbf(tot);
        return rbf(v * (1.f / (1.f + expf(-v))));
      };
      const float qkv_val = conv(cq, wq, xq);
      qk[tid] = qkv_val;
      if (tid < 16) vv[tid] = conv(cv, wvv, xv);
      if (warp == 0) {
        const float bb = __shfl_sync(0xffffffffu, gsc, 0);
        const float aa = __shfl_sync(0xffffffffu, gsc, 1);
        const float dt = __shfl_sync(0xffffffffu, gsc, 2);
        const float al = __shfl_sync(0xffffffffu, gsc, 3);
        if (lane == 0) {
          gt[0] = rbf(1.f / (1.f + expf(-bb)));  // beta
          const float xx = aa + dt;
          const float sp = xx > 20.f ? xx : log1pf(expf(xx));
          gt[1] = expf(-expf(al) * sp);          // decay = exp(g)
        }
      }
      {
        const float sq = warp_sum(qkv_val * qkv_val);
        if (lane == 0) pn[warp] = sq;
      }
      csync();
      const float qs = rsqrtf(pn[0] + pn[1] + pn[2] + pn[3] + 1e-6f);
      const float ks = rsqrtf(pn[4] + pn[5] + pn[6] + pn[7] + 1e-6f);
      const float beta = gt[0], decay = gt[1];
      float kr[8], qr[8];
      float pr = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        kr[i] = qk[DK + rbase + i] * ks;
        qr[i] = qk[rbase + i] * qs * p.dk_scale;
        S[i] *= decay;
        pr = fmaf(S[i], kr[i], pr);
      }
      pr += __shfl_xor_sync(0xffffffffu, pr, 16);
      if (lane < 16) pp[warp * 16 + lane] = pr;
      csync();
      float pred = 0.f;
#pragma unroll
      for (int i = 0; i < kWarps; ++i) pred += pp[i * 16 + c];
      const float delta_c = (vv[c] - pred) * beta;
      float o = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        S[i] = fmaf(kr[i], delta_c, S[i]);
        o = fmaf(S[i], qr[i], o);
        S_out[(size_t)(rbase + i) * DK + col] = S[i];
      }
      o += __shfl_xor_sync(0xffffffffu, o, 16);
      if (lane < 16) po[warp * 16 + lane] = o;
      csync();
      if (tid < 16) {
        float out = 0.f;
#pragma unroll
        for (int i = 0; i < kWarps; ++i) out += po[i * 16 + tid];
        const float ob = rbf(out);
        core[tid] = tagged(ob, tg);
        float sq = ob * ob;
#pragma unroll
        for (int o2 = 8; o2; o2 >>= 1) sq += __shfl_xor_sync(0x0000ffffu, sq, o2);
        if (tid == 0) st_u64(ssq, ftag(sq, tg));
      }
    }
  }

  // per-head items pay off from four rows up (two rows: 32 items leave most SMs idle, 1.14 vs
  // 0.99 ms per step measured with Qwen3.5-0.8B)
  __device__ __forceinline__ void delta(int l) {
    if constexpr (NB >= 4) delta_heads(l);
    else delta_tiles(l);
  }

  // ---- long split-KV ranges: position blocks (long-context kernels, AG > 0) -------------------
  // Warp w takes the blocks w, w + 8, ... of PB = 8 positions of [j0, j1), LPP = 4 lanes per
  // position. Lane sub of a position holds the 16-byte chunks sub, sub + 4, ... of its K row, so
  // each load instruction reads 64 contiguous bytes of every row (8 rows per instruction). A lane
  // issues all loads of its K chunks first, computes its partial scores for every query head of
  // the KV head (G <= GM), adds them over the position's lanes, then issues the loads of its EPL
  // elements of every V row of the block and, while they travel, updates the running maximum,
  // the rescale and the probabilities once per block and head; P.V follows with the block's
  // probabilities broadcast by shuffles. Rounding as the position loop (FlashAttention-2): fp32
  // row sums, P rounded to bf16 for P.V. The warps' partial states are merged one head at a time
  // and written as this split's partials.
  template <int GM, int EPL>
  __device__ __forceinline__ void attn_blocks(const bf16 *kc, const bf16 *vc, int j0, int j1, long long pos,
                                              int b, int kvh, int s, unsigned tg) {
    constexpr int D = EPL * 32, LPP = 4, PB = 32 / LPP, KE = D / LPP, KQ = KE / 8;
    const int G = p.HQ / p.HKV;
    const float *qs = reinterpret_cast<const float *>(U);      // [G][D]
    const float *kn = qs + G * D;                               // [D]
    const float *vn = kn + D;                                   // [D]
    float *mg = reinterpret_cast<float *>(U) + G * D + 2 * D;  // [kWarps][D + 2]
    const float scale = p.att_scale;
    const int sub = lane % LPP, pl = lane / LPP;
    float o[GM][EPL], m[GM], ls[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      m[g] = -INFINITY;
      ls[g] = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[g][e] = 0.f;
    }
    auto dot8 = [](const float4 &a0, const float4 &a1, const float (&k)[8], float acc) {
      acc = fmaf(a0.x, k[0], acc); acc = fmaf(a0.y, k[1], acc); acc = fmaf(a0.z, k[2], acc);
      acc = fmaf(a0.w, k[3], acc); acc = fmaf(a1.x, k[4], acc); acc = fmaf(a1.y, k[5], acc);
      acc = fmaf(a1.z, k[6], acc); acc = fmaf(a1.w, k[7], acc);
      return acc;
    };
    const int nblk = (j1 - j0 + PB - 1) / PB;
    for (int blk = warp; blk < nblk; blk += kWarps) {
      const int jb = j0 + blk * PB, j = jb + pl;
      const bool valid = j < j1, cur = j == pos;
      const bf16 *krow = kc + (size_t)j * D + sub * 8;
      uint4 kr[KQ];
#pragma unroll
      for (int i = 0; i < KQ; ++i) kr[i] = (valid && !cur) ? ldg_u4(krow + i * LPP * 8) : make_uint4(0, 0, 0, 0);
      float sa[GM], sb[GM];
#pragma unroll
      for (int g = 0; g < GM; ++g) sa[g] = sb[g] = 0.f;
#pragma unroll
      for (int i = 0; i < KQ; ++i) {
        float kf[8];
        if (cur) {
#pragma unroll
          for (int e = 0; e < 8; ++e) kf[e] = kn[(i * LPP + sub) * 8 + e];
        } else {
          unpack8(kr[i], kf);
        }
#pragma unroll
        for (int g = 0; g < GM; ++g)
          if (g < G) {
            const float4 *q4 = reinterpret_cast<const float4 *>(qs + g * D + (i * LPP + sub) * 8);
            if (i & 1) sb[g] = dot8(q4[0], q4[1], kf, sb[g]);
            else sa[g] = dot8(q4[0], q4[1], kf, sa[g]);
          }
      }
      const int cnt = min(PB, j1 - jb);
      using VT = typename std::conditional<EPL == 8, uint4, uint2>::type;
      VT vr[PB];
#pragma unroll
      for (int jj = 0; jj < PB; ++jj) {
        const int jr = jb + jj;
        const bool ld = jj < cnt && jr != pos;
        if constexpr (EPL == 8) vr[jj] = ld ? ldg_u4(vc + (size_t)jr * D + lane * 8) : make_uint4(0, 0, 0, 0);
        else vr[jj] = ld ? ldg_u2(vc + (size_t)jr * D + lane * 4) : make_uint2(0, 0);
      }
      // lane 0's position is always in range, so every block maximum is finite
      float pb[GM];
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        pb[g] = 0.f;
        if (g < G) {
          float t = sa[g] + sb[g];
#pragma unroll
          for (int o2 = 1; o2 < LPP; o2 <<= 1) t += __shfl_xor_sync(0xffffffffu, t, o2);
          const float sv = valid ? t * scale : -INFINITY;
          const float mn = fmaxf(m[g], warp_max(sv));
          const float corr = expf(m[g] - mn);
          const float pe = valid ? expf(sv - mn) : 0.f;
          ls[g] = fmaf(ls[g], corr, sub == 0 ? pe : 0.f);
          pb[g] = rbf(pe);
#pragma unroll
          for (int e = 0; e < EPL; ++e) o[g][e] *= corr;
          m[g] = mn;
        }
      }
#pragma unroll
      for (int jj = 0; jj < PB; ++jj) {
        if (jj < cnt) {
          float vf[8];
          if (jb + jj == pos) {
#pragma unroll
            for (int e = 0; e < EPL; ++e) vf[e] = vn[lane * EPL + e];
          } else {
            if constexpr (EPL == 8) unpack8(vr[jj], vf);
            else unpack8(make_uint4(vr[jj].x, vr[jj].y, 0, 0), vf);
          }
#pragma unroll
          for (int g = 0; g < GM; ++g)
            if (g < G) {
              const float pj = __shfl_sync(0xffffffffu, pb[g], jj * LPP);
#pragma unroll
              for (int e = 0; e < EPL; ++e) o[g][e] = fmaf(pj, vf[e], o[g][e]);
            }
        }
      }
    }
    trace_mark(2);
    const int MS = D + 2;
    float *mw = mg + (size_t)warp * MS;
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g >= G) break;
      const float lw = warp_sum(ls[g]);
#pragma unroll
      for (int e = 0; e < EPL; ++e) mw[lane * EPL + e] = o[g][e];
      if (lane == 0) {
        mw[D] = m[g];
        mw[D + 1] = lw;
      }
      csync();
      for (int d = tid; d < D; d += kCT) {
        float M = -INFINITY;
        for (int i = 0; i < kWarps; ++i) M = fmaxf(M, mg[(size_t)i * MS + D]);
        float O = 0.f, Lw = 0.f;
        if (M != -INFINITY) {
          for (int i = 0; i < kWarps; ++i) {
            const float *ms = mg + (size_t)i * MS;
            const float mi = ms[D];
            if (mi == -INFINITY) continue;
            const float f = expf(mi - M);
            O = fmaf(ms[d], f, O);
            Lw = fmaf(ms[D + 1], f, Lw);
          }
        }
        const int hq = kvh * G + g;
        const size_t base = ((size_t)b * p.HQ + hq) * p.splits + s;
        st_u64(p.att_o + base * D + d, ftag(O, tg));
        if (d == 0) st_u64x2(p.att_ml + 2 * base, ftag(M, tg), ftag(Lw, tg));
      }
      csync();
    }
  }

  // ---- attention: q/k norm, RoPE, KV append, split-KV partials ----------------------------
  // Work item = (row b, KV head, split of the populated prefix). Warp w serves query head
  // w % G over positions j with (j - j0) / 1 % P == w / G (P = kWarps / G position lanes); the
  // P partial softmax states of each head are merged in shared memory.
  __device__ __forceinline__ void attn(int l) {
    stage_begin();
    const XbLayerWeights &w = p.layers[l];
    const unsigned tg = tag(l, 0);
    const int D = p.D, HQ = p.HQ, HKV = p.HKV, G = HQ / HKV, RD = p.RD;
    const int P = kWarps / G;
    const bool q35 = p.family == XB_FAMILY_QWEN35;
    const int qrow = q35 ? 2 * D : D;
    const int koff = HQ * qrow, voff = koff + HKV * D;
    const int EPL = D / 32;  // elements per lane (4 or 8)
    const int splits = p.splits;
    const int items = p.B * HKV * splits;
    float *qs = reinterpret_cast<float *>(U);        // [G][D]
    float *kn = qs + G * D;                          // [D]
    float *vn = kn + D;                              // [D]
    float *mg = vn + D;                              // [kWarps][D+2]
    bf16 *kc_all = (bf16 *)p.sa[l];
    bf16 *vc_all = (bf16 *)p.sb[l];
    const float scale = p.att_scale;
    for (int item = blockIdx.x; item < items; item += p.ncta) {
      const int b = item / (HKV * splits);
      const int kvh = (item / splits) % HKV;
      const int s = item % splits;
      if (p.q_len[b] == 0) continue;
      const int kvl = p.kv_len[b];
      const long long pos = hdr->pos[b];
      const int chunk = (kvl + splits - 1) / splits;
      const int j0 = min(kvl, s * chunk), j1 = min(kvl, j0 + chunk);
      const unsigned *x = p.proj + (size_t)b * p.pstride;
      // Long ranges: this item's K/V rows head for L2 while the query is still being computed
      // upstream (the position loop keeps too few loads in flight to pull them from HBM itself).
      // The long-context kernels' position blocks issue a block's loads together and do without
      // (measured faster: the range prefetch delayed the q/k polls).
      if (AG == 0 && tid == 0 && j1 - j0 >= 64) {
        const size_t off = (((size_t)b * HKV + kvh) * p.C + j0) * D;
        prefetch_l2(kc_all + off, (size_t)(j1 - j0) * D * 2);
        prefetch_l2(vc_all + off, (size_t)(j1 - j0) * D * 2);
      }
      // warps 0..G-1: query heads; warp G: new key; warp G+1: new value
      if (warp <= G) {
        const bool isk = warp == G;
        const int hq = kvh * G + warp;
        const unsigned *src = isk ? x + koff + kvh * D : x + hq * qrow;
        const bf16 *nw = (const bf16 *)(isk ? w.k_norm : w.q_norm);
        float v[8], ss = 0.f;
        uint4 q4[2];
        auto qaddr = [&](int i) { return src + lane * EPL + 4 * i; };
        auto qwant = [&](int i) { return 4 * i < EPL; };
#pragma unroll
        for (int i = 0; i < 2; ++i) q4[i] = qwant(i) ? ldcg_u4(qaddr(i)) : make_uint4(0, 0, 0, 0);
        settle(q4, qaddr, qwant, [&](const uint4 &w4) { return tag4_ok(w4, tg); });
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          v[4 * i] = bf_lo(q4[i].x); v[4 * i + 1] = bf_lo(q4[i].y);
          v[4 * i + 2] = bf_lo(q4[i].z); v[4 * i + 3] = bf_lo(q4[i].w);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < EPL) ss = fmaf(v[e], v[e], ss);
        ss = warp_sum(ss);
        const float r = rsqrtf(ss / (float)D + p.eps);
        float *dst = isk ? kn : qs + warp * D;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < EPL) {
            const float wv = bf(nw[lane * EPL + e]);
            v[e] = q35 ? rbf(v[e] * r * (1.f + wv)) : rbf(wv * rbf(v[e] * r));
            dst[lane * EPL + e] = v[e];
          }
        __syncwarp();
        const int half = RD / 2;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < EPL) {
            const int d = lane * EPL + e;
            if (d < RD) {
              const unsigned cw = rope[b * kRopeFreqs + (d < half ? d : d - half)];
              const float cs = bf_lo(cw), sn = bf_hi(cw);
              const float rot = d < half ? -dst[d + half] : dst[d - half];
              v[e] = rbf(rbf(v[e] * cs) + rbf(rot * sn));
            }
          }
        __syncwarp();
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < EPL) dst[lane * EPL + e] = v[e];
      } else if (warp == G + 1) {
        uint4 v4[2];
        auto vaddr = [&](int i) { return x + voff + kvh * D + lane * EPL + 4 * i; };
        auto vwant = [&](int i) { return 4 * i < EPL; };
#pragma unroll
        for (int i = 0; i < 2; ++i) v4[i] = vwant(i) ? ldcg_u4(vaddr(i)) : make_uint4(0, 0, 0, 0);
        settle(v4, vaddr, vwant, [&](const uint4 &w4) { return tag4_ok(w4, tg); });
#pragma unroll
        for (int i = 0; i < 2; ++i)
          if (4 * i < EPL) {
            vn[lane * EPL + 4 * i] = bf_lo(v4[i].x);
            vn[lane * EPL + 4 * i + 1] = bf_lo(v4[i].y);
            vn[lane * EPL + 4 * i + 2] = bf_lo(v4[i].z);
            vn[lane * EPL + 4 * i + 3] = bf_lo(v4[i].w);
          }
      }
      csync();
      trace_mark(1);
      bf16 *kc = kc_all + (((size_t)b * HKV + kvh) * p.C) * D;
      bf16 *vc = vc_all + (((size_t)b * HKV + kvh) * p.C) * D;
      // KV append (compiler/common/kernels/kv_cache.py:8-42): the s == 0 item writes slot pos.
      if (s == 0 && pos >= 0 && pos < p.C && tid < D) {
        kc[(size_t)pos * D + tid] = tobf(kn[tid]);
        vc[(size_t)pos * D + tid] = tobf(vn[tid]);
      }
      if constexpr (AG > 0) {
        if (j1 - j0 >= kAttBlockMin) {
          attn_blocks<AG, AE>(kc, vc, j0, j1, pos, b, kvh, s, tg);
          continue;
        }
      }
      // split-KV partial over positions [j0, j1) for query head g = warp % G
      const int g = warp % G, lane_pos = warp / G;
      float q[8], o[8];
      float m = -INFINITY, lsum = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o[e] = 0.f;
        q[e] = e < EPL ? qs[g * D + lane * EPL + e] : 0.f;
      }
      // one position per step, the next position's K/V rows prefetched (kept packed)
      uint4 kraw = make_uint4(0, 0, 0, 0), vraw = kraw;
      auto fetch = [&](int j, uint4 &kr4, uint4 &vr4) {
        if (j < j1 && j != pos) {
          if (EPL == 8) {
            kr4 = ldg_u4(kc + (size_t)j * D + lane * 8);
            vr4 = ldg_u4(vc + (size_t)j * D + lane * 8);
          } else {
            const uint2 k2 = ldg_u2(kc + (size_t)j * D + lane * 4);
            const uint2 v2 = ldg_u2(vc + (size_t)j * D + lane * 4);
            kr4 = make_uint4(k2.x, k2.y, 0, 0);
            vr4 = make_uint4(v2.x, v2.y, 0, 0);
          }
        }
      };
      fetch(j0 + lane_pos, kraw, vraw);
      for (int j = j0 + lane_pos; j < j1; j += P) {
        const uint4 kcur = kraw, vcur = vraw;
        fetch(j + P, kraw, vraw);
        float kf[8], vf[8];
        if (j == pos) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            kf[e] = e < EPL ? kn[lane * EPL + e] : 0.f;
            vf[e] = e < EPL ? vn[lane * EPL + e] : 0.f;
          }
        } else {
          unpack8(kcur, kf);
          unpack8(vcur, vf);
        }
        float sc = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < EPL) sc = fmaf(q[e], kf[e], sc);
        sc = warp_sum(sc) * scale;
        const float mn = fmaxf(m, sc);
        const float corr = expf(m - mn);
        const float pe = expf(sc - mn);
        lsum = lsum * corr + pe;
        // FlashAttention-2 rounding: the row sum over fp32 probabilities, P.V over bf16 ones
        const float pb = rbf(pe);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < EPL) o[e] = fmaf(pb, vf[e], o[e] * corr);
        m = mn;
      }
      trace_mark(2);
      // merge the P partial states of each head
      const int MS = D + 2;
      float *mw = mg + (size_t)warp * MS;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < EPL) mw[lane * EPL + e] = o[e];
      if (lane == 0) { mw[D] = m; mw[D + 1] = lsum; }
      csync();
      for (int idx = tid; idx < G * D; idx += kCT) {
        const int gg = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int i = 0; i < P; ++i) M = fmaxf(M, mg[(size_t)(i * G + gg) * MS + D]);
        float O = 0.f, Lw = 0.f;
        if (M != -INFINITY) {
          for (int i = 0; i < P; ++i) {
            const float *ms = mg + (size_t)(i * G + gg) * MS;
            const float mi = ms[D];
            if (mi == -INFINITY) continue;
            const float f = expf(mi - M);
            O = fmaf(ms[d], f, O);
            Lw = fmaf(ms[D + 1], f, Lw);
          }
        }
        const int hq = kvh * G + gg;
        const size_t base = ((size_t)b * HQ + hq) * splits + s;
        st_u64(p.att_o + base * D + d, ftag(O, tg));
        if (d == 0) st_u64x2(p.att_ml + 2 * base, ftag(M, tg), ftag(Lw, tg));
      }
      csync();
    }
  }

  // ---- combine split partials, then the Qwen3.5 sigmoid output gate -----------------------
  __device__ __forceinline__ void comb(int l) {
    stage_begin();
    const unsigned tg = tag(l, 0);
    const int D = p.D, HQ = p.HQ, splits = p.splits;
    const bool q35 = p.family == XB_FAMILY_QWEN35;
    const int chunks = D / 32;
    const int items = p.B * HQ * chunks;
    float *ms = red;                 // [splits]  (splits <= 256)
    float *ls = red + 256;           // [splits]
    float *po = red + 512;           // [kWarps][32] O partials
    float *pl = red + 512 + 256;     // [kWarps] L partials
    for (int item = blockIdx.x; item < items; item += p.ncta) {
      const int b = item / (HQ * chunks);
      const int hq = (item / chunks) % HQ;
      const int ck = item % chunks;
      const int d = ck * 32 + lane;
      unsigned *dst = p.att_out + (size_t)b * HQ * D + hq * D;
      if (p.q_len[b] == 0) {
        if (warp == 0) dst[d] = tagged(0.f, tg);
        continue;
      }
      const size_t base = ((size_t)b * HQ + hq) * splits;
      for (int s = tid; s < splits; s += kCT) {
        ulonglong2 v = ldcg_u64x2(p.att_ml + 2 * (base + s));
        if (ftag_tag(v.x) != tg || ftag_tag(v.y) != tg)
          v = repoll2f(p.att_ml + 2 * (base + s), tg, abort_flag(), p.ctrl);
        ms[s] = ftag_val(v.x);
        ls[s] = ftag_val(v.y);
      }
      csync();
      trace_mark(1);
      float M = -INFINITY;
      for (int s = 0; s < splits; ++s) M = fmaxf(M, ms[s]);
      float O = 0.f, Lw = 0.f;
      if (M != -INFINITY) {
        constexpr int MSP = 10;  // splits handled per pass per warp
        for (int s0 = warp; s0 < splits; s0 += kWarps * MSP) {
          u64 vo[MSP];
#pragma unroll
          for (int i = 0; i < MSP; ++i) {
            const int s = s0 + i * kWarps;
            vo[i] = (s < splits && ms[s] != -INFINITY) ? ldcg_u64(p.att_o + (base + s) * D + d)
                                                       : ftag(0.f, tg);
          }
#pragma unroll
          for (int i = 0; i < MSP; ++i) {
            const int s = s0 + i * kWarps;
            if (s >= splits || ms[s] == -INFINITY) continue;
            const float ov = ftag_tag(vo[i]) == tg ? ftag_val(vo[i])
                                                   : repoll1f(p.att_o + (base + s) * D + d, tg, abort_flag(),
                                                              p.ctrl);
            const float f = expf(ms[s] - M);
            O = fmaf(ov, f, O);
            Lw = fmaf(ls[s], f, Lw);
          }
        }
      }
      po[warp * 32 + lane] = O;
      if (lane == 0) pl[warp] = Lw;
      csync();
      if (warp == 0) {
        float Ot = 0.f, Lt = 0.f;
        for (int i = 0; i < kWarps; ++i) { Ot += po[i * 32 + lane]; Lt += pl[i]; }
        float y = Lt > 0.f ? rbf(Ot / Lt) : 0.f;
        if (q35) {
          const float gtv =
              bf_lo(poll1(p.proj + (size_t)b * p.pstride + hq * 2 * D + D + d, tg));
          const float sg = rbf(1.f / (1.f + expf(-gtv)));
          y = rbf(y * sg);
        }
        dst[d] = tagged(y, tg);
      }
      csync();
    }
  }
};

template <class V> __device__ __forceinline__ void walk_step(const StepParams &p, V &v) {
  for (int l = 0; l < p.L; ++l) {
    if (is_delta(p, l)) {
      v.gemv(l, ST_IN_DELTA);
      v.delta(l);
      v.gemv(l, ST_OUT_DELTA);
    } else {
      v.gemv(l, ST_QKV);
      v.attn(l);
      v.comb(l);
      v.gemv(l, ST_O);
    }
    v.gemv(l, ST_GATEUP);
    v.gemv(l, ST_DOWN);
  }
  v.gemv(-1, ST_LMHEAD);
}

// Clears this CTA's share of the tagged buffers, then waits (bounded) until every CTA has cleared
// its share, so that no stage of this launch writes a value that another CTA's clear erases.
// Every thread of the CTA takes part. The last CTA of the launch records the epoch of the clear
// and resets the arrival counter.
static __device__ __noinline__ void scrub_tagged(const StepParams &p) {
  int lo, hi;
  cta_range((int)p.scrub_chunks, blockIdx.x, p.ncta, lo, hi);
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int i = lo + (int)threadIdx.x; i < hi; i += kThreads) __stcg(p.scrub_base + i, z);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(p.ctrl + CTL_SCRUB_BAR, 1u);
    const uint64_t t0 = globaltimer();
    while (ld_acquire(p.ctrl + CTL_SCRUB_BAR) < (unsigned)p.ncta) {
      if (ld_volatile(p.ctrl + CTL_ERR)) break;
      if (globaltimer() - t0 > c_wait_limit_ns) {
        atomicCAS(p.ctrl + CTL_ERR, 0u, (unsigned)DERR_WAIT);
        break;
      }
    }
  }
  __syncthreads();
}

template <int NB, int AG = 0, int AE = 0, int LK = 0>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(1024) char smem[];
  SmemHdr *hdr = reinterpret_cast<SmemHdr *>(smem);
  float *hres = reinterpret_cast<float *>(smem + kHdrBytes);
  float *red = reinterpret_cast<float *>(smem + kHdrBytes + kResBytes);
  unsigned *rope = reinterpret_cast<unsigned *>(smem + kHdrBytes + kResBytes + kRedFloats * 4);
  char *U = smem + kUOffset;
  char *ring = U + p.ubytes;
  if (threadIdx.x == 0) {
    for (int i = 0; i < p.nslots; ++i) {
      mbar_init(&hdr->full[i], 1);
      mbar_init(&hdr->empty[i], kWarps);
    }
    hdr->abort = 0;
    hdr->is_last = 0;
    hdr->epoch = ld_volatile(p.ctrl + CTL_EPOCH);
    // unsigned difference: an epoch moved backwards also counts as "long ago"
    hdr->scrub = hdr->epoch - ld_volatile(p.ctrl + CTL_SCRUBBED) >= kScrubInterval;
    mbar_fence_init();
  }
  // validate token ids once (out-of-range ids are recorded and read as id 0 nowhere: abort)
  if (threadIdx.x < XB_MAX_BATCH) {
    const int b = threadIdx.x;
    const long long id = b < p.B ? token_id(p, b) : 0;
    hdr->ids[b] = id;
    hdr->pos[b] = b < p.B ? position(p, b) : 0;
    if (id < 0 || id >= p.V) atomicCAS(p.ctrl + CTL_ERR, 0u, (unsigned)DERR_TOKEN);
  }
  __syncthreads();
  if (hdr->scrub) scrub_tagged(p);
  const bool bad = ld_volatile(p.ctrl + CTL_ERR) != 0;
  if (threadIdx.x >= kCT) {
    if (threadIdx.x == kCT && !bad) {
      Producer pr(p, hdr, ring);
      const uint64_t t_start = globaltimer();
      walk_step(p, pr);
      if (p.trace) {
        p.trace[(size_t)blockIdx.x * kTraceStride + 3 * kTraceStages + 3] = globaltimer() - t_start;
        p.trace[(size_t)blockIdx.x * kTraceStride + 3 * kTraceStages + 4] = pr.empty_wait;
        p.trace[(size_t)blockIdx.x * kTraceStride + 3 * kTraceStages + 5] = (unsigned long long)pr.issued;
      }
      // Drain: never leave with bulk copies in flight into this CTA's shared memory. Phases of
      // one slot complete in order, so waiting for the last copy issued into each slot suffices.
      for (int k = max(0, pr.issued - p.nslots); k < pr.issued; ++k) {
        const int slot = k % p.nslots;
        const unsigned parity = (unsigned)((k / p.nslots) & 1);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(&hdr->full[slot], parity)) {
          if (globaltimer() - t0 > 2 * c_wait_limit_ns) {
            atomicCAS(p.ctrl + CTL_ERR, 0u, (unsigned)DERR_DRAIN);
            break;
          }
        }
      }
    }
  } else if (!bad) {
    Consumer<NB, AG, AE, LK> c(p, hdr, red, rope, hres, U, ring);
    c.rope_table();
    walk_step(p, c);
    c.trace_end();
  }
  __syncthreads();
}

// Host helpers of this translation unit's kernels (each compilation keeps its own constants).
template <int NB, int AG = 0, int AE = 0, int LK = 0>
static cudaError_t launch_decode(const StepParams &prm, size_t smem, int ncta, cudaStream_t stream) {
  // The attribute is per function and process-wide; set it once to the opt-in maximum.
  static std::mutex mu;
  static bool configured = false;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured) {
      const cudaError_t e = cudaFuncSetAttribute(decode_kernel<NB, AG, AE, LK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)kSmemLimit);
      if (e != cudaSuccess) return e;
      configured = true;
    }
  }
  (void)smem;
  void *args[] = {const_cast<StepParams *>(&prm)};
  return cudaLaunchCooperativeKernel((const void *)decode_kernel<NB, AG, AE, LK>, dim3(ncta), dim3(kThreads), args,
                                     smem, stream);
}
static cudaError_t set_fault_constants(int stage, unsigned long long limit) {
  cudaError_t e = cudaMemcpyToSymbol(c_withhold_stage, &stage, sizeof(stage));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_wait_limit_ns, &limit, sizeof(limit));
  return e;
}

// Batch rows 4 and 8 (kernels of the tensor-core compilation, decode_tc.cu).
cudaError_t launch_tensor_tiles(int NB, const StepParams &prm, size_t smem, int ncta, cudaStream_t stream);
cudaError_t set_fault_tensor_tiles(int stage, unsigned long long limit);
// One or two batch rows with long split-KV items (kernels of decode_long.cu): kind 1 for head
// dimension 128 with up to two query heads per KV head, kind 2 for head dimension 256 with up to
// four.
cudaError_t launch_long_attention(int NB, int kind, const StepParams &prm, size_t smem, int ncta,
                                  cudaStream_t stream);
cudaError_t set_fault_long_attention(int stage, unsigned long long limit);
// One or two batch rows of wide models (hidden size >= kWideHidden): the kernels whose GEMV
// stages with few rows per ring slot run one tile per warp (decode_wide.cu, and
// decode_wide_long.cu with the long-context attention of head dimension 256).
constexpr int kWideHidden = 2048;
cudaError_t launch_wide(int NB, const StepParams &prm, size_t smem, int ncta, cudaStream_t stream);
cudaError_t set_fault_wide(int stage, unsigned long long limit);
cudaError_t launch_wide_long(int NB, const StepParams &prm, size_t smem, int ncta, cudaStream_t stream);
cudaError_t set_fault_wide_long(int stage, unsigned long long limit);

} // namespace xb
