// Host-side definitions shared by the translation units of libxinfer_b200.so.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "xinfer_b200.h"

// The device plan of one model (xb_model_create): geometry, borrowed weight pointers, the
// per-layer weight table and RoPE inverse frequencies in device memory.
struct XbModel {
  XbGeometry g;
  XbModelWeights w;
  XbLayerWeights *d_layers = nullptr;  // device table
  float *d_inv_freq = nullptr;
  int device = 0;
  int num_sms = 0;
};

namespace xb {
// Records `msg` as the calling thread's last error and returns `code`.
int fail(int code, const std::string &msg);
// out[m, n] (rows ldo elements apart) = x[m, k] . w[n, k]^T in bf16 with fp32 accumulation
// (gemm_tc.cu); xb_gemm_bf16 is the packed case ldo = n. A device-side wait that expired sets
// bit 0 of *err (a library-wide word when err is null).
int gemm_bf16(int m, int n, int k, const void *x, const void *w, void *out, long long ldo, void *stream,
              unsigned *err);
} // namespace xb
