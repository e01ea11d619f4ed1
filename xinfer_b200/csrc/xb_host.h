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
} // namespace xb
