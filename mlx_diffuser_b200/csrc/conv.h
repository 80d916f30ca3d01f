// Internal interface between the convolution entry point and its kernels.
#pragma once

#include "common.cuh"

namespace sv {

struct ConvArgs {
  const void* features;      // [n, cin]
  int64_t n;
  int cin;
  const int32_t* nbr;        // [n, kvol]
  int kvol;
  const int32_t* row_order;  // [n] permutation or null
  const void* weight;        // layout below
  int layout;                // sv_weight_layout
  const void* bias;          // [cout] or null
  int cout;
  int dtype;                 // sv_dtype of features / weight / bias / out
  void* out;                 // [n, cout]
  int32_t* status;           // device status word or null
  const void* residual;      // [n, cout] added before rounding, or null; may equal `out`
};

// CUDA-core kernel: any dtype, shape and layout.
int conv_simt_launch(const ConvArgs& a, cudaStream_t s);

// tcgen05 kernel: fp16/bf16, OKI weight layout, shapes accepted by conv_tc_supported().
// `tile_order` (nullable) lists the 128-row tiles of `row_order`, most expensive first;
// `counter` is one device word the persistent scheduler hands out work items from.
bool conv_tc_supported(const ConvArgs& a);
int conv_tc_launch(const ConvArgs& a, const int32_t* tile_order, int32_t* counter,
                   cudaStream_t s);

}  // namespace sv
