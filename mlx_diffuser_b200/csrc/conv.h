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
  int64_t n_rows;            // output rows to compute: row_order[0 .. n_rows) (n when no list)
  // Halo rows written by other GPUs: tiles at tile-order positions >= wait_from are staged only
  // after every one of the wait_count flags has reached wait_epoch (tcgen05 kernel only).
  int32_t wait_from;         // INT32_MAX: nothing to wait for
  int32_t wait_count;
  int64_t wait_epoch;
  int64_t* const* wait_flags;
};

// CUDA-core kernel: any dtype, shape and layout.
int conv_simt_launch(const ConvArgs& a, cudaStream_t s);

// tcgen05 kernel: fp16/bf16, OKI weight layout, shapes accepted by conv_tc_supported().
// `tile_order` (nullable) lists the 128-row tiles of `row_order`, most expensive first;
// `counter` is one device word the persistent scheduler hands out work items from.
bool conv_tc_supported(const ConvArgs& a);
int conv_tc_launch(const ConvArgs& a, const int32_t* tile_order, int32_t* counter,
                   cudaStream_t s);

// 3xTF32 tcgen05 kernel for fp32 (OKI layout, Cin % 32 == 0, Cout % 32 == 0, K <= 27):
// `split` holds conv_tf32_split_bytes() of scratch for the weight's hi / lo halves.
bool conv_tf32_supported(const ConvArgs& a);
size_t conv_tf32_split_bytes(int kvol, int cin, int cout);
int conv_tf32_launch(const ConvArgs& a, const int32_t* tile_order, int32_t* counter, void* split,
                     cudaStream_t s);

}  // namespace sv
