// C-ABI entry points for the convolution, weight repacking and error reporting.
#include <string>

#include "conv.h"

namespace sv {

namespace {
thread_local std::string g_last_error;

// Tiled transpose of a rows x cols matrix (element type E): the (K*Cin) x Cout weight view
// becomes Cout x (K*Cin), i.e. (K, Cin, Cout) -> (Cout, K, Cin).
template <typename E>
__global__ void transpose_kernel(const E* __restrict__ in, int64_t rows, int64_t cols,
                                 E* __restrict__ out) {
  __shared__ E tile[32][33];
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = in[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * rows + r] = tile[threadIdx.x][i];
  }
}

int transpose(const void* in, int64_t rows, int64_t cols, int esize, void* out, cudaStream_t s) {
  if (rows == 0 || cols == 0) return SV_OK;
  const dim3 block(32, 8), grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
  if ((rows + 31) / 32 > 65535) SV_FAIL(SV_ERR_UNSUPPORTED, "weight too large to repack");
  if (esize == 4)
    transpose_kernel<uint32_t><<<grid, block, 0, s>>>(static_cast<const uint32_t*>(in), rows,
                                                       cols, static_cast<uint32_t*>(out));
  else
    transpose_kernel<uint16_t><<<grid, block, 0, s>>>(static_cast<const uint16_t*>(in), rows,
                                                       cols, static_cast<uint16_t*>(out));
  SV_LAUNCH_CHECK();
  return SV_OK;
}

bool valid_dtype(int d) { return d == SV_FLOAT32 || d == SV_FLOAT16 || d == SV_BFLOAT16; }

// Would the AUTO/TCGEN05 choice take a tensor-core kernel for this shape (after a repack)?
// fp16/bf16 run on conv_tc, fp32 on the 3xTF32 kernel.
bool tc_path(const ConvArgs& a, int algo) {
  if (algo == SV_CONV_SIMT) return false;
  ConvArgs b = a;
  b.layout = SV_WEIGHT_OKI;  // a KIO weight is repacked into an aligned workspace
  if (a.layout == SV_WEIGHT_KIO) b.weight = reinterpret_cast<const void*>(uintptr_t(256));
  return a.dtype == SV_FLOAT32 ? conv_tf32_supported(b) : conv_tc_supported(b);
}

}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }

}  // namespace sv

using namespace sv;

extern "C" const char* sv_last_error(void) { return g_last_error.c_str(); }

extern "C" int sv_abi_version(void) { return 1; }

extern "C" size_t sv_conv3d_workspace_bytes(int64_t n, int cin, int cout, int kvol, int dtype,
                                            int layout, int algo) {
  if (!valid_dtype(dtype) || (layout != SV_WEIGHT_KIO && layout != SV_WEIGHT_OKI)) return 0;
  ConvArgs a{};
  a.n = n;
  a.cin = cin;
  a.cout = cout;
  a.kvol = kvol;
  a.dtype = dtype;
  a.layout = layout;
  a.features = a.out = reinterpret_cast<void*>(uintptr_t(256));
  if (!tc_path(a, algo)) return 0;
  // scheduler word, then (for a KIO weight) the repacked weight, then (fp32) its hi/lo halves
  const size_t repack =
      layout == SV_WEIGHT_KIO ? align_up((size_t)kvol * cin * cout * dtype_size(dtype), 256) : 0;
  const size_t split = dtype == SV_FLOAT32 ? conv_tf32_split_bytes(kvol, cin, cout) : 0;
  return 256 + repack + split;
}

extern "C" int sv_weight_kio_to_oki(const void* w_kio, int kvol, int cin, int cout, int dtype,
                                    void* w_oki, sv_stream_t stream) {
  if (!valid_dtype(dtype)) SV_FAIL(SV_ERR_BAD_DTYPE, "sv_weight_kio_to_oki: unknown dtype");
  if (kvol < 0 || cin < 0 || cout < 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "negative size");
  if ((int64_t)kvol * cin * cout == 0) return SV_OK;
  if (!w_kio || !w_oki) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_weight_kio_to_oki: null pointer");
  return transpose(w_kio, (int64_t)kvol * cin, cout, dtype_size(dtype), w_oki, to_stream(stream));
}

extern "C" int sv_conv3d_forward_rows(const void* features, int64_t n, int cin,
                                      const int32_t* nbr, int kvol, const int32_t* rows,
                                      int64_t n_rows, const int32_t* tile_order,
                                      const void* weight, int layout, const void* bias,
                                      const void* residual, int cout, int dtype, void* out,
                                      int algo, void* workspace, size_t workspace_bytes,
                                      int32_t* status, sv_stream_t stream);

extern "C" int sv_conv3d_forward(const void* features, int64_t n, int cin, const int32_t* nbr,
                                 int kvol, const int32_t* row_order, const int32_t* tile_order,
                                 const void* weight,
                                 int layout, const void* bias, int cout, int dtype, void* out,
                                 int algo, void* workspace, size_t workspace_bytes,
                                 int32_t* status, sv_stream_t stream) {
  return sv_conv3d_forward_residual(features, n, cin, nbr, kvol, row_order, tile_order, weight,
                                    layout, bias, nullptr, cout, dtype, out, algo, workspace,
                                    workspace_bytes, status, stream);
}

extern "C" int sv_conv3d_forward_residual(const void* features, int64_t n, int cin,
                                          const int32_t* nbr, int kvol,
                                          const int32_t* row_order, const int32_t* tile_order,
                                          const void* weight, int layout, const void* bias,
                                          const void* residual, int cout, int dtype, void* out,
                                          int algo, void* workspace, size_t workspace_bytes,
                                          int32_t* status, sv_stream_t stream) {
  return sv_conv3d_forward_rows(features, n, cin, nbr, kvol, row_order, n, tile_order, weight,
                                layout, bias, residual, cout, dtype, out, algo, workspace,
                                workspace_bytes, status, stream);
}

extern "C" int sv_conv3d_forward_rows(const void* features, int64_t n, int cin,
                                      const int32_t* nbr, int kvol, const int32_t* rows,
                                      int64_t n_rows, const int32_t* tile_order,
                                      const void* weight, int layout, const void* bias,
                                      const void* residual, int cout, int dtype, void* out,
                                      int algo, void* workspace, size_t workspace_bytes,
                                      int32_t* status, sv_stream_t stream) {
  const int32_t* row_order = rows;
  // a row list may be longer than n: -1 entries pad schedule segments to whole tiles
  if (n_rows < 0 || n_rows > (int64_t)INT32_MAX - 256)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_forward_rows: bad n_rows");
  if (n_rows != n && rows == nullptr)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_forward_rows: a row subset needs its row list");
  if (n < 0 || cin < 0 || cout < 0 || kvol < 1)
    SV_FAIL(SV_ERR_BAD_SHAPE, "sv_conv3d_forward: negative size or empty kernel");
  if (!valid_dtype(dtype)) SV_FAIL(SV_ERR_BAD_DTYPE, "sv_conv3d_forward: unknown dtype");
  if (layout != SV_WEIGHT_KIO && layout != SV_WEIGHT_OKI)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_forward: unknown weight layout");
  if (algo != SV_CONV_AUTO && algo != SV_CONV_SIMT && algo != SV_CONV_TCGEN05)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_forward: unknown algorithm");
  if (n_rows == 0 || cout == 0) return SV_OK;
  if (!features || !nbr || !out || (!weight && cin > 0))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_forward: null pointer");
  cudaStream_t s = to_stream(stream);
  ConvArgs a{features, n, cin, nbr, kvol, row_order, weight, layout, bias, cout, dtype, out,
             status, residual, n_rows, INT32_MAX, 0, 0, nullptr};
  const bool use_tc = tc_path(a, algo) && aligned16(weight);
  if (algo == SV_CONV_TCGEN05 && !use_tc)
    SV_FAIL(SV_ERR_UNSUPPORTED,
            "tcgen05 convolution needs Cin % 32 == 0, Cout % 32 == 0, kernel volume <= 27 and "
            "16-byte aligned features/weight/out/residual");
  if (!use_tc) return conv_simt_launch(a, s);
  const size_t need = sv_conv3d_workspace_bytes(n, cin, cout, kvol, dtype, layout, algo);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    SV_FAIL(SV_ERR_WORKSPACE,
            "sv_conv3d_forward: the tcgen05 path needs sv_conv3d_workspace_bytes() of workspace");
  int32_t* counter = static_cast<int32_t*>(workspace);
  size_t used = 256;
  if (layout == SV_WEIGHT_KIO) {
    void* packed = static_cast<uint8_t*>(workspace) + used;
    int rc = transpose(weight, (int64_t)kvol * cin, cout, dtype_size(dtype), packed, s);
    if (rc != SV_OK) return rc;
    a.weight = packed;
    a.layout = SV_WEIGHT_OKI;
    used += align_up((size_t)kvol * cin * cout * dtype_size(dtype), 256);
  }
  // tile_order only makes sense together with the row schedule it was derived from
  if (dtype == SV_FLOAT32)
    return conv_tf32_launch(a, row_order ? tile_order : nullptr, counter,
                            static_cast<uint8_t*>(workspace) + used, s);
  return conv_tc_launch(a, row_order ? tile_order : nullptr, counter, s);
}

extern "C" int sv_conv3d_forward_halo(const void* features, int64_t n, int cin,
                                      const int32_t* nbr, int kvol, const int32_t* rows,
                                      int64_t n_rows, const int32_t* tile_order,
                                      int32_t halo_from_tile, int64_t* const* flags,
                                      int flag_count, int64_t epoch, const void* weight,
                                      const void* bias, const void* residual, int cout,
                                      int dtype, void* out, void* workspace,
                                      size_t workspace_bytes, int32_t* status,
                                      sv_stream_t stream) {
  if (n_rows < 0 || n_rows > (int64_t)INT32_MAX - 256 || n < 0 || cin < 0 || cout < 0 ||
      kvol < 1)
    SV_FAIL(SV_ERR_BAD_SHAPE, "sv_conv3d_forward_halo: bad sizes");
  if (!valid_dtype(dtype)) SV_FAIL(SV_ERR_BAD_DTYPE, "sv_conv3d_forward_halo: unknown dtype");
  if (flag_count < 0 || flag_count > 8 || (flag_count > 0 && !flags))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_forward_halo: 0 to 8 flags");
  if (n_rows == 0 || cout == 0) return SV_OK;
  if (!features || !nbr || !out || !weight || !rows)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_forward_halo: null pointer");
  ConvArgs a{features, n, cin, nbr, kvol, rows, weight, SV_WEIGHT_OKI, bias, cout, dtype, out,
             status, residual, n_rows, halo_from_tile, flag_count, epoch, flags};
  if (dtype == SV_FLOAT32 || !tc_path(a, SV_CONV_TCGEN05) || !aligned16(weight))
    SV_FAIL(SV_ERR_UNSUPPORTED,
            "sv_conv3d_forward_halo runs on the tcgen05 kernel: fp16/bf16, Cin % 32 == 0, "
            "Cout % 32 == 0, 16-byte aligned operands");
  if (workspace == nullptr || workspace_bytes < 256 || !aligned16(workspace))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_conv3d_forward_halo: needs 256 bytes of workspace");
  return conv_tc_launch(a, tile_order, static_cast<int32_t*>(workspace), to_stream(stream));
}
