// Backward pass of the submanifold convolution: pair lists, weight / bias gradients on CUDA
// cores, and the weight transform that turns the input gradient into a forward convolution.
//
// mlx_diffuser trains through its gather-matmul fallback (src/mlx_diffuser/layers/sparse.py:233,
// src/mlx_diffuser/kernels/sparse.py:39-55) and lets MLX differentiate
//     out = bias + sum_k (features[max(nbr[:, k], 0)] @ W[k]) * (nbr[:, k] >= 0).
// Its gradients are
//     d features[q] = sum over (p, k) with nbr[p, k] == q of dOut[p] @ W[k]^T
//     d W[k]        = sum over p with nbr[p, k] >= 0 of features[nbr[p, k]]^T dOut[p]
//     d bias        = sum over p of dOut[p].
// * Input gradient: in a submanifold map with unique coordinates, nbr[p, k] == q exactly when
//   nbr[q, K-1-k] == p (offset K-1-k is the negated offset k), so d features is the forward
//   convolution of dOut over the same map with W'[j] = W[K-1-j]^T -- sv_weight_flip_transpose
//   builds W' in the spconv layout and the tensor-core kernel runs unchanged.
// * Weight gradient: per offset, a reduction over the (source, destination) pairs of that
//   offset. sv_kmap_pairs_* lists them, offset after offset, destinations ascending (an ordered
//   compaction of the map); the tensor-core kernel (wgrad_tc.cu) and the CUDA-core kernel below
//   consume those lists.
#include <cub/device/device_scan.cuh>

#include "common.cuh"

namespace sv {
namespace {

constexpr int PAIR_THREADS = 256;
constexpr int PAIR_ITERS = 4;
constexpr int PAIR_TILE = PAIR_THREADS * PAIR_ITERS;  // map rows per tile

__device__ __forceinline__ bool pair_valid(const int32_t* __restrict__ nbr, int64_t n, int kvol,
                                           int k, int64_t p, int32_t* src, int32_t* status) {
  if (p >= n) return false;
  const int32_t s = __ldg(&nbr[p * kvol + k]);
  if (s >= n) {
    report(status, SV_DEVICE_BAD_INDEX);
    return false;
  }
  *src = s;
  return s >= 0;
}

// grid (tiles, kvol): counts[k * tiles + t] = valid pairs of offset k among rows of tile t.
__global__ void __launch_bounds__(PAIR_THREADS)
    pairs_count_kernel(const int32_t* __restrict__ nbr, int64_t n, int kvol,
                       int32_t* __restrict__ counts, int32_t* status) {
  __shared__ int s_warp[PAIR_THREADS / 32];
  const int k = blockIdx.y;
  const int64_t base = (int64_t)blockIdx.x * PAIR_TILE;
  int cnt = 0;
  int32_t src;
#pragma unroll
  for (int i = 0; i < PAIR_ITERS; ++i)
    cnt += pair_valid(nbr, n, kvol, k, base + i * PAIR_THREADS + threadIdx.x, &src, status);
  cnt = __reduce_add_sync(0xffffffffu, cnt);
  if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < PAIR_THREADS / 32; ++w) t += s_warp[w];
    counts[(int64_t)k * gridDim.x + blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(PAIR_THREADS)
    pairs_emit_kernel(const int32_t* __restrict__ nbr, int64_t n, int kvol,
                      const int32_t* __restrict__ incl, int64_t total,
                      int32_t* __restrict__ pair_src, int32_t* __restrict__ pair_dst,
                      int32_t* status) {
  __shared__ int s_warp[PAIR_ITERS][PAIR_THREADS / 32];
  const int k = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tile = (int64_t)k * gridDim.x + blockIdx.x;
  const int64_t base = (int64_t)blockIdx.x * PAIR_TILE;
  int64_t pos0 = tile == 0 ? 0 : (int64_t)incl[tile - 1];
  bool flag[PAIR_ITERS];
  int32_t src[PAIR_ITERS];
  uint32_t ballot[PAIR_ITERS];
#pragma unroll
  for (int i = 0; i < PAIR_ITERS; ++i) {
    src[i] = -1;
    flag[i] = pair_valid(nbr, n, kvol, k, base + i * PAIR_THREADS + threadIdx.x, &src[i],
                         nullptr);
    ballot[i] = __ballot_sync(0xffffffffu, flag[i]);
    if (lane == 0) s_warp[i][warp] = __popc(ballot[i]);
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < PAIR_ITERS; ++i) {
    int before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < PAIR_THREADS / 32; ++w) {
      const int c = s_warp[i][w];
      before += w < warp ? c : 0;
      all += c;
    }
    if (flag[i]) {
      const int64_t pos = pos0 + before + __popc(ballot[i] & ((1u << lane) - 1u));
      if (pos < total) {
        pair_src[pos] = src[i];
        pair_dst[pos] = (int32_t)(base + i * PAIR_THREADS + threadIdx.x);
      } else {
        report(status, SV_DEVICE_BAD_INDEX);  // the map changed since the count
      }
    }
    pos0 += all;
  }
}

int64_t pair_tiles(int64_t n) { return (n + PAIR_TILE - 1) / PAIR_TILE; }

size_t pair_scan_bytes(int64_t entries) {
  size_t b = 0;
  cub::DeviceScan::InclusiveSum(nullptr, b, (const int32_t*)nullptr, (int32_t*)nullptr,
                                (int)entries);
  return b;
}

// offsets[k] = first pair of offset k (k = 0..kvol), read from the tile scan.
__global__ void pair_offsets_kernel(const int32_t* __restrict__ incl, int64_t tiles, int kvol,
                                    int32_t* __restrict__ offsets) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k > kvol) return;
  offsets[k] = k == 0 ? 0 : incl[(int64_t)k * tiles - 1];
}

// ---- weight gradient on CUDA cores ----------------------------------------------------------
// Block (o-tile of 64, i-tile of 64, offset k): 256 threads each own a 4 x 4 sub-tile of
// dW_oki[o][k][i] and walk the offset's pairs in chunks of 16, staging dOut[dst] and
// features[src] rows through shared memory. fp32 accumulation, one rounding.
constexpr int WG_T = 64, WG_K = 16;

template <typename T>
__global__ void __launch_bounds__(256)
    wgrad_simt_kernel(const T* __restrict__ feat, const T* __restrict__ dout, int cin, int cout,
                      int kvol, const int32_t* __restrict__ offsets,
                      const int32_t* __restrict__ pair_src, const int32_t* __restrict__ pair_dst,
                      T* __restrict__ dweight) {
  __shared__ float As[WG_K][WG_T];  // dOut[dst][o0 + m]
  __shared__ float Bs[WG_K][WG_T];  // features[src][i0 + n]
  const int k = blockIdx.z;
  const int o0 = blockIdx.y * WG_T, i0 = blockIdx.x * WG_T;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int32_t begin = __ldg(&offsets[k]), end = __ldg(&offsets[k + 1]);
  float acc[4][4] = {};
  for (int32_t j0 = begin; j0 < end; j0 += WG_K) {
    for (int e = threadIdx.x; e < WG_K * WG_T; e += 256) {
      const int r = e / WG_T, c = e % WG_T;
      const int32_t j = j0 + r;
      float a = 0.f, b = 0.f;
      if (j < end) {
        if (o0 + c < cout) a = to_f32(dout[(int64_t)__ldg(&pair_dst[j]) * cout + o0 + c]);
        if (i0 + c < cin) b = to_f32(feat[(int64_t)__ldg(&pair_src[j]) * cin + i0 + c]);
      }
      As[r][c] = a;
      Bs[r][c] = b;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < WG_K; ++r) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        av[i] = As[r][ty * 4 + i];
        bv[i] = Bs[r][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[i][jj] = fmaf(av[i], bv[jj], acc[i][jj]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int o = o0 + ty * 4 + i;
    if (o >= cout) continue;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int c = i0 + tx * 4 + jj;
      if (c < cin) dweight[((int64_t)o * kvol + k) * cin + c] = from_f32<T>(acc[i][jj]);
    }
  }
}

// ---- bias gradient: column sums, two deterministic passes --------------------------------------
constexpr int DB_ROWS = 1024;  // rows per partial sum

template <typename T>
__global__ void dbias_partial_kernel(const T* __restrict__ dout, int64_t n, int c,
                                     float* __restrict__ partial) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= c) return;
  const int64_t r0 = (int64_t)blockIdx.y * DB_ROWS;
  const int64_t r1 = r0 + DB_ROWS < n ? r0 + DB_ROWS : n;
  float s = 0.f;
  for (int64_t r = r0; r < r1; ++r) s += to_f32(dout[r * c + col]);
  partial[(int64_t)blockIdx.y * c + col] = s;
}

template <typename T>
__global__ void dbias_final_kernel(const float* __restrict__ partial, int parts, int c,
                                   T* __restrict__ dbias) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= c) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += partial[(int64_t)p * c + col];
  dbias[col] = from_f32<T>(s);
}

// ---- W'[i][j][o] = W[o][K-1-j][i] (spconv layout in and out) ---------------------------------
template <typename E>
__global__ void flip_transpose_kernel(const E* __restrict__ w, int cout, int kvol, int cin,
                                      E* __restrict__ out) {
  __shared__ E tile[32][33];
  const int j = blockIdx.z;
  const int kj = kvol - 1 - j;
  const int o0 = blockIdx.y * 32, i0 = blockIdx.x * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int o = o0 + r, i = i0 + threadIdx.x;
    if (o < cout && i < cin) tile[r][threadIdx.x] = w[((int64_t)o * kvol + kj) * cin + i];
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int i = i0 + r, o = o0 + threadIdx.x;
    if (o < cout && i < cin) out[((int64_t)i * kvol + j) * cout + o] = tile[threadIdx.x][r];
  }
}

bool valid_dtype(int d) { return d == SV_FLOAT32 || d == SV_FLOAT16 || d == SV_BFLOAT16; }

}  // namespace
}  // namespace sv

using namespace sv;

extern "C" size_t sv_kmap_pairs_workspace_bytes(int64_t n, int kvol) {
  if (n <= 0 || kvol <= 0) return 256;
  const int64_t entries = pair_tiles(n) * kvol;
  return 2 * align_up((size_t)entries * 4, 256) + align_up(pair_scan_bytes(entries), 256);
}

extern "C" int sv_kmap_pairs_count(const int32_t* nbr, int64_t n, int kvol, int64_t* out_total,
                                   void* workspace, size_t workspace_bytes, int32_t* status,
                                   sv_stream_t stream) {
  if (!out_total) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_pairs_count: null out_total");
  *out_total = 0;
  if (n < 0 || kvol < 1 || kvol > 65535)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_pairs_count: bad n or kernel volume");
  if (n == 0) return SV_OK;
  if (n * (int64_t)kvol > INT32_MAX - PAIR_TILE)
    SV_FAIL(SV_ERR_UNSUPPORTED, "sv_kmap_pairs_count: more than 2^31 map entries");
  if (!nbr) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_pairs_count: null map");
  if (!workspace || workspace_bytes < sv_kmap_pairs_workspace_bytes(n, kvol))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_kmap_pairs_count: workspace too small");
  cudaStream_t s = to_stream(stream);
  const int64_t tiles = pair_tiles(n), entries = tiles * kvol;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t eb = align_up((size_t)entries * 4, 256);
  int32_t* counts = reinterpret_cast<int32_t*>(ws);
  int32_t* incl = reinterpret_cast<int32_t*>(ws + eb);
  void* tmp = ws + 2 * eb;
  size_t tmp_bytes = align_up(pair_scan_bytes(entries), 256);
  pairs_count_kernel<<<dim3((unsigned)tiles, (unsigned)kvol), PAIR_THREADS, 0, s>>>(
      nbr, n, kvol, counts, status);
  SV_LAUNCH_CHECK();
  SV_CUDA_TRY(cub::DeviceScan::InclusiveSum(tmp, tmp_bytes, counts, incl, (int)entries, s));
  int32_t total = 0;
  SV_CUDA_TRY(cudaMemcpyAsync(&total, incl + (entries - 1), sizeof(int32_t),
                              cudaMemcpyDeviceToHost, s));
  SV_CUDA_TRY(cudaStreamSynchronize(s));
  *out_total = total;
  return SV_OK;
}

extern "C" int sv_kmap_pairs_emit(const int32_t* nbr, int64_t n, int kvol, int32_t* offsets,
                                  int32_t* pair_src, int32_t* pair_dst, int64_t total,
                                  void* workspace, size_t workspace_bytes, int32_t* status,
                                  sv_stream_t stream) {
  if (n < 0 || kvol < 1 || kvol > 65535 || total < 0)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_pairs_emit: bad sizes");
  if (!offsets) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_pairs_emit: null offsets");
  cudaStream_t s = to_stream(stream);
  if (n == 0) {
    SV_CUDA_TRY(cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (kvol + 1), s));
    return SV_OK;
  }
  if (!nbr || (total > 0 && (!pair_src || !pair_dst)))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_pairs_emit: null pointer");
  if (!workspace || workspace_bytes < sv_kmap_pairs_workspace_bytes(n, kvol))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_kmap_pairs_emit: workspace too small");
  const int64_t tiles = pair_tiles(n), entries = tiles * kvol;
  const size_t eb = align_up((size_t)entries * 4, 256);
  const int32_t* incl = reinterpret_cast<const int32_t*>(static_cast<uint8_t*>(workspace) + eb);
  pairs_emit_kernel<<<dim3((unsigned)tiles, (unsigned)kvol), PAIR_THREADS, 0, s>>>(
      nbr, n, kvol, incl, total, pair_src, pair_dst, status);
  SV_LAUNCH_CHECK();
  pair_offsets_kernel<<<(kvol + 1 + 127) / 128, 128, 0, s>>>(incl, tiles, kvol, offsets);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

// Defined in wgrad_tc.cu.
extern "C" int sv_conv3d_wgrad_tc_supported(int cin, int cout, int kvol, int dtype);
extern "C" int sv_conv3d_wgrad_tc(const void* features, const void* dout, int cin, int cout,
                                  int kvol, const int32_t* offsets, const int32_t* pair_src,
                                  const int32_t* pair_dst, int dtype, void* dweight,
                                  void* workspace, size_t workspace_bytes, int32_t* status,
                                  sv_stream_t stream);

static int wgrad_simt(const void* features, const void* dout, int cin, int cout, int kvol,
                      const int32_t* offsets, const int32_t* pair_src, const int32_t* pair_dst,
                      int dtype, void* dweight, sv_stream_t stream) {
  if (!valid_dtype(dtype)) SV_FAIL(SV_ERR_BAD_DTYPE, "wgrad: unknown dtype");
  if (cin < 0 || cout < 0 || kvol < 1 || kvol > 65535)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "wgrad: bad sizes");
  if ((int64_t)cin * cout == 0) return SV_OK;
  if (!offsets || !dweight) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "wgrad: null pointer");
  cudaStream_t s = to_stream(stream);
  const dim3 grid((unsigned)((cin + WG_T - 1) / WG_T), (unsigned)((cout + WG_T - 1) / WG_T),
                  (unsigned)kvol);
  if (grid.y > 65535) SV_FAIL(SV_ERR_UNSUPPORTED, "wgrad: too many output channels");
  if (dtype == SV_FLOAT32)
    wgrad_simt_kernel<float><<<grid, 256, 0, s>>>(
        static_cast<const float*>(features), static_cast<const float*>(dout), cin, cout, kvol,
        offsets, pair_src, pair_dst, static_cast<float*>(dweight));
  else if (dtype == SV_FLOAT16)
    wgrad_simt_kernel<__half><<<grid, 256, 0, s>>>(
        static_cast<const __half*>(features), static_cast<const __half*>(dout), cin, cout, kvol,
        offsets, pair_src, pair_dst, static_cast<__half*>(dweight));
  else
    wgrad_simt_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(features), static_cast<const __nv_bfloat16*>(dout), cin,
        cout, kvol, offsets, pair_src, pair_dst, static_cast<__nv_bfloat16*>(dweight));
  SV_LAUNCH_CHECK();
  return SV_OK;
}

extern "C" size_t sv_conv3d_wgrad_workspace_bytes(int cin, int cout, int kvol, int dtype,
                                                  int algo) {
  if (algo == SV_CONV_SIMT) return 0;
  return sv_conv3d_wgrad_tc_supported(cin, cout, kvol, dtype) ? 256 : 0;
}

extern "C" int sv_conv3d_wgrad(const void* features, const void* dout, int cin, int cout,
                               int kvol, const int32_t* offsets, const int32_t* pair_src,
                               const int32_t* pair_dst, int dtype, void* dweight, int algo,
                               void* workspace, size_t workspace_bytes, int32_t* status,
                               sv_stream_t stream) {
  if (algo != SV_CONV_AUTO && algo != SV_CONV_SIMT && algo != SV_CONV_TCGEN05)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_wgrad: unknown algorithm");
  const bool tc = algo != SV_CONV_SIMT && sv_conv3d_wgrad_tc_supported(cin, cout, kvol, dtype) &&
                  aligned16(features) && aligned16(dout) && aligned16(dweight);
  if (algo == SV_CONV_TCGEN05 && !tc)
    SV_FAIL(SV_ERR_UNSUPPORTED,
            "tcgen05 weight gradient needs fp16/bf16, Cin % 64 == 0, Cout % 128 == 0 and "
            "16-byte aligned operands");
  if (tc)
    return sv_conv3d_wgrad_tc(features, dout, cin, cout, kvol, offsets, pair_src, pair_dst,
                              dtype, dweight, workspace, workspace_bytes, status, stream);
  return wgrad_simt(features, dout, cin, cout, kvol, offsets, pair_src, pair_dst, dtype, dweight,
                    stream);
}

extern "C" size_t sv_conv3d_dbias_workspace_bytes(int64_t n, int channels) {
  if (n <= 0 || channels <= 0) return 256;
  return align_up((size_t)((n + DB_ROWS - 1) / DB_ROWS) * channels * 4, 256);
}

extern "C" int sv_conv3d_dbias(const void* dout, int64_t n, int channels, int dtype, void* dbias,
                               void* workspace, size_t workspace_bytes, sv_stream_t stream) {
  if (!valid_dtype(dtype)) SV_FAIL(SV_ERR_BAD_DTYPE, "dbias: unknown dtype");
  if (n < 0 || channels < 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "dbias: negative size");
  if (channels == 0) return SV_OK;
  if (!dbias) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "dbias: null output");
  cudaStream_t s = to_stream(stream);
  const int64_t parts = n > 0 ? (n + DB_ROWS - 1) / DB_ROWS : 0;
  if (parts > 65535) SV_FAIL(SV_ERR_UNSUPPORTED, "dbias: more than 65535 * 1024 rows");
  if (parts > 0 && (!dout || !workspace || workspace_bytes < sv_conv3d_dbias_workspace_bytes(n, channels)))
    SV_FAIL(SV_ERR_WORKSPACE, "dbias: workspace too small or null input");
  float* partial = static_cast<float*>(workspace);
  const unsigned cb = (unsigned)((channels + 255) / 256);
  if (dtype == SV_FLOAT32) {
    if (parts) dbias_partial_kernel<float><<<dim3(cb, (unsigned)parts), 256, 0, s>>>(
        static_cast<const float*>(dout), n, channels, partial);
    dbias_final_kernel<float><<<cb, 256, 0, s>>>(partial, (int)parts, channels,
                                                 static_cast<float*>(dbias));
  } else if (dtype == SV_FLOAT16) {
    if (parts) dbias_partial_kernel<__half><<<dim3(cb, (unsigned)parts), 256, 0, s>>>(
        static_cast<const __half*>(dout), n, channels, partial);
    dbias_final_kernel<__half><<<cb, 256, 0, s>>>(partial, (int)parts, channels,
                                                  static_cast<__half*>(dbias));
  } else {
    if (parts) dbias_partial_kernel<__nv_bfloat16><<<dim3(cb, (unsigned)parts), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(dout), n, channels, partial);
    dbias_final_kernel<__nv_bfloat16><<<cb, 256, 0, s>>>(partial, (int)parts, channels,
                                                         static_cast<__nv_bfloat16*>(dbias));
  }
  SV_LAUNCH_CHECK();
  return SV_OK;
}

extern "C" int sv_weight_flip_transpose(const void* w_oki, int cout, int kvol, int cin, int dtype,
                                        void* out, sv_stream_t stream) {
  if (!valid_dtype(dtype)) SV_FAIL(SV_ERR_BAD_DTYPE, "sv_weight_flip_transpose: unknown dtype");
  if (cout < 0 || cin < 0 || kvol < 1 || kvol > 65535)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_weight_flip_transpose: bad sizes");
  if ((int64_t)cout * cin == 0) return SV_OK;
  if (!w_oki || !out) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_weight_flip_transpose: null pointer");
  if ((cout + 31) / 32 > 65535) SV_FAIL(SV_ERR_UNSUPPORTED, "weight too large to transform");
  cudaStream_t s = to_stream(stream);
  const dim3 block(32, 8), grid((unsigned)((cin + 31) / 32), (unsigned)((cout + 31) / 32),
                                (unsigned)kvol);
  if (dtype == SV_FLOAT32)
    flip_transpose_kernel<uint32_t><<<grid, block, 0, s>>>(
        static_cast<const uint32_t*>(w_oki), cout, kvol, cin, static_cast<uint32_t*>(out));
  else
    flip_transpose_kernel<uint16_t><<<grid, block, 0, s>>>(
        static_cast<const uint16_t*>(w_oki), cout, kvol, cin, static_cast<uint16_t*>(out));
  SV_LAUNCH_CHECK();
  return SV_OK;
}
