// Stride-f sparse downsample / upsample.
//
// Restates sparse_downsample (src/mlx_diffuser/layers/sparse.py:245-284) and sparse_upsample
// (:287-295):
//  * coordinates: spatial columns floor-divided by f, then np.unique(axis=0,
//    return_inverse=True). np.unique orders rows lexicographically as signed int32 tuples; here
//    every column is offset by its minimum and the four fields are packed, most significant
//    first, into one 64-bit key, whose unsigned order is that lexicographic order. A stable
//    radix sort of (key, row) gives the unique rows (segment heads), the inverse, and the fine
//    rows of each coarse row in their original order;
//  * features: fp32 sums over each segment in fine-row order (np.add.at's order), divided by
//    count + 1 -- the reference's zero-initialised include_self mean (:264-266);
//  * upsample: a row gather through the inverse.
#include <algorithm>

#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include "common.cuh"

namespace sv {
namespace {

__device__ __forceinline__ int floordiv(int v, int f) {
  int q = v / f;
  if ((v % f) != 0 && (v < 0)) --q;
  return q;
}

// bounds[0..3] = min of (b, c1//f, c2//f, c3//f); bounds[4..7] = max.
__global__ void init_bounds_kernel(int32_t* bounds) {
  if (threadIdx.x < 4) bounds[threadIdx.x] = INT32_MAX;
  else if (threadIdx.x < 8) bounds[threadIdx.x] = INT32_MIN;
}

__global__ void bounds_kernel(const int4* __restrict__ coords, int64_t n, int f,
                              int32_t* bounds) {
  int mn[4] = {INT32_MAX, INT32_MAX, INT32_MAX, INT32_MAX};
  int mx[4] = {INT32_MIN, INT32_MIN, INT32_MIN, INT32_MIN};
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int4 c = __ldg(&coords[i]);
    const int v[4] = {c.x, floordiv(c.y, f), floordiv(c.z, f), floordiv(c.w, f)};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      mn[j] = min(mn[j], v[j]);
      mx[j] = max(mx[j], v[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    for (int o = 16; o > 0; o >>= 1) {
      mn[j] = min(mn[j], __shfl_xor_sync(0xffffffffu, mn[j], o));
      mx[j] = max(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], o));
    }
  }
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      atomicMin(&bounds[j], mn[j]);
      atomicMax(&bounds[4 + j], mx[j]);
    }
  }
}

struct Packing {
  int32_t lo[4];     // minimum of each field
  int shift[4];      // bit position of each field
  uint64_t mask[4];  // width mask of each field
};

__global__ void pack_keys_kernel(const int4* __restrict__ coords, int64_t n, int f, Packing pk,
                                 uint64_t* __restrict__ keys, int32_t* __restrict__ rows) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int4 c = __ldg(&coords[i]);
  const int v[4] = {c.x, floordiv(c.y, f), floordiv(c.z, f), floordiv(c.w, f)};
  uint64_t key = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    key |= (uint64_t)(uint32_t)((int64_t)v[j] - (int64_t)pk.lo[j]) << pk.shift[j];
  keys[i] = key;
  rows[i] = (int32_t)i;
}

__global__ void heads_kernel(const uint64_t* __restrict__ keys, int64_t n,
                             int32_t* __restrict__ heads) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  heads[j] = (j == 0 || keys[j] != keys[j - 1]) ? 1 : 0;
}

__global__ void emit_kernel(const uint64_t* __restrict__ keys, const int32_t* __restrict__ rows,
                            const int32_t* __restrict__ heads, const int32_t* __restrict__ seg,
                            int64_t n, Packing pk, int4* __restrict__ out_coords,
                            int32_t* __restrict__ inverse, int32_t* __restrict__ seg_offsets) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const int32_t s = seg[j] - 1;
  inverse[rows[j]] = s;
  if (heads[j]) {
    seg_offsets[s] = (int32_t)j;
    const uint64_t key = keys[j];
    int v[4];
#pragma unroll
    for (int f = 0; f < 4; ++f)
      v[f] = (int)((int64_t)pk.lo[f] + (int64_t)((key >> pk.shift[f]) & pk.mask[f]));
    out_coords[s] = make_int4(v[0], v[1], v[2], v[3]);
  }
  if (j == n - 1) seg_offsets[s + 1] = (int32_t)n;
}

template <typename T, int VEC>
__global__ void pool_kernel(const T* __restrict__ feat, int channels,
                            const int32_t* __restrict__ sorted_rows,
                            const int32_t* __restrict__ seg, int64_t m, T* __restrict__ out) {
  // One thread per (coarse row, VEC channels).
  const int groups = channels / VEC;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= m * groups) return;
  const int64_t j = t / groups;
  const int g = (int)(t - j * groups);
  const int32_t s0 = __ldg(&seg[j]), s1 = __ldg(&seg[j + 1]);
  float acc[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
  for (int32_t r = s0; r < s1; ++r) {
    const T* src = feat + (int64_t)__ldg(&sorted_rows[r]) * channels + g * VEC;
    if constexpr (VEC * sizeof(T) == 16) {
      uint4 raw = __ldg(reinterpret_cast<const uint4*>(src));
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[v] += to_f32(e[v]);
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[v] += to_f32(src[v]);
    }
  }
  const float denom = (float)(s1 - s0) + 1.0f;
  T* dst = out + j * channels + g * VEC;
  if constexpr (VEC * sizeof(T) == 16) {
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int v = 0; v < VEC; ++v) e[v] = from_f32<T>(acc[v] / denom);
    *reinterpret_cast<uint4*>(dst) = raw;
  } else {
#pragma unroll
    for (int v = 0; v < VEC; ++v) dst[v] = from_f32<T>(acc[v] / denom);
  }
}

template <int BYTES>
__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, int64_t m, int row_bytes,
                                   const int32_t* __restrict__ index, int64_t n,
                                   uint8_t* __restrict__ dst, int32_t* status) {
  // One thread per (fine row, BYTES-wide chunk).
  const int chunks = row_bytes / BYTES;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n * chunks) return;
  const int64_t i = t / chunks;
  const int c = (int)(t - i * chunks);
  int64_t r = __ldg(&index[i]);
  if (r < 0 || r >= m) {
    report(status, SV_DEVICE_BAD_INDEX);
    r = -1;
  }
  uint8_t* d = dst + i * row_bytes + (int64_t)c * BYTES;
  if constexpr (BYTES == 16) {
    *reinterpret_cast<uint4*>(d) =
        r >= 0 ? __ldg(reinterpret_cast<const uint4*>(src + r * row_bytes + (int64_t)c * BYTES))
               : make_uint4(0, 0, 0, 0);
  } else {
    *d = r >= 0 ? src[r * row_bytes + c] : (uint8_t)0;
  }
}

size_t sort_bytes(int64_t n) {
  size_t b = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, b, (const uint64_t*)nullptr, (uint64_t*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, (int)n, 0, 64);
  return b;
}

size_t scan_bytes(int64_t n) {
  size_t b = 0;
  cub::DeviceScan::InclusiveSum(nullptr, b, (const int32_t*)nullptr, (int32_t*)nullptr, (int)n);
  return b;
}

int bits_for(int64_t range) {
  int b = 0;
  while (b < 63 && (range >> b) != 0) ++b;
  return b;
}

template <typename T>
int launch_pool(const void* f, int channels, const int32_t* rows, const int32_t* seg, int64_t m,
                void* out, cudaStream_t s) {
  constexpr int V16 = 16 / sizeof(T);
  const bool vec = channels % V16 == 0 && aligned16(f) && aligned16(out);
  const int per = vec ? V16 : 1;
  const int64_t threads_total = m * (channels / per);
  const unsigned blocks = (unsigned)((threads_total + 255) / 256);
  if (blocks == 0) return SV_OK;
  if (vec)
    pool_kernel<T, V16><<<blocks, 256, 0, s>>>(static_cast<const T*>(f), channels, rows, seg, m,
                                               static_cast<T*>(out));
  else
    pool_kernel<T, 1><<<blocks, 256, 0, s>>>(static_cast<const T*>(f), channels, rows, seg, m,
                                             static_cast<T*>(out));
  SV_LAUNCH_CHECK();
  return SV_OK;
}

}  // namespace
}  // namespace sv

using namespace sv;

extern "C" size_t sv_downsample_workspace_bytes(int64_t n) {
  if (n <= 0) return 256;
  const size_t k = align_up((size_t)n * 8, 256);
  const size_t r = align_up((size_t)n * 4, 256);
  // keys, keys_sorted, rows, heads, seg, bounds, cub scratch
  return 2 * k + 3 * r + 256 + align_up(std::max(sort_bytes(n), scan_bytes(n)), 256);
}

extern "C" int sv_downsample_coords(const int32_t* coords, int64_t n, int factor,
                                    int32_t* out_coords, int32_t* inverse, int32_t* sorted_rows,
                                    int32_t* seg_offsets, int64_t* out_m, void* workspace,
                                    size_t workspace_bytes, sv_stream_t stream) {
  if (factor < 1) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "factor must be positive");
  if (n < 0 || out_m == nullptr)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_downsample_coords: bad arguments");
  *out_m = 0;
  if (n == 0) return SV_OK;
  if (n > INT32_MAX - 1)
    SV_FAIL(SV_ERR_UNSUPPORTED, "sv_downsample_coords: more than 2^31-2 rows");
  if (!coords || !out_coords || !inverse || !sorted_rows || !seg_offsets)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_downsample_coords: null pointer");
  if (!aligned16(coords) || !aligned16(out_coords))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "coords must be 16-byte aligned");
  if (workspace == nullptr || workspace_bytes < sv_downsample_workspace_bytes(n))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_downsample_coords: workspace too small");
  cudaStream_t s = to_stream(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t kb = align_up((size_t)n * 8, 256), rb = align_up((size_t)n * 4, 256);
  uint64_t* keys = reinterpret_cast<uint64_t*>(ws);
  uint64_t* keys_sorted = reinterpret_cast<uint64_t*>(ws + kb);
  int32_t* rows = reinterpret_cast<int32_t*>(ws + 2 * kb);
  int32_t* heads = reinterpret_cast<int32_t*>(ws + 2 * kb + rb);
  int32_t* seg = reinterpret_cast<int32_t*>(ws + 2 * kb + 2 * rb);
  int32_t* bounds = reinterpret_cast<int32_t*>(ws + 2 * kb + 3 * rb);
  void* tmp = ws + 2 * kb + 3 * rb + 256;
  size_t tmp_bytes = workspace_bytes - (2 * kb + 3 * rb + 256);

  const int4* c4 = reinterpret_cast<const int4*>(coords);
  init_bounds_kernel<<<1, 32, 0, s>>>(bounds);
  SV_LAUNCH_CHECK();
  const unsigned bb = (unsigned)std::min<int64_t>((n + 255) / 256, 4 * num_sms());
  bounds_kernel<<<bb, 256, 0, s>>>(c4, n, factor, bounds);
  SV_LAUNCH_CHECK();
  int32_t hb[8];
  SV_CUDA_TRY(cudaMemcpyAsync(hb, bounds, sizeof(hb), cudaMemcpyDeviceToHost, s));
  SV_CUDA_TRY(cudaStreamSynchronize(s));
  Packing pk;
  int width[4];
  int total = 0;
  for (int j = 3; j >= 0; --j) {
    pk.lo[j] = hb[j];
    width[j] = bits_for((int64_t)hb[4 + j] - (int64_t)hb[j]);
    pk.shift[j] = total;
    total += width[j];
  }
  if (total > 64)
    SV_FAIL(SV_ERR_UNSUPPORTED,
            "sv_downsample_coords: coordinate ranges need more than 64 key bits");
  for (int j = 0; j < 4; ++j) pk.mask[j] = width[j] >= 64 ? ~0ull : ((1ull << width[j]) - 1);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  pack_keys_kernel<<<blocks, 256, 0, s>>>(c4, n, factor, pk, keys, rows);
  SV_LAUNCH_CHECK();
  SV_CUDA_TRY(cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, keys, keys_sorted, rows,
                                              sorted_rows, (int)n, 0, std::max(total, 1), s));
  heads_kernel<<<blocks, 256, 0, s>>>(keys_sorted, n, heads);
  SV_LAUNCH_CHECK();
  size_t scan_tmp = tmp_bytes;
  SV_CUDA_TRY(cub::DeviceScan::InclusiveSum(tmp, scan_tmp, heads, seg, (int)n, s));
  emit_kernel<<<blocks, 256, 0, s>>>(keys_sorted, sorted_rows, heads, seg, n, pk,
                                     reinterpret_cast<int4*>(out_coords), inverse, seg_offsets);
  SV_LAUNCH_CHECK();
  int32_t m32 = 0;
  SV_CUDA_TRY(cudaMemcpyAsync(&m32, seg + (n - 1), sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  SV_CUDA_TRY(cudaStreamSynchronize(s));
  *out_m = m32;
  return SV_OK;
}

extern "C" int sv_downsample_features(const void* features, int64_t n, int channels, int dtype,
                                      const int32_t* sorted_rows, const int32_t* seg_offsets,
                                      int64_t m, void* out, sv_stream_t stream) {
  if (n < 0 || m < 0 || channels < 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "negative size");
  if (dtype != SV_FLOAT32 && dtype != SV_FLOAT16 && dtype != SV_BFLOAT16)
    SV_FAIL(SV_ERR_BAD_DTYPE, "sv_downsample_features: unknown dtype");
  if (m == 0 || channels == 0) return SV_OK;
  if (!features || !sorted_rows || !seg_offsets || !out)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_downsample_features: null pointer");
  cudaStream_t s = to_stream(stream);
  if (dtype == SV_FLOAT32)
    return launch_pool<float>(features, channels, sorted_rows, seg_offsets, m, out, s);
  if (dtype == SV_FLOAT16)
    return launch_pool<__half>(features, channels, sorted_rows, seg_offsets, m, out, s);
  return launch_pool<__nv_bfloat16>(features, channels, sorted_rows, seg_offsets, m, out, s);
}

extern "C" int sv_upsample_features(const void* coarse, int64_t m, int channels, int dtype,
                                    const int32_t* inverse, int64_t n, void* out,
                                    int32_t* status, sv_stream_t stream) {
  if (n < 0 || m < 0 || channels < 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "negative size");
  if (dtype != SV_FLOAT32 && dtype != SV_FLOAT16 && dtype != SV_BFLOAT16)
    SV_FAIL(SV_ERR_BAD_DTYPE, "sv_upsample_features: unknown dtype");
  if (n == 0 || channels == 0) return SV_OK;
  if (!coarse || !inverse || !out)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_upsample_features: null pointer");
  cudaStream_t s = to_stream(stream);
  const int row_bytes = channels * dtype_size(dtype);
  const bool vec = row_bytes % 16 == 0 && aligned16(coarse) && aligned16(out);
  const int per = vec ? 16 : 1;
  const int64_t total = n * (row_bytes / per);
  const unsigned blocks = (unsigned)((total + 255) / 256);
  if (vec)
    gather_rows_kernel<16><<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(coarse), m,
                                                  row_bytes, inverse, n,
                                                  static_cast<uint8_t*>(out), status);
  else
    gather_rows_kernel<1><<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(coarse), m,
                                                 row_bytes, inverse, n,
                                                 static_cast<uint8_t*>(out), status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}
