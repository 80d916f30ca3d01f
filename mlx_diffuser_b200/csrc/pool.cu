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
//
// The same keyed sort groups voxels into attention windows, _attention_groups
// (src/mlx_diffuser/layers/sparse.py:321-342): key (b, (c + shift) // window) per spatial
// column, or (b) alone without a window. The reference collects row indices into a dict keyed by
// that tuple, so groups come out in the order of their first row and each group's rows
// ascending; here a second stable sort of the key-sorted rows by their segment's first row
// gives that order.
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

// The key fields of a row: (b, (c1 + shift0) // f, (c2 + shift1) // f, (c3 + shift2) // f),
// with int32 wrap-around on the addition (NumPy int32 arithmetic), or (b, 0, 0, 0) when the
// spatial columns do not take part.
struct KeySpec {
  int f;
  int shift[3];
  int spatial;
};

__device__ __forceinline__ void key_fields(const int4& c, const KeySpec& ks, int v[4]) {
  v[0] = c.x;
  if (ks.spatial) {
    v[1] = floordiv((int)((uint32_t)c.y + (uint32_t)ks.shift[0]), ks.f);
    v[2] = floordiv((int)((uint32_t)c.z + (uint32_t)ks.shift[1]), ks.f);
    v[3] = floordiv((int)((uint32_t)c.w + (uint32_t)ks.shift[2]), ks.f);
  } else {
    v[1] = v[2] = v[3] = 0;
  }
}

__global__ void bounds_kernel(const int4* __restrict__ coords, int64_t n, KeySpec ks,
                              int32_t* bounds) {
  int mn[4] = {INT32_MAX, INT32_MAX, INT32_MAX, INT32_MAX};
  int mx[4] = {INT32_MIN, INT32_MIN, INT32_MIN, INT32_MIN};
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int4 c = __ldg(&coords[i]);
    int v[4];
    key_fields(c, ks, v);
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

__global__ void pack_keys_kernel(const int4* __restrict__ coords, int64_t n, KeySpec ks,
                                 Packing pk, uint64_t* __restrict__ keys,
                                 int32_t* __restrict__ rows) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int4 c = __ldg(&coords[i]);
  int v[4];
  key_fields(c, ks, v);
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

// Workspace regions shared by the downsample and the window grouping.
struct KeySort {
  uint64_t* keys;
  uint64_t* keys_sorted;
  int32_t* rows;
  int32_t* heads;
  int32_t* seg;  // inclusive scan of heads: segment id + 1 at each sorted position
  int32_t* bounds;
  void* tmp;
  size_t tmp_bytes;
  Packing pk;
  int bits;
};

size_t key_sort_bytes(int64_t n) {
  const size_t k = align_up((size_t)n * 8, 256);
  const size_t r = align_up((size_t)n * 4, 256);
  // keys, keys_sorted, rows, heads, seg, bounds, cub scratch
  return 2 * k + 3 * r + 256 + align_up(std::max(sort_bytes(n), scan_bytes(n)), 256);
}

// Stable sort of the rows by their packed key (KeySpec), then segment heads and ids. Reads the
// key bounds back to size the packing, so it synchronises the stream once.
int key_sort(const int4* c4, int64_t n, const KeySpec& ks, uint8_t* ws, size_t ws_bytes,
             int32_t* sorted_rows, KeySort* out, cudaStream_t s) {
  const size_t kb = align_up((size_t)n * 8, 256), rb = align_up((size_t)n * 4, 256);
  KeySort& k = *out;
  k.keys = reinterpret_cast<uint64_t*>(ws);
  k.keys_sorted = reinterpret_cast<uint64_t*>(ws + kb);
  k.rows = reinterpret_cast<int32_t*>(ws + 2 * kb);
  k.heads = reinterpret_cast<int32_t*>(ws + 2 * kb + rb);
  k.seg = reinterpret_cast<int32_t*>(ws + 2 * kb + 2 * rb);
  k.bounds = reinterpret_cast<int32_t*>(ws + 2 * kb + 3 * rb);
  k.tmp = ws + 2 * kb + 3 * rb + 256;
  k.tmp_bytes = align_up(std::max(sort_bytes(n), scan_bytes(n)), 256);
  if (ws_bytes < 2 * kb + 3 * rb + 256 + k.tmp_bytes)
    SV_FAIL(SV_ERR_WORKSPACE, "key sort: workspace too small");

  init_bounds_kernel<<<1, 32, 0, s>>>(k.bounds);
  SV_LAUNCH_CHECK();
  const unsigned bb = (unsigned)std::min<int64_t>((n + 255) / 256, 4 * num_sms());
  bounds_kernel<<<bb, 256, 0, s>>>(c4, n, ks, k.bounds);
  SV_LAUNCH_CHECK();
  int32_t hb[8];
  SV_CUDA_TRY(cudaMemcpyAsync(hb, k.bounds, sizeof(hb), cudaMemcpyDeviceToHost, s));
  SV_CUDA_TRY(cudaStreamSynchronize(s));
  int width[4];
  int total = 0;
  for (int j = 3; j >= 0; --j) {
    k.pk.lo[j] = hb[j];
    width[j] = bits_for((int64_t)hb[4 + j] - (int64_t)hb[j]);
    k.pk.shift[j] = total;
    total += width[j];
  }
  if (total > 64) SV_FAIL(SV_ERR_UNSUPPORTED, "coordinate ranges need more than 64 key bits");
  for (int j = 0; j < 4; ++j) k.pk.mask[j] = width[j] >= 64 ? ~0ull : ((1ull << width[j]) - 1);
  k.bits = std::max(total, 1);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  pack_keys_kernel<<<blocks, 256, 0, s>>>(c4, n, ks, k.pk, k.keys, k.rows);
  SV_LAUNCH_CHECK();
  size_t t = k.tmp_bytes;
  SV_CUDA_TRY(cub::DeviceRadixSort::SortPairs(k.tmp, t, k.keys, k.keys_sorted, k.rows,
                                              sorted_rows, (int)n, 0, k.bits, s));
  heads_kernel<<<blocks, 256, 0, s>>>(k.keys_sorted, n, k.heads);
  SV_LAUNCH_CHECK();
  t = k.tmp_bytes;
  SV_CUDA_TRY(cub::DeviceScan::InclusiveSum(k.tmp, t, k.heads, k.seg, (int)n, s));
  return SV_OK;
}

// seg_start[s] = sorted position of segment s's head.
__global__ void seg_start_kernel(const int32_t* __restrict__ heads,
                                 const int32_t* __restrict__ seg, int64_t n,
                                 int32_t* __restrict__ seg_start) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  if (heads[j]) seg_start[seg[j] - 1] = (int32_t)j;
}

// key2[p] = the first (smallest) row of sorted position p's segment: segments hold their rows
// in ascending order, so that is the row at the segment's head.
__global__ void group_key_kernel(const int32_t* __restrict__ sorted_rows,
                                 const int32_t* __restrict__ seg,
                                 const int32_t* __restrict__ seg_start, int64_t n,
                                 uint32_t* __restrict__ key2) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  key2[j] = (uint32_t)sorted_rows[seg_start[seg[j] - 1]];
}

__global__ void heads32_kernel(const uint32_t* __restrict__ keys, int64_t n,
                               int32_t* __restrict__ heads) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  heads[j] = (j == 0 || keys[j] != keys[j - 1]) ? 1 : 0;
}

__global__ void group_offsets_kernel(const int32_t* __restrict__ heads,
                                     const int32_t* __restrict__ seg, int64_t n,
                                     int32_t* __restrict__ offsets) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  if (heads[j]) offsets[seg[j] - 1] = (int32_t)j;
  if (j == n - 1) offsets[seg[j]] = (int32_t)n;
}

}  // namespace
}  // namespace sv

using namespace sv;

extern "C" size_t sv_downsample_workspace_bytes(int64_t n) {
  if (n <= 0) return 256;
  return key_sort_bytes(n);
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
  KeySpec ks;
  ks.f = factor;
  ks.shift[0] = ks.shift[1] = ks.shift[2] = 0;
  ks.spatial = 1;
  KeySort k;
  int rc = key_sort(reinterpret_cast<const int4*>(coords), n, ks,
                    static_cast<uint8_t*>(workspace), workspace_bytes, sorted_rows, &k, s);
  if (rc != SV_OK) return rc;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  emit_kernel<<<blocks, 256, 0, s>>>(k.keys_sorted, sorted_rows, k.heads, k.seg, n, k.pk,
                                     reinterpret_cast<int4*>(out_coords), inverse, seg_offsets);
  SV_LAUNCH_CHECK();
  int32_t m32 = 0;
  SV_CUDA_TRY(cudaMemcpyAsync(&m32, k.seg + (n - 1), sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  SV_CUDA_TRY(cudaStreamSynchronize(s));
  *out_m = m32;
  return SV_OK;
}

extern "C" size_t sv_window_groups_workspace_bytes(int64_t n) {
  if (n <= 0) return 256;
  const size_t r = align_up((size_t)n * 4, 256);
  // key sort + sorted rows + segment starts + group keys (unsorted, sorted)
  return key_sort_bytes(n) + 4 * r;
}

extern "C" int sv_window_groups(const int32_t* coords, int64_t n, int window,
                                const int32_t shift[3], int32_t* perm, int32_t* offsets,
                                int64_t* out_groups, void* workspace, size_t workspace_bytes,
                                sv_stream_t stream) {
  if (n < 0 || out_groups == nullptr)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_window_groups: bad arguments");
  if (window < 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "window size must be positive (0: none)");
  *out_groups = 0;
  if (n == 0) return SV_OK;
  if (n > INT32_MAX - 1) SV_FAIL(SV_ERR_UNSUPPORTED, "sv_window_groups: more than 2^31-2 rows");
  if (!coords || !perm || !offsets)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_window_groups: null pointer");
  if (!aligned16(coords)) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "coords must be 16-byte aligned");
  if (workspace == nullptr || workspace_bytes < sv_window_groups_workspace_bytes(n))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_window_groups: workspace too small");
  cudaStream_t s = to_stream(stream);
  KeySpec ks;
  ks.f = window > 0 ? window : 1;
  for (int j = 0; j < 3; ++j) ks.shift[j] = (window > 0 && shift) ? shift[j] : 0;
  ks.spatial = window > 0 ? 1 : 0;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t base = key_sort_bytes(n), rb = align_up((size_t)n * 4, 256);
  int32_t* sorted_rows = reinterpret_cast<int32_t*>(ws + base);
  int32_t* seg_start = reinterpret_cast<int32_t*>(ws + base + rb);
  uint32_t* key2 = reinterpret_cast<uint32_t*>(ws + base + 2 * rb);
  uint32_t* key2_sorted = reinterpret_cast<uint32_t*>(ws + base + 3 * rb);
  KeySort k;
  int rc = key_sort(reinterpret_cast<const int4*>(coords), n, ks, ws, base, sorted_rows, &k, s);
  if (rc != SV_OK) return rc;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  seg_start_kernel<<<blocks, 256, 0, s>>>(k.heads, k.seg, n, seg_start);
  SV_LAUNCH_CHECK();
  group_key_kernel<<<blocks, 256, 0, s>>>(sorted_rows, k.seg, seg_start, n, key2);
  SV_LAUNCH_CHECK();
  // groups in the order of their first row (dict insertion order), rows ascending inside
  size_t t = k.tmp_bytes;
  SV_CUDA_TRY(cub::DeviceRadixSort::SortPairs(k.tmp, t, key2, key2_sorted, sorted_rows, perm,
                                              (int)n, 0, std::max(bits_for(n), 1), s));
  heads32_kernel<<<blocks, 256, 0, s>>>(key2_sorted, n, k.heads);
  SV_LAUNCH_CHECK();
  t = k.tmp_bytes;
  SV_CUDA_TRY(cub::DeviceScan::InclusiveSum(k.tmp, t, k.heads, k.seg, (int)n, s));
  group_offsets_kernel<<<blocks, 256, 0, s>>>(k.heads, k.seg, n, offsets);
  SV_LAUNCH_CHECK();
  int32_t g32 = 0;
  SV_CUDA_TRY(cudaMemcpyAsync(&g32, k.seg + (n - 1), sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  SV_CUDA_TRY(cudaStreamSynchronize(s));
  *out_groups = g32;
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
