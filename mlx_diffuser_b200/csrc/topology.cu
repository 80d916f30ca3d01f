// Topology producers around the sparse-voxel path:
//
//  * occupancy -> coordinates: TrellisSparseStructureDecoder.occupied_coordinates
//    (src/mlx_diffuser/models/trellis.py:278-285) takes np.argwhere(logits > threshold) of the
//    decoder's [B, D, H, W] occupancy logits on the host. Here it is an ordered stream
//    compaction: a count pass (one count per 1024-element tile), a scan of the tile counts, and
//    an emit pass that writes (b, d, h, w) rows in row-major order, which is argwhere's order.
//    The comparison is made in the logits' type against the threshold rounded to that type
//    (MLX promotes a Python float scalar to the array's floating type); NaN is never occupied.
//  * sparse_subdivide (src/mlx_diffuser/layers/sparse.py:298-318): every row becomes eight
//    rows, child j = 4z + 2y + x at (b, 2*c1 + z, 2*c2 + y, 2*c3 + x), each carrying its
//    parent's feature row. int32 arithmetic wraps like MLX's.
#include <cub/device/device_scan.cuh>

#include "common.cuh"

namespace sv {
namespace {

constexpr int OCC_THREADS = 256;
constexpr int OCC_ITERS = 4;
constexpr int OCC_TILE = OCC_THREADS * OCC_ITERS;  // logical elements per tile

struct Grid4 {
  int64_t shape[4];
  int64_t stride[4];  // in elements
  int64_t total;
  int contiguous;
};

__device__ __forceinline__ int64_t grid_offset(const Grid4& g, int64_t e) {
  if (g.contiguous) return e;
  const int64_t w = e % g.shape[3];
  int64_t r = e / g.shape[3];
  const int64_t h = r % g.shape[2];
  r /= g.shape[2];
  const int64_t d = r % g.shape[1];
  const int64_t b = r / g.shape[1];
  return b * g.stride[0] + d * g.stride[1] + h * g.stride[2] + w * g.stride[3];
}

template <typename T>
__device__ __forceinline__ bool occupied(const T* __restrict__ logits, const Grid4& g, int64_t e,
                                         float thr) {
  return e < g.total && to_f32(logits[grid_offset(g, e)]) > thr;
}

template <typename T>
__global__ void __launch_bounds__(OCC_THREADS)
    occ_count_kernel(const T* __restrict__ logits, Grid4 g, float thr,
                     int32_t* __restrict__ tile_counts) {
  __shared__ int s_warp[OCC_THREADS / 32];
  const int64_t base = (int64_t)blockIdx.x * OCC_TILE;
  int cnt = 0;
#pragma unroll
  for (int i = 0; i < OCC_ITERS; ++i)
    cnt += occupied(logits, g, base + i * OCC_THREADS + threadIdx.x, thr) ? 1 : 0;
  cnt = __reduce_add_sync(0xffffffffu, cnt);
  if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
#pragma unroll
    for (int w = 0; w < OCC_THREADS / 32; ++w) t += s_warp[w];
    tile_counts[blockIdx.x] = t;
  }
}

template <typename T>
__global__ void __launch_bounds__(OCC_THREADS)
    occ_emit_kernel(const T* __restrict__ logits, Grid4 g, float thr,
                    const int32_t* __restrict__ tile_incl, int64_t m, int4* __restrict__ out,
                    int32_t* status) {
  __shared__ int s_warp[OCC_ITERS][OCC_THREADS / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t base = (int64_t)blockIdx.x * OCC_TILE;
  int64_t pos0 = blockIdx.x == 0 ? 0 : (int64_t)tile_incl[blockIdx.x - 1];
  bool flag[OCC_ITERS];
  uint32_t ballot[OCC_ITERS];
#pragma unroll
  for (int i = 0; i < OCC_ITERS; ++i) {
    flag[i] = occupied(logits, g, base + i * OCC_THREADS + threadIdx.x, thr);
    ballot[i] = __ballot_sync(0xffffffffu, flag[i]);
    if (lane == 0) s_warp[i][warp] = __popc(ballot[i]);
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < OCC_ITERS; ++i) {
    int before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < OCC_THREADS / 32; ++w) {
      const int c = s_warp[i][w];
      before += w < warp ? c : 0;
      all += c;
    }
    if (flag[i]) {
      const int64_t pos = pos0 + before + __popc(ballot[i] & ((1u << lane) - 1u));
      const int64_t e = base + i * OCC_THREADS + threadIdx.x;
      if (pos < m) {
        const int64_t w = e % g.shape[3];
        int64_t r = e / g.shape[3];
        const int64_t h = r % g.shape[2];
        r /= g.shape[2];
        const int64_t d = r % g.shape[1];
        const int64_t b = r / g.shape[1];
        out[pos] = make_int4((int)b, (int)d, (int)h, (int)w);
      } else {
        report(status, SV_DEVICE_BAD_INDEX);  // the logits changed since the count
      }
    }
    pos0 += all;
  }
}

int make_grid(const int64_t shape[4], const int64_t strides[4], Grid4* g) {
  if (!shape || !strides) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "occupancy: null shape or strides");
  g->total = 1;
  for (int j = 0; j < 4; ++j) {
    if (shape[j] < 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "occupancy: negative extent");
    if (shape[j] > INT32_MAX) SV_FAIL(SV_ERR_UNSUPPORTED, "occupancy: extent above 2^31-1");
    g->shape[j] = shape[j];
    g->stride[j] = strides[j];
    g->total *= shape[j];
    if (g->total > INT32_MAX - OCC_TILE)
      SV_FAIL(SV_ERR_UNSUPPORTED, "occupancy: more than 2^31 - 1025 grid cells");
  }
  g->contiguous = strides[3] == 1 && strides[2] == shape[3] &&
                  strides[1] == shape[2] * shape[3] &&
                  strides[0] == shape[1] * shape[2] * shape[3];
  return SV_OK;
}

// The threshold as MLX compares it: a Python float becomes a float32 scalar, which takes the
// logits' floating type.
float rounded_threshold(double threshold, int dtype) {
  const float t32 = (float)threshold;
  if (dtype == SV_FLOAT16) return __half2float(__float2half_rn(t32));
  if (dtype == SV_BFLOAT16) return __bfloat162float(__float2bfloat16_rn(t32));
  return t32;
}

int64_t occ_tiles(int64_t total) { return (total + OCC_TILE - 1) / OCC_TILE; }

size_t occ_scan_bytes(int64_t tiles) {
  size_t b = 0;
  cub::DeviceScan::InclusiveSum(nullptr, b, (const int32_t*)nullptr, (int32_t*)nullptr,
                                (int)tiles);
  return b;
}

__global__ void subdivide_coords_kernel(const int4* __restrict__ coords, int64_t n,
                                        int4* __restrict__ out) {
  const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= n * 8) return;
  const int4 c = __ldg(&coords[o >> 3]);
  const uint32_t j = (uint32_t)(o & 7);
  out[o] = make_int4(c.x, (int)((uint32_t)c.y * 2u + (j >> 2)),
                     (int)((uint32_t)c.z * 2u + ((j >> 1) & 1u)),
                     (int)((uint32_t)c.w * 2u + (j & 1u)));
}

template <int BYTES>
__global__ void expand_rows_kernel(const uint8_t* __restrict__ src, int64_t n, int row_bytes,
                                   uint8_t* __restrict__ dst) {
  // One thread per (output row, BYTES-wide chunk); output row o copies source row o / 8.
  const int chunks = row_bytes / BYTES;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n * 8 * chunks) return;
  const int64_t o = t / chunks;
  const int c = (int)(t - o * chunks);
  const uint8_t* s = src + (o >> 3) * row_bytes + (int64_t)c * BYTES;
  uint8_t* d = dst + o * row_bytes + (int64_t)c * BYTES;
  if constexpr (BYTES == 16)
    *reinterpret_cast<uint4*>(d) = __ldg(reinterpret_cast<const uint4*>(s));
  else
    *d = *s;
}

}  // namespace
}  // namespace sv

using namespace sv;

extern "C" size_t sv_occupancy_workspace_bytes(const int64_t shape[4]) {
  if (!shape) return 0;
  int64_t total = 1;
  for (int j = 0; j < 4; ++j) total *= shape[j] > 0 ? shape[j] : 0;
  const int64_t tiles = occ_tiles(total);
  if (tiles == 0) return 256;
  return 2 * align_up((size_t)tiles * 4, 256) + align_up(occ_scan_bytes(tiles), 256);
}

static int occ_prepare(const void* logits, int dtype, const int64_t shape[4],
                       const int64_t strides[4], void* workspace, size_t workspace_bytes,
                       Grid4* g, int32_t** counts, int32_t** incl, void** tmp,
                       size_t* tmp_bytes) {
  if (dtype != SV_FLOAT32 && dtype != SV_FLOAT16 && dtype != SV_BFLOAT16)
    SV_FAIL(SV_ERR_BAD_DTYPE, "occupancy: unknown dtype");
  int rc = make_grid(shape, strides, g);
  if (rc != SV_OK) return rc;
  if (g->total == 0) return SV_OK;
  if (!logits) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "occupancy: null logits");
  if (workspace == nullptr || workspace_bytes < sv_occupancy_workspace_bytes(shape))
    SV_FAIL(SV_ERR_WORKSPACE, "occupancy: workspace too small");
  const int64_t tiles = occ_tiles(g->total);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t tb = align_up((size_t)tiles * 4, 256);
  *counts = reinterpret_cast<int32_t*>(ws);
  *incl = reinterpret_cast<int32_t*>(ws + tb);
  *tmp = ws + 2 * tb;
  *tmp_bytes = align_up(occ_scan_bytes(tiles), 256);
  return SV_OK;
}

extern "C" int sv_occupancy_count(const void* logits, int dtype, const int64_t shape[4],
                                  const int64_t strides[4], double threshold, int64_t* out_m,
                                  void* workspace, size_t workspace_bytes, sv_stream_t stream) {
  if (!out_m) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_occupancy_count: null out_m");
  *out_m = 0;
  Grid4 g;
  int32_t *counts = nullptr, *incl = nullptr;
  void* tmp = nullptr;
  size_t tmp_bytes = 0;
  int rc = occ_prepare(logits, dtype, shape, strides, workspace, workspace_bytes, &g, &counts,
                       &incl, &tmp, &tmp_bytes);
  if (rc != SV_OK || g.total == 0) return rc;
  cudaStream_t s = to_stream(stream);
  const float thr = rounded_threshold(threshold, dtype);
  const unsigned tiles = (unsigned)occ_tiles(g.total);
  if (dtype == SV_FLOAT32)
    occ_count_kernel<float><<<tiles, OCC_THREADS, 0, s>>>(static_cast<const float*>(logits), g,
                                                          thr, counts);
  else if (dtype == SV_FLOAT16)
    occ_count_kernel<__half><<<tiles, OCC_THREADS, 0, s>>>(static_cast<const __half*>(logits),
                                                           g, thr, counts);
  else
    occ_count_kernel<__nv_bfloat16><<<tiles, OCC_THREADS, 0, s>>>(
        static_cast<const __nv_bfloat16*>(logits), g, thr, counts);
  SV_LAUNCH_CHECK();
  SV_CUDA_TRY(cub::DeviceScan::InclusiveSum(tmp, tmp_bytes, counts, incl, (int)tiles, s));
  int32_t m32 = 0;
  SV_CUDA_TRY(cudaMemcpyAsync(&m32, incl + (tiles - 1), sizeof(int32_t), cudaMemcpyDeviceToHost,
                              s));
  SV_CUDA_TRY(cudaStreamSynchronize(s));
  *out_m = m32;
  return SV_OK;
}

extern "C" int sv_occupancy_emit(const void* logits, int dtype, const int64_t shape[4],
                                 const int64_t strides[4], double threshold, int32_t* out_coords,
                                 int64_t m, int32_t* status, void* workspace,
                                 size_t workspace_bytes, sv_stream_t stream) {
  Grid4 g;
  int32_t *counts = nullptr, *incl = nullptr;
  void* tmp = nullptr;
  size_t tmp_bytes = 0;
  int rc = occ_prepare(logits, dtype, shape, strides, workspace, workspace_bytes, &g, &counts,
                       &incl, &tmp, &tmp_bytes);
  if (rc != SV_OK || g.total == 0 || m == 0) return rc;
  if (m < 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_occupancy_emit: negative m");
  if (!out_coords || !aligned16(out_coords))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_occupancy_emit: out_coords null or not 16-byte aligned");
  cudaStream_t s = to_stream(stream);
  const float thr = rounded_threshold(threshold, dtype);
  const unsigned tiles = (unsigned)occ_tiles(g.total);
  int4* out = reinterpret_cast<int4*>(out_coords);
  if (dtype == SV_FLOAT32)
    occ_emit_kernel<float><<<tiles, OCC_THREADS, 0, s>>>(static_cast<const float*>(logits), g,
                                                         thr, incl, m, out, status);
  else if (dtype == SV_FLOAT16)
    occ_emit_kernel<__half><<<tiles, OCC_THREADS, 0, s>>>(static_cast<const __half*>(logits), g,
                                                          thr, incl, m, out, status);
  else
    occ_emit_kernel<__nv_bfloat16><<<tiles, OCC_THREADS, 0, s>>>(
        static_cast<const __nv_bfloat16*>(logits), g, thr, incl, m, out, status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

extern "C" int sv_subdivide(const int32_t* coords, int64_t n, const void* features,
                            int64_t row_bytes, int32_t* out_coords, void* out_features,
                            sv_stream_t stream) {
  if (n < 0 || row_bytes < 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_subdivide: negative size");
  if (n == 0) return SV_OK;
  if (n > INT64_MAX / 8 / (row_bytes > 0 ? row_bytes : 1))
    SV_FAIL(SV_ERR_UNSUPPORTED, "sv_subdivide: output too large");
  if (row_bytes > INT32_MAX) SV_FAIL(SV_ERR_UNSUPPORTED, "sv_subdivide: row above 2^31 bytes");
  if (!coords || !out_coords) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_subdivide: null coords");
  if (!aligned16(coords) || !aligned16(out_coords))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "coords must be 16-byte aligned");
  cudaStream_t s = to_stream(stream);
  subdivide_coords_kernel<<<(unsigned)((n * 8 + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const int4*>(coords), n, reinterpret_cast<int4*>(out_coords));
  SV_LAUNCH_CHECK();
  if (row_bytes == 0) return SV_OK;
  if (!features || !out_features) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_subdivide: null features");
  const int rb = (int)row_bytes;
  const bool vec = rb % 16 == 0 && aligned16(features) && aligned16(out_features);
  const int64_t threads = n * 8 * (vec ? rb / 16 : rb);
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  if (vec)
    expand_rows_kernel<16><<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(features), n, rb,
                                                  static_cast<uint8_t*>(out_features));
  else
    expand_rows_kernel<1><<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(features), n, rb,
                                                 static_cast<uint8_t*>(out_features));
  SV_LAUNCH_CHECK();
  return SV_OK;
}
