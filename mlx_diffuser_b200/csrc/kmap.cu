// Kernel-map construction: coordinate hash table, K-offset neighbour probe, and the
// mask-grouped row schedule for the tensor-core convolution.
//
// Restates build_neighbor_map (src/mlx_diffuser/layers/sparse.py:146-175) on the GPU:
//  * the reference's dict keyed by the 4-tuple (b, c1, c2, c3) becomes an open-addressing
//    table whose slots hold only a row index (4 bytes); a slot's key is the coordinate row it
//    points at, so keys are exact for every int32 value (no packing, no range limit);
//  * "a later duplicate overwrites an earlier one" (the dict comprehension, :159) becomes
//    atomicMax on the slot: the largest row index among equal rows wins;
//  * offsets are enumerated in the reference's order (:160-169); a neighbour coordinate that
//    leaves the int32 range simply misses, as a Python dict lookup of that tuple would.
#include <algorithm>
#include <mutex>
#include <string>

#include <cub/device/device_radix_sort.cuh>

#include "common.cuh"

namespace sv {
namespace {

__device__ __forceinline__ uint32_t hash_coord(int b, int x, int y, int z) {
  uint64_t h = (uint64_t)(uint32_t)b * 0x9E3779B97F4A7C15ull;
  h += (uint64_t)(uint32_t)x * 0xC2B2AE3D27D4EB4Full;
  h += (uint64_t)(uint32_t)y * 0x165667B19E3779F9ull;
  h += (uint64_t)(uint32_t)z * 0x27D4EB2F165667C5ull;
  // 64-bit finaliser (MurmurHash3 fmix64)
  h ^= h >> 33;
  h *= 0xFF51AFD7ED558CCDull;
  h ^= h >> 33;
  h *= 0xC4CEB9FE1A85EC53ull;
  h ^= h >> 33;
  return (uint32_t)h;
}

__device__ __forceinline__ bool same(int4 a, int b, int x, int y, int z) {
  return a.x == b && a.y == x && a.z == y && a.w == z;
}

__global__ void kmap_insert_kernel(const int4* __restrict__ coords, int64_t n, int32_t* table,
                                   uint32_t mask, int32_t* status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int4 c = __ldg(&coords[i]);
  uint32_t h = hash_coord(c.x, c.y, c.z, c.w) & mask;
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    int32_t cur = *((volatile int32_t*)&table[h]);
    if (cur < 0) {
      const int32_t prev = atomicCAS(&table[h], -1, (int32_t)i);
      if (prev < 0) return;  // claimed an empty slot
      cur = prev;
    }
    // A slot's key never changes once claimed: it only moves to larger rows of the same key.
    if (same(__ldg(&coords[cur]), c.x, c.y, c.z, c.w)) {
      atomicMax(&table[h], (int32_t)i);
      return;
    }
    h = (h + 1) & mask;
  }
  report(status, SV_DEVICE_TABLE_FULL);
}

__device__ __forceinline__ int32_t kmap_lookup(const int4* __restrict__ coords,
                                               const int32_t* __restrict__ table, uint32_t mask,
                                               int b, int x, int y, int z) {
  uint32_t h = hash_coord(b, x, y, z) & mask;
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    const int32_t cur = __ldg(&table[h]);
    if (cur < 0) return -1;
    if (same(__ldg(&coords[cur]), b, x, y, z)) return cur;
    h = (h + 1) & mask;
  }
  return -1;
}

// One thread per (row, offset): writes nbr row-major, so consecutive threads store
// consecutive words.
__global__ void kmap_probe_kernel(const int4* __restrict__ coords, int64_t n,
                                  const int32_t* __restrict__ table, uint32_t mask, int k0,
                                  int k1, int k2, int d0, int d1, int d2,
                                  int32_t* __restrict__ nbr) {
  const int kvol = k0 * k1 * k2;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * kvol) return;
  const int64_t p = idx / kvol;
  const int k = (int)(idx - p * kvol);
  const int c = k % k2;
  const int b = (k / k2) % k1;
  const int a = k / (k1 * k2);
  const int4 q = __ldg(&coords[p]);
  const int64_t x = (int64_t)q.y + (int64_t)(a - k0 / 2) * d0;
  const int64_t y = (int64_t)q.z + (int64_t)(b - k1 / 2) * d1;
  const int64_t z = (int64_t)q.w + (int64_t)(c - k2 / 2) * d2;
  int32_t r = -1;
  if (x >= INT32_MIN && x <= INT32_MAX && y >= INT32_MIN && y <= INT32_MAX && z >= INT32_MIN &&
      z <= INT32_MAX)
    r = kmap_lookup(coords, table, mask, q.x, (int)x, (int)y, (int)z);
  nbr[idx] = r;
}

// ---- block table (3x3x3 kernels, dilation 1) ---------------------------------------------------
// The table holds 2x2x2 blocks of voxels instead of single voxels: a slot is a block's full key
// (batch, c1 >> 1, c2 >> 1, c3 >> 1) -- 16 bytes, claimed with one 128-bit compare-and-swap --
// and, in a parallel array, the rows of its 8 cells (32 bytes, cell = (c1 & 1) << 2 |
// (c2 & 1) << 1 | (c3 & 1)). The 27 neighbours of a voxel lie in exactly 8 blocks (two per axis),
// so a row's map takes 8 independent key probes instead of 27, each one 16-byte load; neighbouring
// rows share blocks, so most of those loads hit L1. A duplicate coordinate row resolves to the
// largest row index (atomicMax on its cell), as with the voxel table and the reference's dict.
// An empty slot's c1 >> 1 field holds 0x7F7F7F7F, a value an arithmetic shift of an int32 cannot
// produce, so the keys array is cleared with a byte memset.

constexpr int32_t BLOCK_EMPTY = 0x7F7F7F7F;

__device__ __forceinline__ bool same4(int4 a, int4 b) {
  return a.x == b.x && a.y == b.y && a.z == b.z && a.w == b.w;
}

__global__ void kmap_block_insert_kernel(const int4* __restrict__ coords, int64_t n,
                                         int4* keys, int32_t* cells, uint32_t mask,
                                         int32_t* status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int4 c = __ldg(&coords[i]);
  const int4 key = make_int4(c.x, c.y >> 1, c.z >> 1, c.w >> 1);
  const int cell = ((c.y & 1) << 2) | ((c.z & 1) << 1) | (c.w & 1);
  uint32_t h = hash_coord(key.x, key.y, key.z, key.w) & mask;
  const int4 empty = make_int4(BLOCK_EMPTY, BLOCK_EMPTY, BLOCK_EMPTY, BLOCK_EMPTY);
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    // A plain 16-byte read (L2, not L1) may be stale or interleave with another thread's
    // compare-and-swap of the slot. A read equal to the key is genuine (a mix of old and new
    // fields cannot equal a key, whose c1, c2, c3 fields are never 0x7F7F7F7F); anything else is
    // confirmed by the CAS, which returns the slot's value atomically (and claims it when empty).
    int4 cur = __ldcg(&keys[h]);
    if (!same4(cur, key)) {
      cur = atomicCAS(&keys[h], empty, key);
      if (cur.y == BLOCK_EMPTY) cur = key;  // claimed the empty slot
    }
    if (same4(cur, key)) {
      atomicMax(&cells[(int64_t)h * 8 + cell], (int32_t)i);
      return;
    }
    h = (h + 1) & mask;
  }
  report(status, SV_DEVICE_TABLE_FULL);
}

// Slot of the block `key`, or -1 when no row lies in it.
__device__ __forceinline__ int64_t block_find(const int4* __restrict__ keys, uint32_t mask,
                                              int4 key, uint32_t h, int4 first) {
  int4 cur = first;
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    if (same4(cur, key)) return (int64_t)h;
    if (cur.y == BLOCK_EMPTY) return -1;
    h = (h + 1) & mask;
    cur = __ldg(&keys[h]);
  }
  return -1;
}

// One thread per row (128 per CTA): the 8 blocks around the row are probed together, then the
// 27 neighbours are read from their cells; the CTA's [128][27] map rows go out through shared
// memory as contiguous stores.
__global__ void __launch_bounds__(128)
    kmap_block_probe_kernel(const int4* __restrict__ coords, int64_t n,
                            const int4* __restrict__ keys, const int32_t* __restrict__ cells,
                            uint32_t mask, int32_t* __restrict__ nbr) {
  __shared__ int32_t stage[128 * 27];
  const int64_t row0 = (int64_t)blockIdx.x * 128;
  const int64_t i = row0 + threadIdx.x;
  if (i < n) {
    const int4 c = __ldg(&coords[i]);
    // the two block coordinates along each axis that the offsets -1, 0, +1 reach (a side whose
    // neighbour leaves the int32 range has no block: its neighbours miss)
    int32_t g[3][2];
    bool ok[3][2];
    const int32_t v3[3] = {c.y, c.z, c.w};
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      const int64_t lo = (int64_t)v3[a] - 1, hi = (int64_t)v3[a] + 1;
      ok[a][0] = lo >= INT32_MIN;
      ok[a][1] = hi <= INT32_MAX;
      g[a][0] = (int32_t)(lo >> 1);
      g[a][1] = (int32_t)(hi >> 1);
    }
    // first probe of all 8 blocks in flight together
    int4 bkey[8];
    uint32_t bh[8];
    int4 first[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      bkey[b] = make_int4(c.x, g[0][b >> 2], g[1][(b >> 1) & 1], g[2][b & 1]);
      bh[b] = hash_coord(bkey[b].x, bkey[b].y, bkey[b].z, bkey[b].w) & mask;
      first[b] = __ldg(&keys[bh[b]]);
    }
    int64_t slot[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const bool in_range = ok[0][b >> 2] && ok[1][(b >> 1) & 1] && ok[2][b & 1];
      slot[b] = in_range ? block_find(keys, mask, bkey[b], bh[b], first[b]) : -1;
    }
    // offset k = 9 (d1 + 1) + 3 (d2 + 1) + (d3 + 1), the reference's order
#pragma unroll
    for (int k = 0; k < 27; ++k) {
      const int d[3] = {k / 9 - 1, (k / 3) % 3 - 1, k % 3 - 1};
      int b = 0, cell = 0;
      bool valid = true;
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        const int64_t v = (int64_t)v3[a] + d[a];
        valid = valid && v >= INT32_MIN && v <= INT32_MAX;
        const int32_t gv = (int32_t)(v >> 1);
        // which of the two blocks along this axis: the upper one when its coordinate differs
        const int side = (d[a] > 0 || (d[a] == 0 && gv != g[a][0])) ? 1 : 0;
        b |= side << (2 - a);
        cell |= (int)(v & 1) << (2 - a);
      }
      const int64_t s = slot[b];
      stage[threadIdx.x * 27 + k] = (valid && s >= 0) ? __ldg(&cells[s * 8 + cell]) : -1;
    }
  }
  __syncthreads();
  const int64_t rows = min((int64_t)128, n - row0);
  int32_t* dst = nbr + row0 * 27;
  for (int j = threadIdx.x; j < rows * 27; j += 128) dst[j] = stage[j];
}

__global__ void row_mask_kernel(const int32_t* __restrict__ nbr, int64_t n, int kvol,
                                uint32_t* __restrict__ masks, int32_t* __restrict__ rows) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  uint32_t m = 0;
  for (int k = 0; k < kvol; ++k) m |= (uint32_t)(__ldg(&nbr[p * kvol + k]) >= 0) << k;
  masks[p] = m;
  rows[p] = (int32_t)p;
}

// Cost of each 128-row tile of the schedule: the number of offsets the tensor-core kernel
// visits for it (popcount of the union of its rows' masks), stored as 32 - cost so that an
// ascending sort lists the most expensive tiles first.
__global__ void tile_cost_kernel(const uint32_t* __restrict__ masks_sorted, int64_t n,
                                 int64_t tiles, uint32_t* __restrict__ keys,
                                 int32_t* __restrict__ ids) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= tiles) return;
  uint32_t u = 0;
  for (int64_t r = t * 128 + lane; r < min(n, (t + 1) * 128); r += 32) u |= masks_sorted[r];
  u = __reduce_or_sync(0xffffffffu, u);
  if (lane == 0) {
    keys[t] = 32u - (uint32_t)__popc(u);
    ids[t] = (int32_t)t;
  }
}

// ---- direct-indexed grid -------------------------------------------------------------------
// When a scene's bounding box (in batch, c1, c2, c3) is not much larger than its row count, a
// dense grid of row indices replaces the hash table: insert is one atomicMax per row (the
// largest duplicate wins, as in the hash table and the reference's dict), a lookup is one
// load, and the 3 offsets along c3 of a row hit neighbouring cells. Cells are row-major in
// (batch, c1, c2, c3).

struct GridBox {
  int32_t lo[4];
  int64_t ext[4];  // extents; cell = ((b * e1 + c1) * e2 + c2) * e3 + c3 after subtracting lo
};

__device__ __forceinline__ bool grid_cell(const GridBox& g, int64_t b, int64_t x, int64_t y,
                                          int64_t z, int64_t* cell) {
  b -= g.lo[0];
  x -= g.lo[1];
  y -= g.lo[2];
  z -= g.lo[3];
  if (b < 0 || b >= g.ext[0] || x < 0 || x >= g.ext[1] || y < 0 || y >= g.ext[2] || z < 0 ||
      z >= g.ext[3])
    return false;
  *cell = ((b * g.ext[1] + x) * g.ext[2] + y) * g.ext[3] + z;
  return true;
}

__global__ void bounds4_kernel(const int4* __restrict__ coords, int64_t n, int32_t* bounds) {
  int mn[4] = {INT32_MAX, INT32_MAX, INT32_MAX, INT32_MAX};
  int mx[4] = {INT32_MIN, INT32_MIN, INT32_MIN, INT32_MIN};
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int4 c = __ldg(&coords[i]);
    const int v[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      mn[j] = min(mn[j], v[j]);
      mx[j] = max(mx[j], v[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    mn[j] = __reduce_min_sync(0xffffffffu, mn[j]);
    mx[j] = __reduce_max_sync(0xffffffffu, mx[j]);
  }
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      atomicMin(&bounds[j], mn[j]);
      atomicMax(&bounds[4 + j], mx[j]);
    }
  }
}

__global__ void bounds4_init_kernel(int32_t* bounds) {
  if (threadIdx.x < 4) bounds[threadIdx.x] = INT32_MAX;
  else if (threadIdx.x < 8) bounds[threadIdx.x] = INT32_MIN;
}

__global__ void grid_insert_kernel(const int4* __restrict__ coords, int64_t n, GridBox g,
                                   int32_t* grid, int32_t* status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int4 c = __ldg(&coords[i]);
  int64_t cell;
  if (!grid_cell(g, c.x, c.y, c.z, c.w, &cell)) {
    report(status, SV_DEVICE_BAD_INDEX);  // outside the box the caller gave: never written
    return;
  }
  atomicMax(&grid[cell], (int32_t)i);
}

// One thread per (row, offset), like kmap_probe_kernel.
__global__ void grid_probe_kernel(const int4* __restrict__ coords, int64_t n, GridBox g,
                                  const int32_t* __restrict__ grid, int k0, int k1, int k2,
                                  int d0, int d1, int d2, int32_t* __restrict__ nbr) {
  const int kvol = k0 * k1 * k2;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * kvol) return;
  const int64_t p = idx / kvol;
  const int k = (int)(idx - p * kvol);
  const int c = k % k2;
  const int b = (k / k2) % k1;
  const int a = k / (k1 * k2);
  const int4 q = __ldg(&coords[p]);
  int64_t cell;
  int32_t r = -1;
  if (grid_cell(g, q.x, (int64_t)q.y + (int64_t)(a - k0 / 2) * d0,
                (int64_t)q.z + (int64_t)(b - k1 / 2) * d1,
                (int64_t)q.w + (int64_t)(c - k2 / 2) * d2, &cell))
    r = __ldg(&grid[cell]);
  nbr[idx] = r;
}

size_t plan_cub_bytes(int64_t n) {
  size_t bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, (int)n, 0, 32);
  return bytes;
}

}  // namespace
}  // namespace sv

using namespace sv;

extern "C" int64_t sv_kmap_table_slots(int64_t n) {
  int64_t slots = 64;
  while (slots < 2 * n) slots <<= 1;
  return slots;
}

extern "C" size_t sv_kmap_workspace_bytes(int64_t table_slots) {
  // block table: 16-byte keys + 8 four-byte cells per slot (the voxel table needs 4 bytes)
  return table_slots > 0 ? (size_t)table_slots * 48 : 0;
}

namespace {

int kmap_check(const int32_t* coords, int64_t n, const int32_t kernel[3],
               const int32_t dilation[3], int32_t* nbr, int64_t table_slots) {
  if (n < 0 || kernel == nullptr || dilation == nullptr)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_build: bad arguments");
  for (int i = 0; i < 3; ++i)
    if (kernel[i] <= 0 || kernel[i] % 2 == 0)
      SV_FAIL(SV_ERR_BAD_SHAPE, "sparse submanifold kernels must have three odd dimensions");
  if (n == 0) return SV_OK;
  if (coords == nullptr || nbr == nullptr)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_build: null coords or nbr");
  if (n > INT32_MAX - 1) SV_FAIL(SV_ERR_UNSUPPORTED, "sv_kmap_build: more than 2^31-2 rows");
  if (!aligned16(coords)) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "coords must be 16-byte aligned");
  if (table_slots < 64 || (table_slots & (table_slots - 1)) != 0 || table_slots > (1ll << 31))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "table_slots must be a power of two in [64, 2^31]");
  return SV_OK;
}

// The map through a table of single voxels (4 bytes per slot): any kernel and dilation.
int kmap_build_voxels(const int32_t* coords, int64_t n, const int32_t kernel[3],
                      const int32_t dilation[3], int32_t* nbr, int64_t table_slots,
                      int32_t* table, int32_t* status, cudaStream_t s) {
  const int64_t kvol = (int64_t)kernel[0] * kernel[1] * kernel[2];
  const uint32_t mask = (uint32_t)(table_slots - 1);
  SV_CUDA_TRY(cudaMemsetAsync(table, 0xFF, (size_t)table_slots * sizeof(int32_t), s));
  const int threads = 256;
  kmap_insert_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, s>>>(
      reinterpret_cast<const int4*>(coords), n, table, mask, status);
  SV_LAUNCH_CHECK();
  const int64_t total = n * kvol;
  kmap_probe_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, s>>>(
      reinterpret_cast<const int4*>(coords), n, table, mask, kernel[0], kernel[1], kernel[2],
      dilation[0], dilation[1], dilation[2], nbr);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

// The 3x3x3, dilation-1 map through the block table (48 bytes per slot).
int kmap_build_blocks(const int32_t* coords, int64_t n, int32_t* nbr, int64_t table_slots,
                      void* workspace, int32_t* status, cudaStream_t s) {
  const uint32_t mask = (uint32_t)(table_slots - 1);
  int4* keys = static_cast<int4*>(workspace);
  int32_t* cells = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + table_slots * 16);
  SV_CUDA_TRY(cudaMemsetAsync(keys, 0x7F, (size_t)table_slots * 16, s));
  SV_CUDA_TRY(cudaMemsetAsync(cells, 0xFF, (size_t)table_slots * 32, s));
  kmap_block_insert_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const int4*>(coords), n, keys, cells, mask, status);
  SV_LAUNCH_CHECK();
  kmap_block_probe_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(
      reinterpret_cast<const int4*>(coords), n, keys, cells, mask, nbr);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

}  // namespace

extern "C" int sv_kmap_build(const int32_t* coords, int64_t n, const int32_t kernel[3],
                             const int32_t dilation[3], int32_t* nbr, int64_t table_slots,
                             void* workspace, size_t workspace_bytes, int32_t* status,
                             sv_stream_t stream) {
  const int rc = kmap_check(coords, n, kernel, dilation, nbr, table_slots);
  if (rc != SV_OK || n == 0) return rc;
  if (workspace == nullptr || workspace_bytes < sv_kmap_workspace_bytes(table_slots))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_kmap_build: workspace too small");
  cudaStream_t s = to_stream(stream);
  const bool k333 = kernel[0] == 3 && kernel[1] == 3 && kernel[2] == 3 && dilation[0] == 1 &&
                    dilation[1] == 1 && dilation[2] == 1;
  if (k333) return kmap_build_blocks(coords, n, nbr, table_slots, workspace, status, s);
  return kmap_build_voxels(coords, n, kernel, dilation, nbr, table_slots,
                           static_cast<int32_t*>(workspace), status, s);
}

extern "C" int sv_coords_bounds(const int32_t* coords, int64_t n, int32_t* bounds_out,
                                void* workspace, size_t workspace_bytes, sv_stream_t stream) {
  if (n < 0 || !bounds_out) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_coords_bounds: bad arguments");
  if (n == 0) {
    for (int j = 0; j < 4; ++j) {
      bounds_out[j] = 0;
      bounds_out[4 + j] = -1;
    }
    return SV_OK;
  }
  if (!coords || !aligned16(coords))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_coords_bounds: coords null or not 16-byte aligned");
  if (!workspace || workspace_bytes < 32)
    SV_FAIL(SV_ERR_WORKSPACE, "sv_coords_bounds: needs 32 bytes of workspace");
  cudaStream_t s = to_stream(stream);
  int32_t* dev_bounds = static_cast<int32_t*>(workspace);
  bounds4_init_kernel<<<1, 32, 0, s>>>(dev_bounds);
  SV_LAUNCH_CHECK();
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 4 * num_sms());
  bounds4_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const int4*>(coords), n, dev_bounds);
  SV_LAUNCH_CHECK();
  SV_CUDA_TRY(cudaMemcpyAsync(bounds_out, dev_bounds, 8 * sizeof(int32_t),
                              cudaMemcpyDeviceToHost, s));
  SV_CUDA_TRY(cudaStreamSynchronize(s));
  return SV_OK;
}

extern "C" size_t sv_kmap_grid_workspace_bytes(const int64_t extent[4]) {
  if (!extent) return 0;
  int64_t cells = 1;
  for (int j = 0; j < 4; ++j) {
    if (extent[j] <= 0) return 0;
    if (cells > INT64_MAX / 4 / extent[j]) return 0;
    cells *= extent[j];
  }
  return (size_t)cells * sizeof(int32_t);
}

extern "C" int sv_kmap_build_grid(const int32_t* coords, int64_t n, const int32_t kernel[3],
                                  const int32_t dilation[3], int32_t* nbr, const int32_t lo[4],
                                  const int64_t extent[4], void* workspace,
                                  size_t workspace_bytes, int32_t* status, sv_stream_t stream) {
  if (n < 0 || kernel == nullptr || dilation == nullptr || lo == nullptr || extent == nullptr)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_build_grid: bad arguments");
  for (int i = 0; i < 3; ++i)
    if (kernel[i] <= 0 || kernel[i] % 2 == 0)
      SV_FAIL(SV_ERR_BAD_SHAPE, "sparse submanifold kernels must have three odd dimensions");
  const int64_t kvol = (int64_t)kernel[0] * kernel[1] * kernel[2];
  if (n == 0) return SV_OK;
  if (coords == nullptr || nbr == nullptr)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_build_grid: null coords or nbr");
  if (n > INT32_MAX - 1) SV_FAIL(SV_ERR_UNSUPPORTED, "sv_kmap_build_grid: more than 2^31-2 rows");
  if (!aligned16(coords)) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "coords must be 16-byte aligned");
  const size_t need = sv_kmap_grid_workspace_bytes(extent);
  if (need == 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_build_grid: bad extents");
  if (workspace == nullptr || workspace_bytes < need)
    SV_FAIL(SV_ERR_WORKSPACE, "sv_kmap_build_grid: workspace smaller than the grid");
  GridBox g;
  for (int j = 0; j < 4; ++j) {
    g.lo[j] = lo[j];
    g.ext[j] = extent[j];
  }
  cudaStream_t s = to_stream(stream);
  int32_t* grid = static_cast<int32_t*>(workspace);
  SV_CUDA_TRY(cudaMemsetAsync(grid, 0xFF, need, s));
  const int threads = 256;
  grid_insert_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, s>>>(
      reinterpret_cast<const int4*>(coords), n, g, grid, status);
  SV_LAUNCH_CHECK();
  const int64_t total = n * kvol;
  grid_probe_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, s>>>(
      reinterpret_cast<const int4*>(coords), n, g, grid, kernel[0], kernel[1], kernel[2],
      dilation[0], dilation[1], dilation[2], nbr);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

extern "C" int64_t sv_conv_plan_tiles(int64_t n) { return n > 0 ? (n + 127) / 128 : 0; }

namespace {
size_t plan_tile_cub_bytes(int64_t tiles) {
  size_t bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, (int)tiles, 0, 6);
  return bytes;
}
}  // namespace

extern "C" size_t sv_conv_plan_workspace_bytes(int64_t n) {
  if (n <= 0) return 0;
  const int64_t tiles = sv_conv_plan_tiles(n);
  // row masks, sorted masks, row ids; tile keys, sorted tile keys, tile ids; CUB scratch
  return align_up((size_t)n * 4, 256) * 3 + align_up((size_t)tiles * 4, 256) * 3 +
         align_up(std::max(plan_cub_bytes(n), plan_tile_cub_bytes(tiles)), 256);
}

extern "C" int sv_conv_plan(const int32_t* nbr, int64_t n, int kvol, int32_t* row_order,
                            int32_t* tile_order, void* workspace, size_t workspace_bytes,
                            sv_stream_t stream) {
  if (n < 0 || kvol <= 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv_plan: bad sizes");
  if (kvol > 32) SV_FAIL(SV_ERR_UNSUPPORTED, "sv_conv_plan: kernel volume above 32");
  if (n == 0) return SV_OK;
  if (n > INT32_MAX) SV_FAIL(SV_ERR_UNSUPPORTED, "sv_conv_plan: more than 2^31-1 rows");
  if (nbr == nullptr || row_order == nullptr)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv_plan: null pointer");
  if (workspace == nullptr || workspace_bytes < sv_conv_plan_workspace_bytes(n))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_conv_plan: workspace too small");
  cudaStream_t s = to_stream(stream);
  const int64_t tiles = sv_conv_plan_tiles(n);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t vec = align_up((size_t)n * 4, 256);
  const size_t tvec = align_up((size_t)tiles * 4, 256);
  uint32_t* masks = reinterpret_cast<uint32_t*>(ws);
  uint32_t* masks_sorted = reinterpret_cast<uint32_t*>(ws + vec);
  int32_t* rows = reinterpret_cast<int32_t*>(ws + 2 * vec);
  uint32_t* tkeys = reinterpret_cast<uint32_t*>(ws + 3 * vec);
  uint32_t* tkeys_sorted = reinterpret_cast<uint32_t*>(ws + 3 * vec + tvec);
  int32_t* tids = reinterpret_cast<int32_t*>(ws + 3 * vec + 2 * tvec);
  void* cub_tmp = ws + 3 * vec + 3 * tvec;
  size_t cub_bytes = workspace_bytes - (3 * vec + 3 * tvec);
  row_mask_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(nbr, n, kvol, masks, rows);
  SV_LAUNCH_CHECK();
  SV_CUDA_TRY(cub::DeviceRadixSort::SortPairs(cub_tmp, cub_bytes, masks, masks_sorted, rows,
                                              row_order, (int)n, 0, kvol, s));
  if (tile_order != nullptr) {
    tile_cost_kernel<<<(unsigned)((tiles + 7) / 8), 256, 0, s>>>(masks_sorted, n, tiles, tkeys,
                                                                 tids);
    SV_LAUNCH_CHECK();
    size_t tile_cub_bytes = cub_bytes;
    SV_CUDA_TRY(cub::DeviceRadixSort::SortPairs(cub_tmp, tile_cub_bytes, tkeys, tkeys_sorted,
                                                tids, tile_order, (int)tiles, 0, 6, s));
  }
  return SV_OK;
}

// ---- allocation-free kernel map ------------------------------------------------------------
//
// For callers that cannot allocate device memory themselves -- a host application that owns
// every byte of GPU memory and forbids plugins from calling cudaMalloc, or a foreign-language
// caller that holds only its input and output buffers and no device allocator -- the hash
// table of sv_kmap_build lives here, in a fixed array compiled into the library. Every GPU that
// loads the library holds this array (SV_KMAP_STATIC_MAX_ROWS rows' worth of slots, 4 MiB)
// until the process exits. All calls on a device share it, so calls whose work overlaps on the
// GPU (different streams, or different host threads on one device) race on the table.

static __device__ __align__(256) int32_t sv_kmap_static_table[2 * SV_KMAP_STATIC_MAX_ROWS];

namespace {
std::mutex g_static_table_mu;
int32_t* g_static_table_addr[256] = {};

// Device address of sv_kmap_static_table on the current device. In host code the array's name
// only stands in for the symbol, so the address is looked up with the device current. A call
// outside stream capture looks it up afresh (the module, and so the array's address, changes
// when the caller resets the device or recreates its primary context) and remembers it; a call
// made while `stream` is capturing cannot look it up and uses the remembered one, which a call
// on that device before the capture must have stored.
int static_table_address(cudaStream_t stream, int32_t** out) {
  int dev = 0;
  SV_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 256) SV_FAIL(SV_ERR_UNSUPPORTED, "device index above 255");
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  SV_CUDA_TRY(cudaStreamIsCapturing(stream, &capture));
  std::lock_guard<std::mutex> lock(g_static_table_mu);
  if (capture == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    SV_CUDA_TRY(cudaGetSymbolAddress(&p, sv_kmap_static_table));
    g_static_table_addr[dev] = static_cast<int32_t*>(p);
  } else if (g_static_table_addr[dev] == nullptr) {
    SV_FAIL(SV_ERR_INVALID_ARGUMENT,
            "sv_kmap_build_static: the first call on a device must come before stream capture");
  }
  *out = g_static_table_addr[dev];
  return SV_OK;
}
}  // namespace

extern "C" int sv_kmap_build_static(const int32_t* coords, int64_t n, const int32_t kernel[3],
                                    const int32_t dilation[3], int32_t* nbr, int32_t* status,
                                    sv_stream_t stream) {
  if (n > SV_KMAP_STATIC_MAX_ROWS)
    SV_FAIL(SV_ERR_UNSUPPORTED,
            "sv_kmap_build_static: at most " + std::to_string(SV_KMAP_STATIC_MAX_ROWS) +
                " coordinate rows (got " + std::to_string(n) +
                "); use sv_kmap_build with a caller-provided workspace");
  const int64_t slots = sv_kmap_table_slots(n);  // <= 2 * SV_KMAP_STATIC_MAX_ROWS
  int32_t* table = nullptr;
  if (n > 0) {
    const int rc = static_table_address(to_stream(stream), &table);
    if (rc != SV_OK) return rc;
  }
  // the voxel table (4 bytes per slot) clears the `slots` words it uses to -1 before inserting,
  // so nothing of an earlier call's table survives into this one
  const int rc = kmap_check(coords, n, kernel, dilation, nbr, slots);
  if (rc != SV_OK || n == 0) return rc;
  return kmap_build_voxels(coords, n, kernel, dilation, nbr, slots, table, status,
                           to_stream(stream));
}
