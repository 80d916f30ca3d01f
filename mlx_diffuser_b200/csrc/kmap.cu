// Kernel-map construction (hash tables and dense grids, neighbour probes) and the mask-grouped
// row schedule for the tensor-core convolution.
//
// Restates build_neighbor_map (src/mlx_diffuser/layers/sparse.py:146-175) on the GPU:
//  * the reference's dict keyed by the 4-tuple (b, c1, c2, c3) becomes one of three exact
//    structures, for every int32 value (no packing, no range limit): a dense grid of row indices
//    over the coordinates' bounding box (for 3x3x3 maps, a grid of 2x2x2 blocks); an
//    open-addressing table of 2x2x2 blocks keyed by their full 16-byte coordinates (3x3x3,
//    dilation 1); or one of single voxels whose slots hold a row index (other kernels).
//    sv_kmap_build_auto picks between the grid and the table on the device;
//  * "a later duplicate overwrites an earlier one" (the dict comprehension, :159) becomes
//    atomicMax on the cell or slot: the largest row index among equal rows wins;
//  * offsets are enumerated in the reference's order (:160-169); a neighbour coordinate that
//    leaves the int32 range simply misses, as a Python dict lookup of that tuple would.
#include <algorithm>
#include <mutex>
#include <string>

#include <cub/block/block_radix_sort.cuh>
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

__device__ __forceinline__ void voxel_insert(const int4* __restrict__ coords, int64_t i, int4 c,
                                             int32_t* table, uint32_t mask, int32_t* status) {
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

__global__ void kmap_insert_kernel(const int4* __restrict__ coords, int64_t n, int32_t* table,
                                   uint32_t mask, int32_t* status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) voxel_insert(coords, i, __ldg(&coords[i]), table, mask, status);
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

// The neighbour of row coordinate q at offset k of a kernel (k0, k1, k2) with dilation
// (d0, d1, d2), in the reference's order; false when it leaves the int32 range (a miss, as a
// dict lookup of that tuple would be).
__device__ __forceinline__ bool offset_coord(int4 q, int k, int k0, int k1, int k2, int d0, int d1,
                                             int d2, int32_t* x, int32_t* y, int32_t* z) {
  const int c = k % k2;
  const int b = (k / k2) % k1;
  const int a = k / (k1 * k2);
  const int64_t xx = (int64_t)q.y + (int64_t)(a - k0 / 2) * d0;
  const int64_t yy = (int64_t)q.z + (int64_t)(b - k1 / 2) * d1;
  const int64_t zz = (int64_t)q.w + (int64_t)(c - k2 / 2) * d2;
  *x = (int32_t)xx;
  *y = (int32_t)yy;
  *z = (int32_t)zz;
  return xx >= INT32_MIN && xx <= INT32_MAX && yy >= INT32_MIN && yy <= INT32_MAX &&
         zz >= INT32_MIN && zz <= INT32_MAX;
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
  const int4 q = __ldg(&coords[p]);
  int32_t x, y, z, r = -1;
  if (offset_coord(q, (int)(idx - p * kvol), k0, k1, k2, d0, d1, d2, &x, &y, &z))
    r = kmap_lookup(coords, table, mask, q.x, x, y, z);
  nbr[idx] = r;
}

// ---- block table (3x3x3 kernels, dilation 1) ---------------------------------------------------
// The table holds 2x2x2 blocks of voxels instead of single voxels: slot h is the block's key
// keys[h] (16 bytes, claimed with one 128-bit compare-and-swap) and, in a parallel array, the
// rows of its 8 cells cells[h][0..7] (32 bytes, one sector; cell = (c1 & 1) << 2 |
// (c2 & 1) << 1 | (c3 & 1)). The 27 neighbours of a voxel lie in exactly 8 blocks (two per axis).
// A duplicate coordinate row resolves to the largest row index (atomicMax on its cell), as with
// the voxel table and the reference's dict.
//
// Key = (batch, (c1 >> 1) + 2^30, (c2 >> 1) + 2^30, (c3 >> 1) + 2^30): an arithmetic shift of an
// int32 lies in [-2^30, 2^30), so the three coordinate fields lie in [0, 2^31) and are never -1;
// one 0xFF byte memset of keys and cells leaves every slot empty (key field -1) with cells -1.

constexpr int32_t BLOCK_BIAS = 0x40000000;

__device__ __forceinline__ bool same4(int4 a, int4 b) {
  return a.x == b.x && a.y == b.y && a.z == b.z && a.w == b.w;
}

__device__ __forceinline__ int4 block_key(int32_t b, int32_t g1, int32_t g2, int32_t g3) {
  return make_int4(b, g1 + BLOCK_BIAS, g2 + BLOCK_BIAS, g3 + BLOCK_BIAS);
}

__device__ __forceinline__ void block_insert(const int4 c, int64_t i, int4* keys, int32_t* cells,
                                             uint32_t mask, int32_t* status) {
  const int4 key = block_key(c.x, c.y >> 1, c.z >> 1, c.w >> 1);
  const int cell = ((c.y & 1) << 2) | ((c.z & 1) << 1) | (c.w & 1);
  uint32_t h = hash_coord(key.x, key.y, key.z, key.w) & mask;
  const int4 empty = make_int4(-1, -1, -1, -1);
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    // the compare-and-swap returns the slot's key atomically, and claims the slot when empty
    const int4 cur = atomicCAS(&keys[h], empty, key);
    if (cur.y == -1 || same4(cur, key)) {
      atomicMax(&cells[(int64_t)h * 8 + cell], (int32_t)i);
      return;
    }
    h = (h + 1) & mask;
  }
  report(status, SV_DEVICE_TABLE_FULL);
}

__global__ void kmap_block_insert_kernel(const int4* __restrict__ coords, int64_t n, int4* keys,
                                         int32_t* cells, uint32_t mask, int32_t* status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) block_insert(__ldg(&coords[i]), i, keys, cells, mask, status);
}

// The probes run one thread per row. Along an axis the row's two blocks (sides 0 and 1) cover
// the 4 consecutive coordinates from 2 ((v - 1) >> 1), and the neighbours v - 1, v, v + 1 are 3 of
// them starting at 1 - (v & 1); so the 8 blocks' cells form a 4x4x4 cube and the 27 neighbours are
// the 3x3x3 window at (1 - (c1 & 1), 1 - (c2 & 1), 1 - (c3 & 1)), picked with selects on the
// three parities. Block s = 4 s1 + 2 s2 + s3 of a row has coordinates ((v - 1) >> 1) + s per axis;
// one whose coordinates leave the int32 range holds no row, and a neighbour whose coordinate
// leaves the range always falls in such a block.
constexpr int PROBE_ROWS = 128;  // rows (threads) per CTA

__device__ __forceinline__ int cell_of(const int4& lo, const int4& hi, int c) {
  switch (c) {
    case 0: return lo.x;
    case 1: return lo.y;
    case 2: return lo.z;
    case 3: return lo.w;
    case 4: return hi.x;
    case 5: return hi.y;
    case 6: return hi.z;
    default: return hi.w;
  }
}

// The row's 27 map entries from its 8 blocks' cells, in the reference's offset order
// k = 9 (d1 + 1) + 3 (d2 + 1) + (d3 + 1).
__device__ __forceinline__ void emit_window(int4 c, const int4 (&lo)[8], const int4 (&hi)[8],
                                            int32_t* row_stage) {
  const bool odd0 = c.y & 1, odd1 = c.z & 1, odd2 = c.w & 1;
  int w1[3][4][4];  // c1 resolved
#pragma unroll
  for (int x = 0; x < 3; ++x)
#pragma unroll
    for (int y = 0; y < 4; ++y)
#pragma unroll
      for (int z = 0; z < 4; ++z) {
        const int b0 = ((x >> 1) << 2) | ((y >> 1) << 1) | (z >> 1);
        const int b1 = (((x + 1) >> 1) << 2) | ((y >> 1) << 1) | (z >> 1);
        const int l0 = ((x & 1) << 2) | ((y & 1) << 1) | (z & 1);
        const int l1 = (((x + 1) & 1) << 2) | ((y & 1) << 1) | (z & 1);
        w1[x][y][z] = odd0 ? cell_of(lo[b0], hi[b0], l0) : cell_of(lo[b1], hi[b1], l1);
      }
  int w2[3][3][4];  // c2 resolved
#pragma unroll
  for (int x = 0; x < 3; ++x)
#pragma unroll
    for (int y = 0; y < 3; ++y)
#pragma unroll
      for (int z = 0; z < 4; ++z) w2[x][y][z] = odd1 ? w1[x][y][z] : w1[x][y + 1][z];
#pragma unroll
  for (int x = 0; x < 3; ++x)
#pragma unroll
    for (int y = 0; y < 3; ++y)
#pragma unroll
      for (int z = 0; z < 3; ++z)
        row_stage[x * 9 + y * 3 + z] = odd2 ? w2[x][y][z] : w2[x][y][z + 1];
}

// Lower block coordinate along each axis, (v - 1) >> 1, and whether each side lies in range.
struct RowBlocks {
  int64_t g[3];
  bool ok[3][2];
};

__device__ __forceinline__ RowBlocks row_blocks(int4 c) {
  RowBlocks rb;
  const int32_t v3[3] = {c.y, c.z, c.w};
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    rb.g[a] = ((int64_t)v3[a] - 1) >> 1;
    rb.ok[a][0] = v3[a] != INT32_MIN;  // v - 1 stays in range
    rb.ok[a][1] = v3[a] != INT32_MAX;  // v + 1 stays in range
  }
  return rb;
}

// The CTA's [PROBE_ROWS][27] map rows go out through shared memory as contiguous stores.
__device__ __forceinline__ void flush_rows(const int32_t* stage, int64_t n, int64_t row0,
                                           int32_t* __restrict__ nbr) {
  __syncthreads();
  const int64_t rows = min((int64_t)PROBE_ROWS, n - row0);
  int32_t* dst = nbr + row0 * 27;
  for (int j = threadIdx.x; j < rows * 27; j += blockDim.x) dst[j] = stage[j];
}

// A row's 8 blocks from the block table: all 8 home slots (key and cells) load together, then a
// block not in its home slot walks the keys.
__device__ __forceinline__ void block_probe_row(int4 c, const int4* __restrict__ keys,
                                                const int4* __restrict__ cells4, uint32_t mask,
                                                int32_t* row_stage) {
  const RowBlocks rb = row_blocks(c);
  int4 key[8], k0[8], lo[8], hi[8];
  uint32_t h0[8];
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const int s0 = b >> 2, s1 = (b >> 1) & 1, s2 = b & 1;
    const bool in = rb.ok[0][s0] && rb.ok[1][s1] && rb.ok[2][s2];
    key[b] = block_key(c.x, (int32_t)(rb.g[0] + s0), (int32_t)(rb.g[1] + s1),
                       (int32_t)(rb.g[2] + s2));
    h0[b] = hash_coord(key[b].x, key[b].y, key[b].z, key[b].w) & mask;
    k0[b] = make_int4(-1, -1, -1, -1);
    lo[b] = k0[b];
    hi[b] = k0[b];
    if (in) {
      k0[b] = __ldg(&keys[h0[b]]);
      lo[b] = __ldg(&cells4[2 * (int64_t)h0[b]]);
      hi[b] = __ldg(&cells4[2 * (int64_t)h0[b] + 1]);
    }
  }
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    if (same4(k0[b], key[b])) continue;
    const int4 none = make_int4(-1, -1, -1, -1);
    int4 l = none, u = none;
    if (k0[b].y != -1) {  // occupied by another block: walk on until the key or an empty slot
      uint32_t h = h0[b];
      for (uint32_t probe = 1; probe <= mask; ++probe) {
        h = (h + 1) & mask;
        const int4 k = __ldg(&keys[h]);
        if (k.y == -1) break;
        if (same4(k, key[b])) {
          l = __ldg(&cells4[2 * (int64_t)h]);
          u = __ldg(&cells4[2 * (int64_t)h + 1]);
          break;
        }
      }
    }
    lo[b] = l;
    hi[b] = u;
  }
  emit_window(c, lo, hi, row_stage);
}

__global__ void __launch_bounds__(PROBE_ROWS)
    kmap_block_probe_kernel(const int4* __restrict__ coords, int64_t n,
                            const int4* __restrict__ keys, const int4* __restrict__ cells4,
                            uint32_t mask, int32_t* __restrict__ nbr) {
  __shared__ int32_t stage[PROBE_ROWS * 27];
  const int64_t row0 = (int64_t)blockIdx.x * PROBE_ROWS;
  if (row0 + threadIdx.x < n)
    block_probe_row(__ldg(&coords[row0 + threadIdx.x]), keys, cells4, mask,
                    stage + threadIdx.x * 27);
  flush_rows(stage, n, row0, nbr);
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

// ---- one-cluster schedule for small maps -----------------------------------------------------
// Up to PLAN_SMALL_ROWS rows the schedule is one launch of a single thread-block cluster, one CTA
// per run of consecutive rows:
//   1. each CTA sorts its run's masks (with the row ids) by a block radix sort in registers and
//      shared memory -- stable, so rows of equal masks keep ascending row order -- and publishes
//      the sorted keys;
//   2. after a cluster barrier every CTA copies all runs' sorted keys into shared memory and
//      places each of its rows by merge rank: its rank in its own run, plus the rows of earlier
//      runs with a key <= its own, plus the rows of later runs with a key < its own (binary
//      searches). That is the position a stable sort of all rows gives. The row's mask is ORed
//      into its 128-row tile's union in global memory;
//   3. after a second barrier CTA 0 orders the tiles by a stable counting rank of their keys
//      32 - popcount(union) (ascending, ties by tile id), the order the device-wide pair sort of
//      the large path gives.
// A device-wide sort takes a histogram pass, a scan and four onesweep passes of a few
// microseconds each however few rows there are; this replaces them and the tile sort.
// Runs of 256 threads x ITEMS rows: a block radix sort's time grows with the rows one CTA sorts
// (measured on B200: 2048 rows ~12 us, 4096 ~19 us, 8192 ~31 us), so the shortest runs that fit
// a cluster are used -- 2048 rows (up to 16 CTAs, a non-portable cluster size) where the device
// can hold such a cluster, else 4096 rows (up to 8, the portable size).
constexpr int PLAN_THREADS = 256;
constexpr int PLAN_SMALL_ROWS = 32768;

template <int ITEMS>
struct PlanRuns {
  static constexpr int RUN = PLAN_THREADS * ITEMS;
  static constexpr int MAX_RUNS = PLAN_SMALL_ROWS / RUN;
  using Sort = cub::BlockRadixSort<uint32_t, PLAN_THREADS, ITEMS, int32_t>;
  static size_t smem(int runs) {
    return std::max(sizeof(typename Sort::TempStorage), (size_t)runs * RUN * 4);
  }
};

__device__ __forceinline__ void plan_cluster_sync() {
  __threadfence();  // global writes of this thread before the barrier's release
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <int ITEMS>
__global__ void __launch_bounds__(PLAN_THREADS, 1)
    plan_small_kernel(const uint32_t* __restrict__ masks, int n, int kvol, uint32_t* run_keys,
                      uint32_t* tile_union, int32_t* __restrict__ row_order,
                      int32_t* __restrict__ tile_order) {
  using R = PlanRuns<ITEMS>;
  extern __shared__ __align__(16) uint8_t plan_smem[];
  const int r = blockIdx.x;  // the grid is one cluster
  const int runs = gridDim.x;
  const int t = threadIdx.x;
  const int tiles = (n + 127) / 128;
  if (r == 0)
    for (int j = t; j < tiles; j += PLAN_THREADS) tile_union[j] = 0;
  // rows past n sort last: the largest key over the sorted bits, and after any real row of that
  // key by stability (they lie in the last run, after every real row)
  const uint32_t pad = kvol >= 32 ? 0xFFFFFFFFu : (1u << kvol) - 1u;
  uint32_t key[ITEMS];
  int32_t val[ITEMS];
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const int idx = r * R::RUN + t * ITEMS + i;
    key[i] = idx < n ? __ldg(&masks[idx]) : pad;
    val[i] = idx;
  }
  typename R::Sort(*reinterpret_cast<typename R::Sort::TempStorage*>(plan_smem)).Sort(key, val, 0, kvol);
  uint4* mine = reinterpret_cast<uint4*>(run_keys + r * R::RUN + t * ITEMS);
#pragma unroll
  for (int i = 0; i < ITEMS / 4; ++i)
    mine[i] = make_uint4(key[4 * i], key[4 * i + 1], key[4 * i + 2], key[4 * i + 3]);
  plan_cluster_sync();

  // all runs' sorted keys into shared memory, eight 16-byte loads in flight per thread
  uint32_t* all = reinterpret_cast<uint32_t*>(plan_smem);
  const uint4* src = reinterpret_cast<const uint4*>(run_keys);
  const int words4 = runs * R::RUN / 4;
  for (int j0 = 0; j0 < words4; j0 += 8 * PLAN_THREADS) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u * PLAN_THREADS + t;
      if (j < words4) v[u] = __ldcg(&src[j]);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u * PLAN_THREADS + t;
      if (j < words4) reinterpret_cast<uint4*>(all)[j] = v[u];
    }
  }
  __syncthreads();
  // merge ranks, the thread's rows searched together in each other run
  int pos[ITEMS];
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) pos[i] = t * ITEMS + i;
  for (int rr = 0; rr < runs; ++rr) {
    if (rr == r) continue;
    const uint32_t* run = all + rr * R::RUN;
    const bool inclusive = rr < r;
    int lo[ITEMS];
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) lo[i] = 0;
#pragma unroll
    for (int step = R::RUN >> 1; step > 0; step >>= 1) {
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        const uint32_t v = run[lo[i] + step - 1];
        if (v < key[i] || (inclusive && v == key[i])) lo[i] += step;
      }
    }
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const uint32_t v = run[lo[i]];
      pos[i] += lo[i] + ((v < key[i] || (inclusive && v == key[i])) ? 1 : 0);
    }
  }
  // rows out, and each tile's union of masks (ORed per tile locally first)
  uint32_t acc = 0;
  int acc_tile = -1;
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    if (pos[i] >= n) continue;
    row_order[pos[i]] = val[i];
    const int tile = pos[i] >> 7;
    if (tile != acc_tile) {
      if (acc_tile >= 0 && tile_order != nullptr) atomicOr(&tile_union[acc_tile], acc);
      acc_tile = tile;
      acc = 0;
    }
    acc |= key[i];
  }
  if (acc_tile >= 0 && tile_order != nullptr) atomicOr(&tile_union[acc_tile], acc);
  plan_cluster_sync();
  if (r != 0 || tile_order == nullptr) return;

  uint32_t* tkey = all;  // the merged keys are no longer needed
  for (int j = t; j < tiles; j += PLAN_THREADS)
    tkey[j] = 32u - (uint32_t)__popc(__ldcg(&tile_union[j]));
  __syncthreads();
  for (int j = t; j < tiles; j += PLAN_THREADS) {
    const uint32_t kj = tkey[j];
    int rank = 0;
    for (int m = 0; m < tiles; ++m) {
      const uint32_t km = tkey[m];
      rank += (km < kj) || (km == kj && m < j);
    }
    tile_order[rank] = j;
  }
}

template <int ITEMS>
int launch_plan_runs(const uint32_t* masks, int64_t n, int kvol, uint32_t* scratch,
                     int32_t* row_order, int32_t* tile_order, cudaStream_t s) {
  using R = PlanRuns<ITEMS>;
  const int runs = (int)((n + R::RUN - 1) / R::RUN);
  SV_CUDA_TRY(cudaFuncSetAttribute(plan_small_kernel<ITEMS>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)R::smem(R::MAX_RUNS)));
  if (R::MAX_RUNS > 8)
    SV_CUDA_TRY(cudaFuncSetAttribute(plan_small_kernel<ITEMS>,
                                     cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(runs);
  cfg.blockDim = dim3(PLAN_THREADS);
  cfg.dynamicSmemBytes = R::smem(runs);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = runs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SV_CUDA_TRY(cudaLaunchKernelEx(&cfg, plan_small_kernel<ITEMS>, masks, (int)n, kvol, scratch,
                                 scratch + PLAN_SMALL_ROWS, row_order, tile_order));
  return SV_OK;
}

// Whether this device can run a 16-CTA cluster of the 2048-row kernel (queried once per device).
bool plan_cluster16_ok() {
  static int known[256] = {};  // 0 unknown, 1 yes, 2 no
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) return false;
  if (known[dev] == 0) {
    using R = PlanRuns<8>;
    bool ok = cudaFuncSetAttribute(plan_small_kernel<8>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)R::smem(R::MAX_RUNS)) == cudaSuccess &&
              cudaFuncSetAttribute(plan_small_kernel<8>,
                                   cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
                  cudaSuccess;
    int clusters = 0;
    if (ok) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(R::MAX_RUNS);
      cfg.blockDim = dim3(PLAN_THREADS);
      cfg.dynamicSmemBytes = R::smem(R::MAX_RUNS);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = R::MAX_RUNS;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      ok = cudaOccupancyMaxActiveClusters(&clusters, plan_small_kernel<8>, &cfg) == cudaSuccess &&
           clusters >= 1;
    }
    cudaGetLastError();  // a refused query leaves no error behind
    known[dev] = ok ? 1 : 2;
  }
  return known[dev] == 1;
}

// masks: n row masks; scratch: PLAN_SMALL_ROWS words of run keys and the tile unions after them
// (16-byte aligned).
int launch_plan_small(const uint32_t* masks, int64_t n, int kvol, uint32_t* scratch,
                      int32_t* row_order, int32_t* tile_order, cudaStream_t s) {
  if (n <= 8 * PlanRuns<8>::RUN || plan_cluster16_ok())
    return launch_plan_runs<8>(masks, n, kvol, scratch, row_order, tile_order, s);
  return launch_plan_runs<16>(masks, n, kvol, scratch, row_order, tile_order, s);
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
  // warp, then CTA reduction: one atomic per CTA and value (atomics from every warp on the same
  // 8 words serialise in L2)
  __shared__ int32_t part[8][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    mn[j] = __reduce_min_sync(0xffffffffu, mn[j]);
    mx[j] = __reduce_max_sync(0xffffffffu, mx[j]);
  }
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      part[j][warp] = mn[j];
      part[4 + j][warp] = mx[j];
    }
  }
  __syncthreads();
  if (warp < 8) {
    int32_t v = lane < warps ? part[warp][lane] : (warp < 4 ? INT32_MAX : INT32_MIN);
    v = warp < 4 ? __reduce_min_sync(0xffffffffu, v) : __reduce_max_sync(0xffffffffu, v);
    if (lane == 0) {
      if (warp < 4) atomicMin(&bounds[warp], v);
      else atomicMax(&bounds[warp], v);
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

// ---- automatic choice on the device ------------------------------------------------------------
// sv_kmap_build_auto reads the coordinates' bounding box on the device. Every later kernel of the
// build derives from those 8 words the same choice, with no host synchronisation: a dense grid
// when the box holds at most AUTO_GRID_CELLS_PER_ROW cells per row and fits the workspace, the hash
// table (block table for 3x3x3 dilation-1 maps, voxel table otherwise) when it does not. For a
// 3x3x3 dilation-1 map the grid is one of 2x2x2 blocks, laid out like the block table's cells
// (8 rows in one 32-byte sector per block, blocks in (batch, c1 >> 1, c2 >> 1, c3 >> 1) order),
// so a row's 27 neighbours are 8 sectors; otherwise a grid of single voxels.
constexpr int64_t AUTO_GRID_CELLS_PER_ROW = 16;
constexpr int64_t AUTO_GRID_MIN_ROWS = 1 << 17;
constexpr size_t AUTO_HEADER = 256;  // bytes before the table: the bounds words

struct AutoPlan {
  bool grid;
  GridBox g;  // voxel grid: cells; block grid: blocks (batch extent in rows, c1..c3 in blocks)
  int64_t cells;
};

__device__ __forceinline__ AutoPlan auto_plan(const int32_t* __restrict__ bounds, int64_t n,
                                              int64_t cap_cells, bool blocks) {
  AutoPlan p;
  p.cells = blocks ? 8 : 1;
  p.grid = true;
  const int64_t limit = min(cap_cells, AUTO_GRID_CELLS_PER_ROW * n);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int32_t lo = __ldg(&bounds[j]), hi = __ldg(&bounds[4 + j]);
    if (blocks && j > 0) {
      lo >>= 1;
      hi >>= 1;
    }
    const int64_t ext = (int64_t)hi - lo + 1;
    p.g.lo[j] = lo;
    p.g.ext[j] = ext;
    if (p.grid && ext >= 1 && p.cells <= limit / ext) p.cells *= ext;
    else p.grid = false;
  }
  return p;
}

// Fills the grid (cells x 4 bytes) or the hash table (hash_bytes) with 0xFF bytes.
__global__ void auto_clear_kernel(const int32_t* __restrict__ bounds, int64_t n, int64_t cap_cells,
                                  bool blocks, int4* region, int64_t hash_bytes) {
  const AutoPlan p = auto_plan(bounds, n, cap_cells, blocks);
  const int64_t words4 = ((p.grid ? p.cells * 4 : hash_bytes) + 15) / 16;
  const int4 ones = make_int4(-1, -1, -1, -1);
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < words4;
       j += (int64_t)gridDim.x * blockDim.x)
    region[j] = ones;
}

// Index of block (b, g1, g2, g3) in the block grid, or -1 outside the box.
__device__ __forceinline__ int64_t grid_block(const GridBox& g, int64_t b, int64_t g1, int64_t g2,
                                              int64_t g3) {
  b -= g.lo[0];
  g1 -= g.lo[1];
  g2 -= g.lo[2];
  g3 -= g.lo[3];
  if ((uint64_t)b >= (uint64_t)g.ext[0] || (uint64_t)g1 >= (uint64_t)g.ext[1] ||
      (uint64_t)g2 >= (uint64_t)g.ext[2] || (uint64_t)g3 >= (uint64_t)g.ext[3])
    return -1;
  return ((b * g.ext[1] + g1) * g.ext[2] + g2) * g.ext[3] + g3;
}

__global__ void auto_insert_kernel(const int4* __restrict__ coords, int64_t n,
                                   const int32_t* __restrict__ bounds, int64_t cap_cells,
                                   void* region, int64_t slots, bool blocks, int32_t* status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const AutoPlan p = auto_plan(bounds, n, cap_cells, blocks);
  const int4 c = __ldg(&coords[i]);
  const uint32_t mask = (uint32_t)(slots - 1);
  int32_t* grid = static_cast<int32_t*>(region);
  if (p.grid && blocks) {
    const int64_t blk = grid_block(p.g, c.x, c.y >> 1, c.z >> 1, c.w >> 1);
    const int cell = ((c.y & 1) << 2) | ((c.z & 1) << 1) | (c.w & 1);
    if (blk >= 0) atomicMax(grid + blk * 8 + cell, (int32_t)i);
    else report(status, SV_DEVICE_BAD_INDEX);  // outside its own bounding box: cannot happen
  } else if (p.grid) {
    int64_t cell;
    if (grid_cell(p.g, c.x, c.y, c.z, c.w, &cell)) atomicMax(grid + cell, (int32_t)i);
    else report(status, SV_DEVICE_BAD_INDEX);
  } else if (blocks) {
    int4* keys = static_cast<int4*>(region);
    block_insert(c, i, keys, reinterpret_cast<int32_t*>(keys + slots), mask, status);
  } else {
    voxel_insert(coords, i, c, grid, mask, status);
  }
}

// 3x3x3, dilation 1: one thread per row, as kmap_block_probe_kernel; the row's 8 blocks come from
// the block grid (one sector each, the index of block s is that of block 0 plus s's steps) or
// from the block table.
__global__ void __launch_bounds__(PROBE_ROWS)
    auto_probe333_kernel(const int4* __restrict__ coords, int64_t n,
                         const int32_t* __restrict__ bounds, int64_t cap_cells,
                         const void* __restrict__ region, int64_t slots,
                         int32_t* __restrict__ nbr) {
  __shared__ int32_t stage[PROBE_ROWS * 27];
  const AutoPlan p = auto_plan(bounds, n, cap_cells, true);
  const int64_t row0 = (int64_t)blockIdx.x * PROBE_ROWS;
  if (row0 + threadIdx.x < n) {
    const int4 c = __ldg(&coords[row0 + threadIdx.x]);
    int32_t* row_stage = stage + threadIdx.x * 27;
    if (p.grid) {
      const RowBlocks rb = row_blocks(c);
      // block 0 relative to the box; side s along an axis is in the box when 0 <= rel + s < ext
      int64_t rel[3];
      bool in[3][2];
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        rel[a] = rb.g[a] - p.g.lo[a + 1];
#pragma unroll
        for (int sd = 0; sd < 2; ++sd)
          in[a][sd] = rb.ok[a][sd] && (uint64_t)(rel[a] + sd) < (uint64_t)p.g.ext[a + 1];
      }
      const int64_t s3 = p.g.ext[3], s2 = p.g.ext[2] * s3;
      const int64_t base = (((int64_t)c.x - p.g.lo[0]) * p.g.ext[1] + rel[0]) * s2 +
                           rel[1] * s3 + rel[2];
      const int4* grid4 = static_cast<const int4*>(region);
      int4 lo[8], hi[8];
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        const int s0 = b >> 2, s1 = (b >> 1) & 1, sb = b & 1;
        lo[b] = make_int4(-1, -1, -1, -1);
        hi[b] = lo[b];
        if (in[0][s0] && in[1][s1] && in[2][sb]) {
          const int64_t blk = base + s0 * s2 + s1 * s3 + sb;
          lo[b] = __ldg(grid4 + 2 * blk);
          hi[b] = __ldg(grid4 + 2 * blk + 1);
        }
      }
      emit_window(c, lo, hi, row_stage);
    } else {
      const int4* keys = static_cast<const int4*>(region);
      block_probe_row(c, keys, keys + slots, (uint32_t)(slots - 1), row_stage);
    }
  }
  flush_rows(stage, n, row0, nbr);
}

// Any kernel and dilation: one thread per (row, offset), on the grid or the voxel table.
__global__ void auto_probe_kernel(const int4* __restrict__ coords, int64_t n,
                                  const int32_t* __restrict__ bounds, int64_t cap_cells,
                                  const int32_t* __restrict__ region, int64_t slots, int k0,
                                  int k1, int k2, int d0, int d1, int d2,
                                  int32_t* __restrict__ nbr) {
  const int kvol = k0 * k1 * k2;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * kvol) return;
  const AutoPlan p = auto_plan(bounds, n, cap_cells, false);
  const int64_t row = idx / kvol;
  const int4 q = __ldg(&coords[row]);
  int32_t x, y, z, r = -1;
  if (offset_coord(q, (int)(idx - row * kvol), k0, k1, k2, d0, d1, d2, &x, &y, &z)) {
    if (p.grid) {
      int64_t cell;
      if (grid_cell(p.g, q.x, x, y, z, &cell)) r = __ldg(&region[cell]);
    } else {
      r = kmap_lookup(coords, region, (uint32_t)(slots - 1), q.x, x, y, z);
    }
  }
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
  // at least 2 slots per row: a load factor of at most 1/2 for the voxel table (one slot per
  // distinct row) and for the block table (one slot per occupied block, at most one per row)
  int64_t slots = 64;
  while (slots < 2 * n) slots <<= 1;
  return slots;
}

extern "C" size_t sv_kmap_workspace_bytes(int64_t table_slots) {
  // block table: a 16-byte key and 8 four-byte cells per slot (the voxel table needs 4 bytes)
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
  int4* cells4 = keys + table_slots;
  SV_CUDA_TRY(cudaMemsetAsync(keys, 0xFF, (size_t)table_slots * 48, s));
  kmap_block_insert_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const int4*>(coords), n, keys, reinterpret_cast<int32_t*>(cells4), mask,
      status);
  SV_LAUNCH_CHECK();
  kmap_block_probe_kernel<<<(unsigned)((n + PROBE_ROWS - 1) / PROBE_ROWS), PROBE_ROWS, 0, s>>>(
      reinterpret_cast<const int4*>(coords), n, keys, cells4, mask, nbr);
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

extern "C" size_t sv_kmap_auto_workspace_bytes(int64_t n) {
  if (n <= 0) return 0;
  const size_t hash = sv_kmap_workspace_bytes(sv_kmap_table_slots(n));
  const size_t grid = align_up((size_t)(AUTO_GRID_CELLS_PER_ROW * n) * 4, 16);
  return AUTO_HEADER + std::max(hash, grid);
}

extern "C" int sv_kmap_build_auto(const int32_t* coords, int64_t n, const int32_t kernel[3],
                                  const int32_t dilation[3], int32_t* nbr, void* workspace,
                                  size_t workspace_bytes, int32_t* status, sv_stream_t stream) {
  const int64_t slots = sv_kmap_table_slots(n);
  const int rc = kmap_check(coords, n, kernel, dilation, nbr, slots);
  if (rc != SV_OK || n == 0) return rc;
  if (workspace == nullptr || workspace_bytes < sv_kmap_auto_workspace_bytes(n))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_kmap_build_auto: workspace too small");
  if (reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_kmap_build_auto: workspace must be 16-byte aligned");
  cudaStream_t s = to_stream(stream);
  const bool k333 = kernel[0] == 3 && kernel[1] == 3 && kernel[2] == 3 && dilation[0] == 1 &&
                    dilation[1] == 1 && dilation[2] == 1;
  int32_t* bounds = static_cast<int32_t*>(workspace);
  uint8_t* region = static_cast<uint8_t*>(workspace) + AUTO_HEADER;
  // A small table stays in L2 and the two launches that read the box cost more than the grid
  // saves: below AUTO_GRID_MIN_ROWS rows the hash table is built directly.
  if (n < AUTO_GRID_MIN_ROWS) {
    if (k333) return kmap_build_blocks(coords, n, nbr, slots, region, status, s);
    return kmap_build_voxels(coords, n, kernel, dilation, nbr, slots,
                             reinterpret_cast<int32_t*>(region), status, s);
  }
  // grid capacity: whole 16-byte words of the region after the header
  const int64_t cap_cells = (int64_t)((workspace_bytes - AUTO_HEADER) / 16) * 4;
  const int64_t hash_bytes = k333 ? slots * 48 : slots * 4;
  const int4* c4 = reinterpret_cast<const int4*>(coords);
  bounds4_init_kernel<<<1, 32, 0, s>>>(bounds);
  SV_LAUNCH_CHECK();
  bounds4_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 4 * num_sms()), 256, 0, s>>>(
      c4, n, bounds);
  SV_LAUNCH_CHECK();
  auto_clear_kernel<<<(unsigned)(4 * num_sms()), 256, 0, s>>>(
      bounds, n, cap_cells, k333, reinterpret_cast<int4*>(region), hash_bytes);
  SV_LAUNCH_CHECK();
  auto_insert_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(c4, n, bounds, cap_cells, region,
                                                                 slots, k333, status);
  SV_LAUNCH_CHECK();
  if (k333) {
    auto_probe333_kernel<<<(unsigned)((n + PROBE_ROWS - 1) / PROBE_ROWS), PROBE_ROWS, 0, s>>>(
        c4, n, bounds, cap_cells, region, slots, nbr);
  } else {
    const int64_t total = n * (int64_t)kernel[0] * kernel[1] * kernel[2];
    auto_probe_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
        c4, n, bounds, cap_cells, reinterpret_cast<const int32_t*>(region), slots, kernel[0],
        kernel[1], kernel[2], dilation[0], dilation[1], dilation[2], nbr);
  }
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
  // row masks, sorted masks, row ids; tile keys, sorted tile keys, tile ids; CUB scratch (the
  // one-cluster schedule's run keys and sorted masks for small maps)
  return align_up((size_t)n * 4, 256) * 3 + align_up((size_t)tiles * 4, 256) * 3 +
         align_up(std::max({plan_cub_bytes(n), plan_tile_cub_bytes(tiles),
                            n <= PLAN_SMALL_ROWS ? (size_t)2 * PLAN_SMALL_ROWS * 4 : (size_t)0}),
                  256);
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
  if (n <= PLAN_SMALL_ROWS)  // sorted masks and run keys in the sort's scratch
    return launch_plan_small(masks, n, kvol, reinterpret_cast<uint32_t*>(cub_tmp), row_order,
                             tile_order, s);
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
