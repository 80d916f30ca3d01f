// Narrow-channel sparse convolution with deduplicated source rows and the A operand in TMEM
// (tcgen05, sm_100a).
//
// Same result as conv_tc.cu (the Metal kernel of src/mlx_diffuser/kernels/sparse.py:14-34 for
// fp16/bf16 features, fp32 accumulation): out[p, o] = bias[o] + sum over offsets k with
// nbr[p,k] >= 0 of features[nbr[p,k]] . W[k][:, o].
//
// Why a second kernel. For Cin <= 128 the per-stage MMA work is small and conv_tc.cu is bound by
// the rate at which one SM's scattered 16-byte row copies are served: every source row is
// fetched once per (tile, offset), about 20 times in all on a surface. Here a tile is 128 rows
// that are neighbours in space (Morton order), so its 27 x 128 neighbour references name only
// ~2 x 128 distinct rows. The plan (built once per map, like the map itself) lists them; the
// kernel gathers each of them once into shared memory and builds every A operand from there.
//
// Per work item (one 128-row tile x BN output channels):
//   warps 2-5   loaders: take the next item from the persistent scheduler, read its plan
//               record, output rows and source-row indices, cp.async its local map [128][27]
//               (int16) and its unique source rows (CIN * 2 bytes each, at most 56 KB) into one
//               of two buffers once the A builders are done with it, then publish its output
//               rows and offset mask once the epilogue is done with the previous ones;
//   warps 10-   A builders, two groups of four warps at 64 input channels, three at 128; in a
//               group one tile row per thread, and group g takes the stages whose index is g
//               modulo the group count: for each (offset, 64-channel block) read the row's
//               128 bytes from the shared buffer (chunks XOR-swizzled by the slot, so the sources
//               of neighbouring rows -- consecutive slots -- use different bank groups) and
//               store them with tcgen05.st into a TMEM stage (32 columns: 64 bf16/fp16 values
//               per lane); the group's next row is read while this one's store completes;
//   warp 0      TMA producer: the B tile W[k][kb*64 : +64, n0 : n0+BN] per stage (as conv_tc);
//   warp 1      TMEM allocator and MMA issuer: tcgen05.mma with A from TMEM, B from shared
//               memory (4 x K=16 per 64-channel block, up to four blocks and one commit per
//               stage), accumulators double-buffered in TMEM;
//   warps 6-9   epilogue (as conv_tc): tcgen05.ld, + bias (+ residual), round, store.
// A local-map entry is the row's slot in the shared buffer, -1 for a missing neighbour, or -2
// when the tile had more distinct rows than the buffer holds: that row is then read from global
// memory through the kernel map.
//
// Every wait is bounded (2 s, plus a CTA-wide abort flag); on expiry the kernel ORs
// SV_DEVICE_WAIT_TIMEOUT into the status word, drains its copies and frees TMEM.
#include <algorithm>
#include <type_traits>

#include <cub/block/block_radix_sort.cuh>
#include <cub/block/block_scan.cuh>
#include <cub/device/device_radix_sort.cuh>

#include "conv.h"

namespace sv {
namespace {

constexpr int DTBM = 128;     // tile rows == TMEM lanes
constexpr int DKVOL = 27;     // 3 x 3 x 3 only
constexpr int DLT = 128;         // loader threads (warps 2-5)
constexpr int DEPI0 = 6;         // first epilogue warp
constexpr int DBLD0 = 10;        // first A-builder warp
// A-builder groups of four warps; group g builds the pipeline stages whose index is g modulo the
// group count. One group alone waits on its own TMEM stores and shared-memory reads; two (three
// at 128 input channels, where a stage is one offset) keep stages in flight while it waits.
__host__ __device__ constexpr int dd_groups(int cin) { return cin == 64 ? 2 : 3; }
__host__ __device__ constexpr int dd_threads(int cin) { return 32 * (DBLD0 + 4 * dd_groups(cin)); }
// One source-row buffer: 448 rows at 64 input channels (p99 of a Morton tile's distinct rows on
// surface scenes is ~450), leaving room for three four-offset B stages (96 KB).
constexpr int DEDUP_BYTES = 56 * 1024;
constexpr int LOADER_BAR = 2;           // named barrier of the four loader warps

__host__ __device__ constexpr int dd_umax(int cin) { return DEDUP_BYTES / (cin * 2); }

// ---- plan layout (caller memory, cached with the map) ----------------------------------------
// [rows: tiles*128 int32][lnbr: tiles*128*27 int16][src: tiles*umax int32][meta: tiles int4]
struct PlanView {
  int32_t* rows;
  int16_t* lnbr;
  int32_t* src;
  int4* meta;  // x = distinct rows kept (<= umax), y = offset mask, z = distinct rows, w = 0
};

__host__ __device__ inline size_t dd_align(size_t v) { return (v + 255) / 256 * 256; }

__host__ __device__ inline size_t dd_plan_bytes(int64_t tiles, int cin) {
  return dd_align((size_t)tiles * DTBM * 4) + dd_align((size_t)tiles * DTBM * DKVOL * 2) +
         dd_align((size_t)tiles * dd_umax(cin) * 4) + dd_align((size_t)tiles * 16);
}

template <typename P>
__host__ __device__ inline PlanView dd_plan_view(P* base, int64_t tiles, int cin) {
  uint8_t* p = (uint8_t*)base;
  PlanView v;
  v.rows = (int32_t*)p;
  p += dd_align((size_t)tiles * DTBM * 4);
  v.lnbr = (int16_t*)p;
  p += dd_align((size_t)tiles * DTBM * DKVOL * 2);
  v.src = (int32_t*)p;
  p += dd_align((size_t)tiles * dd_umax(cin) * 4);
  v.meta = (int4*)p;
  return v;
}

// ---- planner ----------------------------------------------------------------------------------

__device__ __forceinline__ uint64_t spread3(uint32_t v) {  // low 16 bits -> every third bit
  uint64_t x = v & 0xFFFFu;
  x = (x | (x << 32)) & 0x1F00000000FFFFull;
  x = (x | (x << 16)) & 0x1F0000FF0000FFull;
  x = (x | (x << 8)) & 0x100F00F00F00F00Full;
  x = (x | (x << 4)) & 0x10C30C30C30C30C3ull;
  x = (x | (x << 2)) & 0x1249249249249249ull;
  return x;
}

// Sort key of a row: batch (15 bits) above the Morton code of the low 16 bits of (c1, c2, c3).
// Only locality depends on it: coordinates outside [0, 65536) still sort, just less compactly.
__global__ void dd_morton_kernel(const int4* __restrict__ coords, int64_t n,
                                 uint64_t* __restrict__ keys, int32_t* __restrict__ rows) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int4 c = __ldg(&coords[i]);
  keys[i] = ((uint64_t)((uint32_t)c.x & 0x7FFFu) << 48) | (spread3((uint32_t)c.y) << 2) |
            (spread3((uint32_t)c.z) << 1) | spread3((uint32_t)c.w);
  rows[i] = (int32_t)i;
}

// rank[row] = the row's position in Morton order.
__global__ void dd_rank_kernel(const int32_t* __restrict__ sorted_rows, int64_t n,
                               int32_t* __restrict__ rank) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) rank[sorted_rows[i]] = (int32_t)i;
}

// One CTA per tile: the tile's 128 rows (Morton order), the distinct rows their 27 neighbour
// references name, and each reference's slot among them. Slots follow the Morton order of the
// source rows, so the sources of neighbouring tile rows at one offset mostly sit in
// consecutive slots; the kernel swizzles a row's 16-byte chunks by (slot & 7), and consecutive
// slots then fall in different shared-memory bank groups.
template <int UMAX>
__global__ void __launch_bounds__(DTBM)
    dd_plan_tile_kernel(const int32_t* __restrict__ nbr, int64_t n,
                        const int32_t* __restrict__ sorted_rows,
                        const int32_t* __restrict__ rank, PlanView plan, int32_t* status) {
  using Sort = cub::BlockRadixSort<uint32_t, DTBM, DKVOL>;
  using Scan = cub::BlockScan<int32_t, DTBM>;
  __shared__ union {
    typename Sort::TempStorage sort;
    typename Scan::TempStorage scan;
    uint32_t sorted[DTBM * DKVOL];
  } sm;
  __shared__ uint32_t uniq[DTBM * DKVOL];
  __shared__ uint32_t s_mask;
  __shared__ int32_t s_total;

  const int64_t t = blockIdx.x;
  const int r = threadIdx.x;
  const int64_t gr = t * DTBM + r;
  const int32_t orow = gr < n ? sorted_rows[gr] : -1;
  plan.rows[gr] = orow;
  if (r == 0) s_mask = 0;
  uint32_t keys[DKVOL];  // Morton ranks of the sources; a missing neighbour sorts last
  uint32_t mask = 0;
#pragma unroll
  for (int k = 0; k < DKVOL; ++k) {
    int32_t v = orow >= 0 ? __ldg(&nbr[(int64_t)orow * DKVOL + k]) : -1;
    if (v >= n) {
      report(status, SV_DEVICE_BAD_INDEX);
      v = -1;
    }
    keys[k] = v >= 0 ? (uint32_t)__ldg(&rank[v]) : 0xFFFFFFFFu;
    mask |= (uint32_t)(v >= 0) << k;
  }
  __syncthreads();
  atomicOr(&s_mask, mask);
  Sort(sm.sort).Sort(keys);
  __syncthreads();
#pragma unroll
  for (int i = 0; i < DKVOL; ++i) sm.sorted[r * DKVOL + i] = keys[i];
  __syncthreads();
  int32_t flags[DKVOL];
#pragma unroll
  for (int i = 0; i < DKVOL; ++i) {
    const int pos = r * DKVOL + i;
    const bool first = pos == 0 || sm.sorted[pos - 1] != keys[i];
    flags[i] = (keys[i] != 0xFFFFFFFFu && first) ? 1 : 0;
  }
  __syncthreads();  // sm.sorted is dead; its storage becomes the scan's
  int32_t slot[DKVOL];
  int32_t total = 0;
  Scan(sm.scan).ExclusiveSum(flags, slot, total);
#pragma unroll
  for (int i = 0; i < DKVOL; ++i)
    if (flags[i]) uniq[slot[i]] = keys[i];
  if (r == 0) s_total = total;
  __syncthreads();
  const int32_t u = s_total;
  for (int j = r; j < UMAX; j += DTBM)
    plan.src[t * UMAX + j] = j < u ? __ldg(&sorted_rows[uniq[j]]) : -1;
  // each reference's slot: binary search of its rank among the tile's ascending distinct ranks
  int16_t* ln = plan.lnbr + gr * DKVOL;
#pragma unroll 1
  for (int k = 0; k < DKVOL; ++k) {
    int32_t v = orow >= 0 ? __ldg(&nbr[(int64_t)orow * DKVOL + k]) : -1;
    int16_t e = -1;
    if (v >= 0 && v < n) {
      const uint32_t key = (uint32_t)__ldg(&rank[v]);
      int lo = 0, hi = u - 1;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (uniq[mid] < key) lo = mid + 1;
        else hi = mid;
      }
      e = lo < UMAX ? (int16_t)lo : (int16_t)-2;
    }
    ln[k] = e;
  }
  if (r == 0) plan.meta[t] = make_int4(min(u, UMAX), (int32_t)s_mask, u, 0);
}

size_t dd_sort_bytes(int64_t n) {
  size_t bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const uint64_t*)nullptr, (uint64_t*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, (int)n, 0, 63);
  return bytes;
}

// ---- the convolution --------------------------------------------------------------------------

// P: 64-channel K blocks per pipeline stage. At 64 input channels and BN <= 64 four offsets
// share a stage (16 MMAs and one commit, 32 KB of B for BN = 64; three such stages fill TMEM
// beside the two accumulators). Each stage carries a fixed cost -- the commit and the pipeline
// drain it waits for, the barrier round trips, the builders' TMEM store wait -- that measured
// ~700 cycles against ~42 per 128 x 64 x 16 MMA, so fewer, larger stages pay.
__host__ __device__ constexpr int dd_blocks_per_stage(int cin, int bn) {
  return (cin == 64 && bn <= 64) ? 4 : 1;
}

template <int BN, int P>
struct DdLayout {
  static constexpr int STAGES = P == 4 ? 3 : BN <= 32 ? 8 : BN <= 64 ? 6 : 4;
  static constexpr int B_SUB_BYTES = BN * 128;  // one 64-channel block of B
  static constexpr int B_STAGE_BYTES = P * B_SUB_BYTES;
  static constexpr uint32_t A_STAGE_COLS = 32 * P;  // TMEM columns of one stage's A
  static constexpr int B_OFF = 0;
  static constexpr int DEDUP_OFF = B_OFF + STAGES * B_STAGE_BYTES;
  static constexpr int LNBR_OFF = DEDUP_OFF + 2 * DEDUP_BYTES;
  static constexpr int LNBR_BYTES = DTBM * DKVOL * 2;  // 6912 = 432 x 16
  static constexpr int OROW_OFF = LNBR_OFF + 2 * LNBR_BYTES;
  static constexpr int SLOT_OFF = OROW_OFF + 2 * DTBM * 4;
  static constexpr int MISC_OFF = SLOT_OFF + 2 * 16;
  static constexpr int BAR_OFF = MISC_OFF + 32;
  static constexpr int NUM_BARS = 2 * STAGES + 12;
  static constexpr int BYTES = BAR_OFF + NUM_BARS * 8;
  static constexpr int SMEM = BYTES + 1024;
  static constexpr uint32_t ACC_COLS = 2 * BN;
  static constexpr uint32_t A_COL0 = ACC_COLS;
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(A_COL0 + A_STAGE_COLS * STAGES <= TMEM_COLS, "TMEM budget");
  static_assert(B_STAGE_BYTES % 1024 == 0, "swizzle atoms");
  static_assert(LNBR_BYTES % 16 == 0, "16-byte copies of the local map");
  static_assert(BAR_OFF % 8 == 0, "mbarrier alignment");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

struct DdSlot {
  int32_t item;   // < 0: no more work
  int32_t n0;
  uint32_t umask;
  int32_t tile;
};

struct DdSched {
  int32_t* counter;
  int32_t tiles;
  int32_t total_items;  // tiles * (cout / BN), n-slab major
};

__device__ __forceinline__ void mbar_arrive_dd(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool loader_bar_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "n"(LOADER_BAR), "n"(DLT)
      : "memory");
  return r != 0;
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16, A K-major in TMEM (lane = row, two 16-bit
// values per 32-bit column, the lower K index in the low half).
__device__ __forceinline__ void tc_mma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns from registers: lane (base + t) receives thread t's
// r[0..31] in columns col .. col+31.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tc_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

template <typename T>
__device__ __forceinline__ uint32_t dd_pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// The item's 64-channel K blocks in order: offsets of the mask, KB blocks each.
struct SubStages {
  uint32_t m;
  int kb;
  __device__ __forceinline__ bool next(int KB, int* k, int* b) {
    if (m == 0) return false;
    *k = __ffs(m) - 1;
    *b = kb;
    if (++kb == KB) {
      kb = 0;
      m &= m - 1;
    }
    return true;
  }
};

template <int BN, int CIN, typename T, bool kResidual>
__global__ void __launch_bounds__(dd_threads(CIN), 1)
    conv_dd_kernel(const __grid_constant__ CUtensorMap tmap_w, const T* __restrict__ feat,
                   int n, const int32_t* __restrict__ nbr, PlanView plan,
                   const T* __restrict__ bias, const T* residual, int cout, T* out, DdSched sc,
                   int32_t* status) {
  constexpr int P = dd_blocks_per_stage(CIN, BN);
  constexpr int DGROUPS = dd_groups(CIN);
  using L = DdLayout<BN, P>;
  constexpr int S = L::STAGES;
  constexpr int UMAX = dd_umax(CIN);
  constexpr int ROWB = CIN * 2;
  constexpr int KB = CIN / 64;  // 64-channel K stages per offset
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sB = smem + L::B_OFF;
  uint8_t* sDedup = smem + L::DEDUP_OFF;
  int16_t* s_lnbr = reinterpret_cast<int16_t*>(smem + L::LNBR_OFF);
  int32_t* s_orow = reinterpret_cast<int32_t*>(smem + L::OROW_OFF);
  DdSlot* slots = reinterpret_cast<DdSlot*>(smem + L::SLOT_OFF);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  int32_t* s_fetch = reinterpret_cast<int32_t*>(smem + L::MISC_OFF + 8);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  // One arrival per warp wherever a warp finishes a step together (after __syncwarp): an
  // mbarrier takes its arrivals one at a time, and 128 per stage cost more than a narrow
  // stage's MMAs.
  uint64_t* full = bars;                     // [S]: TMA expect_tx + one group's 4 builder warps
  uint64_t* empty = bars + S;                // [S]: tcgen05.commit
  uint64_t* acc_full = bars + 2 * S;         // [2]: tcgen05.commit
  uint64_t* acc_empty = acc_full + 2;        // [2]: 4 epilogue warps
  uint64_t* meta_full = acc_empty + 2;       // [2]: the first loader (rows, slot published)
  uint64_t* dedup_full = meta_full + 2;      // [2]: 128 loaders' cp.async (local map + rows)
  uint64_t* buf_empty = dedup_full + 2;      // [2]: the A-builder warps (local map + rows read)
  uint64_t* meta_empty = buf_empty + 2;      // [2]: 4 epilogue warps (output rows read)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1 + 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
      mbar_init(&meta_full[b], 1);
      mbar_init(&dedup_full[b], DLT);
      mbar_init(&buf_empty[b], 4 * DGROUPS);
      mbar_init(&meta_empty[b], 4);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&tmap_w);
  if (warp == 1) {
    tmem_alloc(s_tmem, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  bool ok = true;

  if (warp == 0) {
    // ---- TMA producer (B operand) ----
    if (lane == 0) {
      int it = 0;
      for (int local = 0; ok; ++local) {
        const int ws = local & 1;
        if (!mbar_wait_bounded(&meta_full[ws], (local >> 1) & 1, s_abort)) {
          ok = false;
          break;
        }
        const DdSlot w = slots[ws];
        if (w.item < 0) break;
        SubStages sub{w.umask, 0};
        for (; ok; ++it) {
          int k[P], kb[P], cnt = 0;
          for (int j = 0; j < P && sub.next(KB, &k[j], &kb[j]); ++j) ++cnt;
          if (cnt == 0) break;
          const int slot = it % S;
          if (!mbar_wait_bounded(&empty[slot], ((it / S) & 1) ^ 1, s_abort)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[slot], (uint32_t)(cnt * L::B_SUB_BYTES));
          for (int j = 0; j < cnt; ++j)
            tma_load_2d(smem_u32(sB + slot * L::B_STAGE_BYTES + j * L::B_SUB_BYTES), &tmap_w,
                        &full[slot], k[j] * CIN + kb[j] * 64, w.n0);
        }
      }
      if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kBF16, DTBM, BN);
      int it = 0;
      for (int local = 0; ok; ++local) {
        const int ws = local & 1;
        if (!mbar_wait_bounded(&meta_full[ws], (local >> 1) & 1, s_abort)) {
          ok = false;
          break;
        }
        const DdSlot w = slots[ws];
        if (w.item < 0) break;
        const int ab = local & 1;
        if (!mbar_wait_bounded(&acc_empty[ab], ((local >> 1) & 1) ^ 1, s_abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * BN);
        int first = 1;
        SubStages sub{w.umask, 0};
        for (; ok; ++it) {
          int k, kb, cnt = 0;
          for (int j = 0; j < P && sub.next(KB, &k, &kb); ++j) ++cnt;
          if (cnt == 0) break;
          const int slot = it % S;
          if (!mbar_wait_bounded(&full[slot], (it / S) & 1, s_abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int j = 0; j < cnt; ++j) {
            const uint32_t a0 = tmem + L::A_COL0 + (uint32_t)(slot * L::A_STAGE_COLS + j * 32);
            const uint32_t b0 = smem_u32(sB + slot * L::B_STAGE_BYTES + j * L::B_SUB_BYTES);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_ts_f16(d, a0 + (uint32_t)(kk * 8), smem_desc_kmajor(b0 + kk * 32, 2u, 128u),
                            idesc, (first && kk == 0) ? 0u : 1u);
            first = 0;
          }
          tc_commit(&empty[slot]);
        }
        tc_commit(&acc_full[ab]);  // also after a timeout, so the epilogue never waits on nothing
      }
      if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else if (warp < DEPI0) {
    // ---- loaders ----
    // CPR 16-byte chunks per source row; loader g copies chunk g % CPR of buffer rows
    // g / CPR + RPP * i (a warp instruction writes 32 / CPR whole rows: conflict-free)
    constexpr int CPR = ROWB / 16;
    constexpr int RPP = DLT / CPR;
    const int g = threadIdx.x - 64;
    const int chunk = g % CPR;
    const int row0 = g / CPR;
    for (int local = 0;; ++local) {
      const int ws = local & 1;
      if (g == 0) *s_fetch = atomicAdd(sc.counter, 1);
      // the fetched item is visible; a loader whose previous wait expired makes all leave
      if (loader_bar_any(!ok)) {
        ok = false;
        break;
      }
      const int32_t item = *s_fetch;
      const bool valid = item < sc.total_items;
      // Everything that does not need the buffer is read before waiting for it: the tile's
      // output rows, its plan record and the first batch of source-row indices.
      constexpr int ORPT = (DTBM + DLT - 1) / DLT;
      constexpr int PASSES = (UMAX + RPP - 1) / RPP;
      constexpr int BATCH = PASSES > 28 ? 28 : PASSES;
      int32_t tile = 0;
      int4 meta = make_int4(0, 0, 0, 0);
      int32_t orows[ORPT];
      int32_t srows[BATCH];
      const int32_t nt = valid ? item / sc.tiles : 0;
      if (valid) {
        tile = item - nt * sc.tiles;
#pragma unroll
        for (int j = 0; j < ORPT; ++j) {
          const int i = g + j * DLT;
          orows[j] = i < DTBM ? __ldg(&plan.rows[(int64_t)tile * DTBM + i]) : -1;
        }
        meta = __ldg(&plan.meta[tile]);
      }
      const int count = min(meta.x, UMAX);
      const int32_t* src_rows = plan.src + (int64_t)tile * UMAX;
#pragma unroll
      for (int i = 0; i < BATCH; ++i) {
        const int r = row0 + RPP * i;
        srows[i] = r < count ? __ldg(&src_rows[r]) : -1;
      }
      // The local map and rows go into the buffer as soon as the A builders are done with it;
      // the output rows and the slot record wait for the epilogue of the tile that used them.
      const uint32_t ph = ((local >> 1) & 1) ^ 1;
      bool fail = loader_bar_any(!mbar_wait_bounded(&buf_empty[ws], ph, s_abort));
      if (valid && !fail) {
        const uint32_t lnbr_dst = smem_u32(s_lnbr + ws * DTBM * DKVOL);
        const uint8_t* lnbr_src =
            reinterpret_cast<const uint8_t*>(plan.lnbr + (int64_t)tile * DTBM * DKVOL);
#pragma unroll
        for (int c = g; c < L::LNBR_BYTES / 16; c += DLT)
          cp_async_16(lnbr_dst + (uint32_t)(c * 16), lnbr_src + c * 16, 16u);
        const uint32_t buf = smem_u32(sDedup + ws * DEDUP_BYTES);
#pragma unroll 1
        for (int i0 = 0; i0 < PASSES && row0 + RPP * i0 < count; i0 += BATCH) {
          if (i0 > 0) {
#pragma unroll
            for (int i = 0; i < BATCH; ++i) {
              const int r = row0 + RPP * (i0 + i);
              srows[i] = r < count ? __ldg(&src_rows[r]) : -1;
            }
          }
#pragma unroll
          for (int i = 0; i < BATCH; ++i) {
            const int r = row0 + RPP * (i0 + i);
            if (r >= count) break;
            int32_t srow = srows[i];
            uint32_t bytes = 16u;
            if (srow < 0 || srow >= n) {
              report(status, SV_DEVICE_BAD_INDEX);
              srow = 0;
              bytes = 0u;
            }
            // chunk c of buffer row r lands at (c & ~7) | ((c ^ r) & 7): the 16-byte chunks of
            // each 128-byte half are XOR-swizzled by the row's slot
            const int pos = (chunk & ~7) | ((chunk ^ r) & 7);
            cp_async_16(buf + (uint32_t)(r * ROWB + pos * 16),
                        feat + (int64_t)srow * CIN + chunk * 8, bytes);
          }
        }
        cp_async_arrive_noinc(&dedup_full[ws]);
      }
      const bool meta_free = fail || mbar_wait_bounded(&meta_empty[ws], ph, s_abort);
      fail = loader_bar_any(fail || !meta_free);
      if (valid && !fail) {
#pragma unroll
        for (int j = 0; j < ORPT; ++j) {
          const int i = g + j * DLT;
          if (i < DTBM) s_orow[ws * DTBM + i] = orows[j];
        }
        if (g == 0) {
          DdSlot w;
          w.item = item;
          w.n0 = nt * BN;
          w.umask = (uint32_t)meta.y;
          w.tile = tile;
          slots[ws] = w;
        }
      } else if (g == 0) {
        DdSlot w;
        w.item = -1;
        w.n0 = 0;
        w.umask = 0;
        w.tile = 0;
        slots[ws] = w;
      }
      asm volatile("bar.sync %0, %1;" ::"n"(LOADER_BAR), "n"(DLT) : "memory");
      if (g == 0) mbar_arrive_dd(&meta_full[ws]);
      if (fail) ok = false;
      if (!valid || fail) break;
    }
    if (!ok) {
      cp_async_wait_all();
      report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else if (warp < DBLD0) {
    // ---- epilogue: warp w reads TMEM lanes 32*(w % 4) .. +31 ----
    const int q = warp & 3;
    const int er = q * 32 + lane;
    for (int local = 0; ok; ++local) {
      const int ws = local & 1;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(&meta_full[ws], (local >> 1) & 1, s_abort))) {
        ok = false;
        break;
      }
      const DdSlot w = slots[ws];
      if (w.item < 0) break;
      const int ab = local & 1;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(&acc_full[ab], (local >> 1) & 1, s_abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int32_t orow = s_orow[ws * DTBM + er];
      const uint32_t t_row = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN);
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t v[32];
        if (w.umask != 0) {
          tmem_ld_32x32b_x32(t_row + ch * 32, v);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0u;
        }
        if (orow >= 0 && orow < n) {
          const int c0 = w.n0 + ch * 32;
          uint32_t res[16];
          if constexpr (kResidual) {
            const uint4* rsrc = reinterpret_cast<const uint4*>(residual + (int64_t)orow * cout + c0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint4 r4 = rsrc[j];
              res[4 * j] = r4.x;
              res[4 * j + 1] = r4.y;
              res[4 * j + 2] = r4.z;
              res[4 * j + 3] = r4.w;
            }
          }
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float lo = __uint_as_float(v[2 * j]);
            float hi = __uint_as_float(v[2 * j + 1]);
            if (bias) {
              lo += to_f32(bias[c0 + 2 * j]);
              hi += to_f32(bias[c0 + 2 * j + 1]);
            }
            if constexpr (kResidual) {
              const T* r2 = reinterpret_cast<const T*>(&res[j]);
              lo += to_f32(r2[0]);
              hi += to_f32(r2[1]);
            }
            packed[j] = dd_pack2<T>(lo, hi);
          }
          uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)orow * cout + c0);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2],
                                packed[4 * j + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_dd(&acc_empty[ab]);
        mbar_arrive_dd(&meta_empty[ws]);
      }
    }
    if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
  } else {
    // ---- A builders: tile row r = 32 * (warp % 4) + lane, TMEM lane r; group grp ----
    // Software-pipelined: the group's next stage's row is read from the shared buffer (or, for a
    // row the buffer could not hold, from global memory) before that stage waits for its slot.
    const int q = warp & 3;
    const int grp = (warp - DBLD0) >> 2;
    const int r = q * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16) + L::A_COL0;
    int it = 0;
    for (int local = 0; ok; ++local) {
      const int ws = local & 1;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(&meta_full[ws], (local >> 1) & 1, s_abort))) {
        ok = false;
        break;
      }
      const DdSlot w = slots[ws];
      if (w.item < 0) break;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(&dedup_full[ws], (local >> 1) & 1, s_abort))) {
        ok = false;
        break;
      }
      const int16_t* ln = s_lnbr + ws * DTBM * DKVOL + r * DKVOL;
      const uint32_t buf = smem_u32(sDedup + ws * DEDUP_BYTES);
      const int32_t orow = s_orow[ws * DTBM + r];
      // the row of (offset k, block kb) into v: chunk j of a buffer row sits at j ^ (slot & 7)
      auto load_stage = [&](uint32_t (&v)[32], int k, int kb) {
        const int e = ln[k];
        if (e >= 0 && e < UMAX) {
          const uint32_t row = buf + (uint32_t)(e * ROWB + kb * 128);
          const uint32_t sw = (uint32_t)(e & 7);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 c = lds128(row + ((((uint32_t)j) ^ sw) << 4));
            v[4 * j] = c.x;
            v[4 * j + 1] = c.y;
            v[4 * j + 2] = c.z;
            v[4 * j + 3] = c.w;
          }
        } else {
          int32_t grow = -1;  // a row the buffer could not hold: read it through the map
          if (e == -2 && orow >= 0 && orow < n) {
            grow = __ldg(&nbr[(int64_t)orow * DKVOL + k]);
            if (grow >= n) grow = -1;
          }
          if (grow >= 0) {
            const uint4* src = reinterpret_cast<const uint4*>(feat + (int64_t)grow * CIN + kb * 64);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint4 c = __ldg(&src[j]);
              v[4 * j] = c.x;
              v[4 * j + 1] = c.y;
              v[4 * j + 2] = c.z;
              v[4 * j + 3] = c.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0u;
          }
        }
      };
      // Stages of the tile in order; this group builds those whose global index it0 + s is
      // congruent to its group number. Each stage: wait for its TMEM slot, store its first row
      // (read while the group's previous stage finished), read and store its second row behind
      // the first store, wait for both stores, signal the MMA; then read the group's next first
      // row.
      SubStages sub{w.umask, 0};
      uint32_t va[32], vb[32];
      int k[P], kb[P];
      auto take = [&]() {
        int c = 0;
        for (int j = 0; j < P && sub.next(KB, &k[j], &kb[j]); ++j) ++c;
        return c;
      };
      const int it0 = it;
      int s = 0;
      int cnt = take();
      while (cnt > 0 && ((it0 + s) % DGROUPS) != grp) {
        ++s;
        cnt = take();
      }
      if (cnt > 0) load_stage(va, k[0], kb[0]);
      while (cnt > 0 && ok) {
        const int gi = it0 + s;
        const int slot = gi % S;
        if (!__all_sync(0xffffffffu,
                        mbar_wait_bounded(&empty[slot], ((gi / S) & 1) ^ 1, s_abort))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t_stage = t_lane + (uint32_t)(slot * L::A_STAGE_COLS);
        tmem_st_32x32b_x32(t_stage, va);
        // the stage's other blocks, alternately into vb and va; a register array is refilled
        // only after its previous TMEM store has completed
#pragma unroll
        for (int j = 1; j < P; ++j) {
          if (j < cnt) {
            if (j >= 2) tc_wait_st();
            if (j & 1) {
              load_stage(vb, k[j], kb[j]);
              tmem_st_32x32b_x32(t_stage + 32u * j, vb);
            } else {
              load_stage(va, k[j], kb[j]);
              tmem_st_32x32b_x32(t_stage + 32u * j, va);
            }
          }
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_dd(&full[slot]);
        ++s;
        cnt = take();
        while (cnt > 0 && ((it0 + s) % DGROUPS) != grp) {
          ++s;
          cnt = take();
        }
        if (cnt > 0) load_stage(va, k[0], kb[0]);
      }
      while (cnt > 0) {  // after an expired wait: keep the stage count in step
        ++s;
        cnt = take();
      }
      it = it0 + s;
      __syncwarp();
      if (lane == 0) mbar_arrive_dd(&buf_empty[ws]);
    }
    if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

typedef CUresult (*EncodeTiledFnDd)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnDd encode_fn_dd() {
  static EncodeTiledFnDd fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnDd>(p);
  }
  return fn;
}

template <int BN, int CIN, typename T, bool kResidual>
int launch_dd(const ConvArgs& a, PlanView plan, int64_t tiles, int32_t* counter,
              cudaStream_t s) {
  using L = DdLayout<BN, dd_blocks_per_stage(CIN, BN)>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  int dev = 0;
  SV_CUDA_TRY(cudaGetDevice(&dev));
  static bool attr_done[256] = {};
  if (dev >= 256 || !attr_done[dev]) {
    SV_CUDA_TRY(cudaFuncSetAttribute(conv_dd_kernel<BN, CIN, T, kResidual>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM));
    if (dev < 256) attr_done[dev] = true;
  }
  EncodeTiledFnDd encode = encode_fn_dd();
  if (encode == nullptr) SV_FAIL(SV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  CUtensorMap tmap;
  const cuuint64_t gdim[2] = {(cuuint64_t)DKVOL * CIN, (cuuint64_t)a.cout};
  const cuuint64_t gstride[1] = {(cuuint64_t)DKVOL * CIN * 2};
  const cuuint32_t box[2] = {64u, (cuuint32_t)BN};
  const cuuint32_t estride[2] = {1, 1};
  CUresult cr = encode(&tmap,
                       kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                       2, const_cast<void*>(a.weight), gdim, gstride, box, estride,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) SV_FAIL(SV_ERR_CUDA, "cuTensorMapEncodeTiled failed for the weight");
  DdSched sc;
  sc.counter = counter;
  sc.tiles = (int32_t)tiles;
  const int64_t items = tiles * (a.cout / BN);
  if (items > INT32_MAX / 2) SV_FAIL(SV_ERR_UNSUPPORTED, "too many tensor-core work items");
  sc.total_items = (int32_t)items;
  const int grid = (int)std::min<int64_t>(items, num_sms());
  SV_CUDA_TRY(cudaMemsetAsync(counter, 0, sizeof(int32_t), s));
  conv_dd_kernel<BN, CIN, T, kResidual><<<grid, dd_threads(CIN), L::SMEM, s>>>(
      tmap, static_cast<const T*>(a.features), (int)a.n, a.nbr, plan,
      static_cast<const T*>(a.bias), static_cast<const T*>(a.residual), a.cout,
      static_cast<T*>(a.out), sc, a.status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

template <int CIN, typename T, bool kResidual>
int launch_dd_bn(const ConvArgs& a, PlanView plan, int64_t tiles, int32_t* counter,
                 cudaStream_t s) {
  if (a.cout % 128 == 0) return launch_dd<128, CIN, T, kResidual>(a, plan, tiles, counter, s);
  if (a.cout % 64 == 0) return launch_dd<64, CIN, T, kResidual>(a, plan, tiles, counter, s);
  return launch_dd<32, CIN, T, kResidual>(a, plan, tiles, counter, s);
}

template <typename T, bool kResidual>
int launch_dd_cin(const ConvArgs& a, PlanView plan, int64_t tiles, int32_t* counter,
                  cudaStream_t s) {
  if (a.cin == 64) return launch_dd_bn<64, T, kResidual>(a, plan, tiles, counter, s);
  return launch_dd_bn<128, T, kResidual>(a, plan, tiles, counter, s);
}

}  // namespace
}  // namespace sv

using namespace sv;

extern "C" int sv_conv_dd_supported(int64_t n, int cin, int cout, int kvol, int dtype) {
  return (dtype == SV_FLOAT16 || dtype == SV_BFLOAT16) && kvol == DKVOL &&
         (cin == 64 || cin == 128) && cout > 0 && cout % 32 == 0 && cout <= 1024 && n >= 0 &&
         n <= INT32_MAX - DTBM;
}

extern "C" size_t sv_conv_dd_plan_bytes(int64_t n, int cin) {
  if (n <= 0 || (cin != 64 && cin != 128)) return 0;
  return dd_plan_bytes((n + DTBM - 1) / DTBM, cin);
}

extern "C" size_t sv_conv_dd_plan_workspace_bytes(int64_t n) {
  if (n <= 0) return 0;
  return dd_align((size_t)n * 8) * 2 + dd_align((size_t)n * 4) * 2 + dd_align(dd_sort_bytes(n));
}

extern "C" int sv_conv_dd_plan(const int32_t* coords, const int32_t* nbr, int64_t n, int kvol,
                               int cin, void* plan, size_t plan_bytes, void* workspace,
                               size_t workspace_bytes, int32_t* status, sv_stream_t stream) {
  if (n < 0 || kvol != DKVOL || (cin != 64 && cin != 128))
    SV_FAIL(SV_ERR_UNSUPPORTED, "sv_conv_dd_plan: 3x3x3 kernels with 64 or 128 input channels");
  if (n == 0) return SV_OK;
  if (n > INT32_MAX - DTBM) SV_FAIL(SV_ERR_UNSUPPORTED, "sv_conv_dd_plan: too many rows");
  if (!coords || !nbr || !plan || !aligned16(coords))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv_dd_plan: null or misaligned pointer");
  if (plan_bytes < sv_conv_dd_plan_bytes(n, cin) || (reinterpret_cast<uintptr_t>(plan) & 255))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_conv_dd_plan: plan buffer too small or not 256-byte aligned");
  if (!workspace || workspace_bytes < sv_conv_dd_plan_workspace_bytes(n))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_conv_dd_plan: workspace too small");
  cudaStream_t s = to_stream(stream);
  const int64_t tiles = (n + DTBM - 1) / DTBM;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t k8 = dd_align((size_t)n * 8), r4 = dd_align((size_t)n * 4);
  uint64_t* keys = reinterpret_cast<uint64_t*>(ws);
  uint64_t* keys_sorted = reinterpret_cast<uint64_t*>(ws + k8);
  int32_t* rows = reinterpret_cast<int32_t*>(ws + 2 * k8);
  int32_t* rows_sorted = reinterpret_cast<int32_t*>(ws + 2 * k8 + r4);
  void* cub_tmp = ws + 2 * k8 + 2 * r4;
  size_t cub_bytes = workspace_bytes - (2 * k8 + 2 * r4);
  dd_morton_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const int4*>(coords), n, keys, rows);
  SV_LAUNCH_CHECK();
  SV_CUDA_TRY(cub::DeviceRadixSort::SortPairs(cub_tmp, cub_bytes, keys, keys_sorted, rows,
                                              rows_sorted, (int)n, 0, 63, s));
  int32_t* rank = rows;  // the sort's input rows are dead now
  dd_rank_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(rows_sorted, n, rank);
  SV_LAUNCH_CHECK();
  PlanView v = dd_plan_view(plan, tiles, cin);
  if (cin == 64)
    dd_plan_tile_kernel<dd_umax(64)><<<(unsigned)tiles, DTBM, 0, s>>>(nbr, n, rows_sorted, rank,
                                                                      v, status);
  else
    dd_plan_tile_kernel<dd_umax(128)><<<(unsigned)tiles, DTBM, 0, s>>>(nbr, n, rows_sorted, rank,
                                                                       v, status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

extern "C" int sv_conv3d_forward_dd(const void* features, int64_t n, int cin,
                                    const int32_t* nbr, int kvol, const void* plan,
                                    size_t plan_bytes, const void* weight, const void* bias,
                                    const void* residual, int cout, int dtype, void* out,
                                    void* workspace, size_t workspace_bytes, int32_t* status,
                                    sv_stream_t stream) {
  if (!sv_conv_dd_supported(n, cin, cout, kvol, dtype))
    SV_FAIL(SV_ERR_UNSUPPORTED, "sv_conv3d_forward_dd: fp16/bf16, 3x3x3, Cin 64 or 128, "
                                "Cout a multiple of 32");
  if (n == 0) return SV_OK;
  if (!features || !nbr || !plan || !weight || !out)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_forward_dd: null pointer");
  if (!aligned16(features) || !aligned16(weight) || !aligned16(out) || !aligned16(residual))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_forward_dd: pointers must be 16-byte aligned");
  if (plan_bytes < sv_conv_dd_plan_bytes(n, cin) || (reinterpret_cast<uintptr_t>(plan) & 255))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_conv3d_forward_dd: plan buffer too small or misaligned");
  if (!workspace || workspace_bytes < 4)
    SV_FAIL(SV_ERR_WORKSPACE, "sv_conv3d_forward_dd: needs a 4-byte scheduler word");
  ConvArgs a{};
  a.features = features;
  a.n = n;
  a.cin = cin;
  a.nbr = nbr;
  a.kvol = kvol;
  a.weight = weight;
  a.layout = SV_WEIGHT_OKI;
  a.bias = bias;
  a.cout = cout;
  a.dtype = dtype;
  a.out = out;
  a.status = status;
  a.residual = residual;
  const int64_t tiles = (n + DTBM - 1) / DTBM;
  PlanView v = dd_plan_view(const_cast<void*>(plan), tiles, cin);
  int32_t* counter = static_cast<int32_t*>(workspace);
  cudaStream_t s = to_stream(stream);
  if (dtype == SV_BFLOAT16) {
    if (residual) return launch_dd_cin<__nv_bfloat16, true>(a, v, tiles, counter, s);
    return launch_dd_cin<__nv_bfloat16, false>(a, v, tiles, counter, s);
  }
  if (residual) return launch_dd_cin<__half, true>(a, v, tiles, counter, s);
  return launch_dd_cin<__half, false>(a, v, tiles, counter, s);
}
