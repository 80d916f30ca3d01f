// Output-stationary sparse convolution on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Computes the Metal kernel's result (src/mlx_diffuser/kernels/sparse.py:14-34) for fp16/bf16
// features: out[p, o] = bias[o] + sum over offsets k with nbr[p,k] >= 0 of
// features[nbr[p,k]] . W[k][:, o], accumulated in fp32 (TMEM) and rounded once.
//
// Shape of the computation: an implicit GEMM whose M dimension is output rows, N is Cout and
// K is (offset, input channel). A work item is 128 output rows (a tile of `row_order`, which
// groups rows with equal neighbour masks) x BN output channels. Its K loop visits only the
// offsets for which at least one of its 128 rows has a neighbour -- the union of the rows'
// masks -- and within an offset walks Cin in BK-channel stages (BK = 64 with the 128-byte
// swizzle, or 32 with the 64-byte swizzle when Cin is an odd multiple of 32). Inputs of 8 or 16
// channels pack PACK = 32 / Cin consecutive offsets into one 32-channel stage: their weight
// columns are adjacent in the spconv (Cout, K*Cin) matrix, so B stays one TMA box (past the last
// offset it reads TMA's zero fill), and each 16-byte A chunk gathers a different offset's
// neighbour. Outputs of 8 or 16 channels run as N = 16 tiles (the smallest MMA N at M = 128)
// whose weight rows past Cout are TMA zero fill; the epilogue stores Cout columns.
//
// Persistent CTAs (one per SM) take work items from an atomic counter. Items run one
// BN-wide slab of output channels at a time (so one slab of weights is live in L2), and within
// a slab in the order `tile_order` gives the row tiles (most offsets first), so the shortest
// items come last. Warp roles (448 threads):
//   warp 0      TMA producer: W[k][kb*BK : +BK, n0 : n0+BN] from the spconv (Cout, K*Cin)
//               matrix, K-major, swizzled, one tiled 2-D load per stage;
//   warp 1      TMEM allocator (two BN-column accumulators) and the single thread that issues
//               tcgen05.mma (M=128, N=BN, K=16, BK/16 per stage) and tcgen05.commit;
//   warps 2-5   gatherers: copy each A stage (128 neighbour rows x 2*BK bytes) with 16-byte
//               cp.async -- whole rows per group of threads, so a warp instruction reads
//               complete rows -- zero-filled for missing neighbours, in the swizzled layout TMA
//               would write;
//   warps 6-9   epilogue: tcgen05.ld of 32 accumulator columns at a time, + bias (+ the
//               residual row, when given), round, 16-byte stores to the row's output; it drains
//               one accumulator while the MMA fills the other;
//   warps 10-13 stagers: fetch the next work item and stage its rows and their neighbour
//               lists (one row per thread, double-buffered) while the current item runs.
// Barriers: a stage ring (full/empty; 4 to 8 deep depending on BN), two accumulator buffers
// (full/empty) and two work-item slots (full/empty). Every wait is bounded: on expiry the
// kernel ORs SV_DEVICE_WAIT_TIMEOUT into the status word, all roles unwind, copies drain and
// TMEM is freed.
#include <algorithm>
#include <type_traits>

#include "conv.h"

namespace sv {
namespace {

constexpr int TBM = 128;       // output rows per tile == TMEM lanes
constexpr int TTHREADS = 448;
constexpr int TMAX_KVOL = 27;
constexpr int STAGER_BAR = 1;  // named barrier of the four stager warps

struct WorkSlot {
  int32_t item;    // < 0: no more work
  int32_t n0;      // first output channel
  uint32_t umask;  // offsets visited
  int32_t pad;
};

template <int BN, int BK>
struct TcLayout {
  static constexpr int ROW_BYTES = BK * 2;                 // one swizzle row of the A/B tiles
  static constexpr uint32_t SWIZZLE = BK == 64 ? 2u : 4u;  // descriptor layout: 128 B / 64 B
  static constexpr int A_STAGE_BYTES = TBM * ROW_BYTES;
  static constexpr int B_STAGE_BYTES = BN * ROW_BYTES;
  static constexpr int STAGE_BUDGET = 192 * 1024;
  static constexpr int STAGES_FIT = STAGE_BUDGET / (A_STAGE_BYTES + B_STAGE_BYTES);
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = STAGES * A_STAGE_BYTES;
  static constexpr int NBR_OFF = B_OFF + STAGES * B_STAGE_BYTES;
  static constexpr int OROW_OFF = NBR_OFF + 2 * TBM * TMAX_KVOL * 4;  // nbr [2][128][27]
  static constexpr int SLOT_OFF = OROW_OFF + 2 * TBM * 4;             // orow [2][128]
  static constexpr int MISC_OFF = SLOT_OFF + 2 * 16;  // tmem, abort, fetch, pad, wmask[4]
  static constexpr int BAR_OFF = MISC_OFF + 32;
  static constexpr int NUM_BARS = 2 * STAGES + 8;
  static constexpr int BYTES = BAR_OFF + NUM_BARS * 8;
  static constexpr int SMEM = BYTES + 1024;  // slack for aligning the base to 1024 bytes
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(STAGES >= 4, "pipeline depth");
  static_assert(BAR_OFF % 8 == 0, "mbarriers need 8-byte alignment");
  static_assert(A_STAGE_BYTES % 1024 == 0 && B_STAGE_BYTES % 1024 == 0, "swizzle atoms");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512, "TMEM columns");
};

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Barrier of the 128 stager threads that also ORs a predicate across them, so that all stagers
// take the same exit decision (one that left alone would leave the others at the barrier).
__device__ __forceinline__ bool stager_bar_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, %2, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "n"(STAGER_BAR)
      : "memory");
  return r != 0;
}

struct Sched {
  int32_t* counter;           // zeroed before the launch
  const int32_t* tile_order;  // row tiles, most expensive first (nullable: identity)
  int32_t row_tiles;
  int32_t n_rows;             // rows of the schedule (row_order[0 .. n_rows)); -1 = padding
  int32_t n_tiles;            // Cout / BN
  int32_t total_items;        // row_tiles * n_tiles; order: n-slab major, then tile_order
  int32_t wait_from;          // tile-order position of the first tile that reads halo rows
  int32_t wait_count;         // flags to wait for before staging such a tile
  int64_t wait_epoch;
  int64_t* wait_flags[8];
};

// The halo rows other GPUs push into this GPU's buffer are complete once each of their flags
// has reached the epoch (system-scope acquire, pairs with the pushers' release). Bounded by 1 s:
// the other roles' waits for the next work item are bounded by 2 s, so this wait always gives up
// first and the launch completes without tripping the abort path.
__device__ __forceinline__ bool wait_halo_flags(const Sched& sc, volatile int* abort) {
  const uint64_t t0 = global_timer_ns();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i >= sc.wait_count) break;
    for (;;) {
      int64_t v;
      asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(sc.wait_flags[i])
                   : "memory");
      if (v >= sc.wait_epoch) break;
      if (*abort || global_timer_ns() - t0 > 1000000000ull) return false;
      __nanosleep(100);
    }
  }
  return true;
}

template <int BN>
__device__ __forceinline__ void decode_item(const Sched& sc, int32_t item, int32_t* row_tile,
                                            int32_t* n0) {
  const int32_t nt = item / sc.row_tiles;
  const int32_t t = item - nt * sc.row_tiles;
  *row_tile = sc.tile_order ? __ldg(&sc.tile_order[t]) : t;
  *n0 = nt * BN;
}

template <int BN, int BK, typename T, bool kResidual, int PACK>
__global__ void __launch_bounds__(TTHREADS, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const T* __restrict__ feat,
                   int n, int cin, const int32_t* __restrict__ nbr, int kvol,
                   const int32_t* __restrict__ row_order, const T* __restrict__ bias,
                   const T* residual, int cout, T* out, Sched sc, int32_t* status) {
  using L = TcLayout<BN, BK>;
  constexpr int S = L::STAGES;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem + L::A_OFF;
  uint8_t* sB = smem + L::B_OFF;
  int32_t* s_nbr = reinterpret_cast<int32_t*>(smem + L::NBR_OFF);
  int32_t* s_orow = reinterpret_cast<int32_t*>(smem + L::OROW_OFF);
  WorkSlot* slots = reinterpret_cast<WorkSlot*>(smem + L::SLOT_OFF);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  int32_t* s_fetch = reinterpret_cast<int32_t*>(smem + L::MISC_OFF + 8);
  uint32_t* s_wmask = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF + 16);  // [4]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;                // [S]
  uint64_t* empty = bars + S;           // [S]
  uint64_t* acc_full = bars + 2 * S;    // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* work_full = acc_empty + 2;  // [2]
  uint64_t* work_empty = work_full + 2; // [2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // stages per mask bit: Cin / BK blocks of one offset, or (PACK > 1) one stage per bit, a bit
  // standing for a group of PACK offsets
  const int kb_per_k = PACK > 1 ? 1 : cin / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1 + TBM);  // TMA expect_tx arrival + 128 cp.async arrivals
      mbar_init(&empty[s], 1);       // tcgen05.commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);      // tcgen05.commit
      mbar_init(&acc_empty[b], TBM);   // every epilogue thread
      mbar_init(&work_full[b], 1);     // one stager, once the item is staged
      mbar_init(&work_empty[b], TBM);  // every epilogue thread, once the item is stored
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
        if (!mbar_wait_bounded(&work_full[ws], (local >> 1) & 1, s_abort)) {
          ok = false;
          break;
        }
        const WorkSlot w = slots[ws];
        if (w.item < 0) break;
        for (uint32_t m = w.umask; m != 0 && ok; m &= m - 1) {
          const int k = __ffs(m) - 1;
          for (int kb = 0; kb < kb_per_k; ++kb, ++it) {
            const int slot = it % S;
            if (!mbar_wait_bounded(&empty[slot], ((it / S) & 1) ^ 1, s_abort)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[slot], L::B_STAGE_BYTES);
            tma_load_2d(smem_u32(sB + slot * L::B_STAGE_BYTES), &tmap_w, &full[slot],
                        PACK > 1 ? k * BK : k * cin + kb * BK, w.n0);
          }
        }
      }
      if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kBF16, TBM, BN);
      int it = 0;
      for (int local = 0; ok; ++local) {
        const int ws = local & 1;
        if (!mbar_wait_bounded(&work_full[ws], (local >> 1) & 1, s_abort)) {
          ok = false;
          break;
        }
        const WorkSlot w = slots[ws];
        if (w.item < 0) break;
        const int ab = local & 1;  // accumulator buffer
        if (!mbar_wait_bounded(&acc_empty[ab], ((local >> 1) & 1) ^ 1, s_abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * BN);
        int first = 1;
        for (uint32_t m = w.umask; m != 0 && ok; m &= m - 1) {
          for (int kb = 0; kb < kb_per_k; ++kb, ++it) {
            const int slot = it % S;
            if (!mbar_wait_bounded(&full[slot], (it / S) & 1, s_abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            fence_proxy_async_smem();  // cp.async wrote A through the generic proxy
            const uint32_t a0 = smem_u32(sA + slot * L::A_STAGE_BYTES);
            const uint32_t b0 = smem_u32(sB + slot * L::B_STAGE_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              tc_mma_f16(d, smem_desc_kmajor(a0 + kk * 32, L::SWIZZLE, L::ROW_BYTES),
                         smem_desc_kmajor(b0 + kk * 32, L::SWIZZLE, L::ROW_BYTES), idesc,
                         (first && kk == 0) ? 0u : 1u);
            first = 0;
            tc_commit(&empty[slot]);
          }
        }
        tc_commit(&acc_full[ab]);  // also after a timeout, so the epilogue never waits on nothing
      }
      if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else if (warp < 6) {
    // ---- gatherers ----
    // CPR 16-byte chunks per row; gatherer g copies chunk g % CPR of tile rows
    // g / CPR + RPP * i (RPP = 128 / CPR rows per pass, TBM / RPP passes): a warp instruction
    // moves 32 / CPR whole rows, so every L2 sector it touches is used in full.
    constexpr int CPR = L::ROW_BYTES / 16;
    constexpr int RPP = 128 / CPR;
    constexpr int PASSES = TBM / RPP;
    const int g = threadIdx.x - 64;
    const uint32_t chunk = g % CPR;
    const int row0 = g / CPR;
    // the swizzle XORs the chunk index with address bits above the row: (row & 7) for 128-byte
    // rows, (row >> 1) & 3 for 64-byte rows; both are the same for all rows row0 + RPP * i
    const uint32_t swz = BK == 64 ? ((chunk ^ (uint32_t)(row0 & 7)) << 4)
                                  : ((chunk ^ (uint32_t)((row0 >> 1) & 3)) << 4);
    int it = 0;
    for (int local = 0; ok; ++local) {
      const int ws = local & 1;
      if (!mbar_wait_bounded(&work_full[ws], (local >> 1) & 1, s_abort)) {
        ok = false;
        break;
      }
      const WorkSlot w = slots[ws];
      if (w.item < 0) break;
      const int32_t* nb = s_nbr + ws * TBM * TMAX_KVOL;
      for (uint32_t m = w.umask; m != 0 && ok; m &= m - 1) {
        const int k = __ffs(m) - 1;
        const T* src[PASSES];
        uint32_t nbytes[PASSES];
        // packed stages: chunk c belongs to offset PACK * k + c / CPC of the group k, and is
        // part c % CPC of that neighbour's CPC-chunk row; otherwise chunk c of offset k's row
        constexpr int CPC = PACK > 1 ? CPR / PACK : CPR;
        const int kc = PACK > 1 ? PACK * k + (int)chunk / CPC : k;
        const uint32_t part = PACK > 1 ? chunk % CPC : chunk;
#pragma unroll
        for (int i = 0; i < PASSES; ++i) {
          const int32_t s_row = kc < kvol ? nb[(row0 + RPP * i) * TMAX_KVOL + kc] : -1;
          src[i] = feat + (s_row >= 0 ? (int64_t)s_row * cin : 0) + part * 8;
          nbytes[i] = s_row >= 0 ? 16u : 0u;
        }
        for (int kb = 0; kb < kb_per_k; ++kb, ++it) {
          const int slot = it % S;
          if (!mbar_wait_bounded(&empty[slot], ((it / S) & 1) ^ 1, s_abort)) {
            ok = false;
            break;
          }
          const uint32_t dst = smem_u32(sA + slot * L::A_STAGE_BYTES) +
                               (uint32_t)row0 * (uint32_t)L::ROW_BYTES + swz;
#pragma unroll
          for (int i = 0; i < PASSES; ++i)
            cp_async_16(dst + (uint32_t)(RPP * i * L::ROW_BYTES), src[i] + kb * BK, nbytes[i]);
          cp_async_arrive_noinc(&full[slot]);
        }
      }
    }
    if (!ok) {
      cp_async_wait_all();
      report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else if (warp < 10) {
    // ---- epilogue: warp w may read TMEM lanes 32*(w % 4) .. +31 ----
    const int q = warp & 3;
    const int er = q * 32 + lane;
    for (int local = 0; ok; ++local) {
      const int ws = local & 1;
      // warp-uniform decisions: tcgen05.ld below needs all 32 lanes
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&work_full[ws], (local >> 1) & 1, s_abort))) {
        ok = false;
        break;
      }
      const WorkSlot w = slots[ws];
      if (w.item < 0) break;
      const int ab = local & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&acc_full[ab], (local >> 1) & 1, s_abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int32_t orow = s_orow[ws * TBM + er];
      const uint32_t t_row = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN);
      if constexpr (BN < 32) {
        // an N = 16 tile: Cout (8 or 16) columns stored, as 16-byte vectors
        uint32_t v[16];
        if (w.umask != 0) {
          tmem_ld_32x32b_x16(t_row, v);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0u;
        }
        const int nc = min(BN, cout - w.n0);
        if (orow >= 0 && nc > 0) {
          uint32_t packed[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float lo = __uint_as_float(v[2 * j]);
            float hi = __uint_as_float(v[2 * j + 1]);
            if (2 * j < nc) {
              if (bias) {
                lo += to_f32(bias[w.n0 + 2 * j]);
                hi += to_f32(bias[w.n0 + 2 * j + 1]);
              }
              if constexpr (kResidual) {
                const T* rrow = residual + (int64_t)orow * cout + w.n0;
                lo += to_f32(rrow[2 * j]);
                hi += to_f32(rrow[2 * j + 1]);
              }
            }
            packed[j] = pack2<T>(lo, hi);
          }
          uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)orow * cout + w.n0);
          dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          if (nc > 8) dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
      }
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
        if (orow >= 0) {
          const int c0 = w.n0 + ch * 32;
          uint32_t res[16];
          if constexpr (kResidual) {
            const uint4* src = reinterpret_cast<const uint4*>(residual + (int64_t)orow * cout + c0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint4 r4 = src[j];
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
            packed[j] = pack2<T>(lo, hi);
          }
          uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)orow * cout + c0);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2],
                                packed[4 * j + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);
      mbar_arrive(&work_empty[ws]);
    }
    if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
  } else {
    // ---- stagers: next work item, its rows and their neighbour lists (one row each) ----
    const int r = threadIdx.x - 320;
    bool halo_ready = sc.wait_count == 0;
    for (int local = 0;; ++local) {
      const int ws = local & 1;
      if (r == 0) {
        const int32_t fetched = atomicAdd(sc.counter, 1);
        *s_fetch = fetched;
        // the first item whose rows read halo rows waits for the peers' pushes; an expired
        // wait is reported (the output is invalid) and the launch completes normally -- it does
        // not abort, so no copy is ever left in flight
        if (!halo_ready && fetched < sc.total_items &&
            fetched % sc.row_tiles >= sc.wait_from) {
          if (!wait_halo_flags(sc, s_abort)) report(status, SV_DEVICE_WAIT_TIMEOUT);
          halo_ready = true;
        }
      }
      // the fetched item is visible, every stager is done with the previous one, and a stager
      // whose wait expired makes all of them leave together
      if (stager_bar_any(!ok)) {
        ok = false;
        break;
      }
      const int32_t item = *s_fetch;
      const bool valid = item < sc.total_items;
      int32_t row_tile = 0, n0 = 0;
      if (valid) decode_item<BN>(sc, item, &row_tile, &n0);
      // the row and its neighbour list load before the wait for the slot, all TMAX_KVOL loads in
      // flight together: checking each value before the next load would put a memory latency
      // per offset on the path to the next item
      int32_t orow = -1;
      if (valid) {
        const int64_t gr = (int64_t)row_tile * TBM + r;
        if (gr < sc.n_rows) orow = row_order ? __ldg(&row_order[gr]) : (int32_t)gr;
      }
      const bool orow_ok = orow >= -1 && orow < n;  // -1: padding between schedule segments
      const int32_t* nrow = nbr + (int64_t)(orow >= 0 && orow_ok ? orow : 0) * kvol;
      int32_t nv[TMAX_KVOL];
#pragma unroll
      for (int k = 0; k < TMAX_KVOL; ++k)
        nv[k] = (k < kvol && orow >= 0 && orow_ok) ? __ldg(&nrow[k]) : -1;
      // slot ws (rows, neighbour lists and accumulator) is free once the epilogue has stored
      // the item two back, which also means the gatherers are done with it
      const bool slot_free =
          mbar_wait_bounded(&work_empty[ws], ((local >> 1) & 1) ^ 1, s_abort);
      uint32_t mask = 0;
      if (valid && slot_free) {
        bool bad = !orow_ok;
        s_orow[ws * TBM + r] = orow_ok ? orow : -1;
        int32_t* nb = s_nbr + ws * TBM * TMAX_KVOL + r * TMAX_KVOL;
#pragma unroll
        for (int k = 0; k < TMAX_KVOL; ++k) {
          if (k < kvol) {
            int32_t v = nv[k];
            if (v >= n) {
              bad = true;
              v = -1;
            }
            nb[k] = v;
            mask |= (uint32_t)(v >= 0) << k;
          }
        }
        if (bad) report(status, SV_DEVICE_BAD_INDEX);
      }
      mask = __reduce_or_sync(0xffffffffu, mask);
      if (lane == 0) s_wmask[warp - 10] = mask;
      // every row is staged; a slot wait that expired anywhere stops all stagers
      const bool fail = stager_bar_any(!slot_free);
      if (r == 0) {
        WorkSlot w;
        w.item = (valid && !fail) ? item : -1;
        w.n0 = n0;
        uint32_t um = s_wmask[0] | s_wmask[1] | s_wmask[2] | s_wmask[3];
        if (PACK > 1) {  // bit g: some row has a neighbour among offsets PACK*g .. PACK*g+PACK-1
          uint32_t gm = 0;
          for (int g = 0; g * PACK < TMAX_KVOL; ++g)
            gm |= (uint32_t)(((um >> (g * PACK)) & ((1u << PACK) - 1u)) != 0) << g;
          um = gm;
        }
        w.umask = um;
        w.pad = 0;
        slots[ws] = w;
        mbar_arrive(&work_full[ws]);
      }
      if (fail) ok = false;
      if (!valid || fail) break;
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

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// The spconv weight as one (Cout, K*Cin) matrix; box of BK input channels x BN output rows.
int weight_map(const ConvArgs& a, bool bf16, int box_k, int box_rows, CUtensorMap* tmap) {
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr) SV_FAIL(SV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t gdim[2] = {(cuuint64_t)a.kvol * a.cin, (cuuint64_t)a.cout};
  const cuuint64_t gstride[1] = {(cuuint64_t)a.kvol * a.cin * 2};
  const cuuint32_t box[2] = {(cuuint32_t)box_k, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1, 1};
  CUresult cr = encode(tmap,
                       bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                       2, const_cast<void*>(a.weight), gdim, gstride, box, estride,
                       CU_TENSOR_MAP_INTERLEAVE_NONE,
                       box_k == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) SV_FAIL(SV_ERR_CUDA, "cuTensorMapEncodeTiled failed for the weight");
  return SV_OK;
}

template <int BN, int BK, typename T, bool kResidual, int PACK>
int launch_bn(const ConvArgs& a, const int32_t* tile_order, int32_t* counter, cudaStream_t s) {
  using L = TcLayout<BN, BK>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  int dev = 0;
  SV_CUDA_TRY(cudaGetDevice(&dev));
  static bool attr_done[256] = {};
  if (dev >= 256 || !attr_done[dev]) {
    SV_CUDA_TRY(cudaFuncSetAttribute(conv_tc_kernel<BN, BK, T, kResidual, PACK>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM));
    if (dev < 256) attr_done[dev] = true;
  }
  CUtensorMap tmap;
  const int rc = weight_map(a, kBF16, BK, BN, &tmap);
  if (rc != SV_OK) return rc;

  Sched sc;
  sc.counter = counter;
  sc.tile_order = tile_order;
  sc.row_tiles = (int32_t)((a.n_rows + TBM - 1) / TBM);
  sc.n_rows = (int32_t)a.n_rows;
  sc.wait_from = a.wait_count > 0 ? a.wait_from : INT32_MAX;
  sc.wait_count = a.wait_count;
  sc.wait_epoch = a.wait_epoch;
  for (int i = 0; i < 8; ++i) sc.wait_flags[i] = i < a.wait_count ? a.wait_flags[i] : nullptr;
  sc.n_tiles = (a.cout + BN - 1) / BN;  // an N = 16 tile covers Cout = 8 too
  const int64_t items = (int64_t)sc.row_tiles * sc.n_tiles;
  if (items > INT32_MAX / 2) SV_FAIL(SV_ERR_UNSUPPORTED, "too many tensor-core work items");
  const int grid = (int)std::min<int64_t>(items, num_sms());
  sc.total_items = (int32_t)items;
  SV_CUDA_TRY(cudaMemsetAsync(counter, 0, sizeof(int32_t), s));
  conv_tc_kernel<BN, BK, T, kResidual, PACK><<<grid, TTHREADS, L::SMEM, s>>>(
      tmap, static_cast<const T*>(a.features), (int)a.n, a.cin, a.nbr, a.kvol,
      a.row_order, static_cast<const T*>(a.bias), static_cast<const T*>(a.residual), a.cout,
      static_cast<T*>(a.out), sc, a.status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

template <int BK, typename T, bool kResidual, int PACK>
int launch_bk(const ConvArgs& a, const int32_t* tile_order, int32_t* counter, cudaStream_t s) {
  if (a.cout < 32) return launch_bn<16, BK, T, kResidual, PACK>(a, tile_order, counter, s);
  if (a.cout % 256 == 0) return launch_bn<256, BK, T, kResidual, PACK>(a, tile_order, counter, s);
  if (a.cout % 128 == 0) return launch_bn<128, BK, T, kResidual, PACK>(a, tile_order, counter, s);
  if (a.cout % 64 == 0) return launch_bn<64, BK, T, kResidual, PACK>(a, tile_order, counter, s);
  return launch_bn<32, BK, T, kResidual, PACK>(a, tile_order, counter, s);
}

template <typename T, bool kResidual>
int launch_res(const ConvArgs& a, const int32_t* tile_order, int32_t* counter,
               cudaStream_t s) {
  if (a.cin == 8) return launch_bk<32, T, kResidual, 4>(a, tile_order, counter, s);
  if (a.cin == 16) return launch_bk<32, T, kResidual, 2>(a, tile_order, counter, s);
  if (a.cin % 64 == 0) return launch_bk<64, T, kResidual, 1>(a, tile_order, counter, s);
  return launch_bk<32, T, kResidual, 1>(a, tile_order, counter, s);
}

template <typename T>
int launch_typed(const ConvArgs& a, const int32_t* tile_order, int32_t* counter,
                 cudaStream_t s) {
  if (a.residual) return launch_res<T, true>(a, tile_order, counter, s);
  return launch_res<T, false>(a, tile_order, counter, s);
}

}  // namespace

bool conv_tc_supported(const ConvArgs& a) {
  return (a.dtype == SV_FLOAT16 || a.dtype == SV_BFLOAT16) && a.layout == SV_WEIGHT_OKI &&
         a.cin > 0 && (a.cin % 32 == 0 || a.cin == 8 || a.cin == 16) && a.cout > 0 &&
         (a.cout % 32 == 0 || a.cout == 8 || a.cout == 16) && a.kvol >= 1 &&
         a.kvol <= TMAX_KVOL && a.n <= INT32_MAX - TBM && (int64_t)a.kvol * a.cin < INT32_MAX &&
         aligned16(a.features) && aligned16(a.weight) && aligned16(a.out) &&
         aligned16(a.residual);
}

int conv_tc_launch(const ConvArgs& a, const int32_t* tile_order, int32_t* counter,
                   cudaStream_t s) {
  if (a.n_rows == 0) return SV_OK;
  if (!conv_tc_supported(a))
    SV_FAIL(SV_ERR_UNSUPPORTED, "shape not supported by the tcgen05 kernel");
  if (counter == nullptr) SV_FAIL(SV_ERR_WORKSPACE, "tcgen05 conv needs a scheduler word");
  if (a.wait_count < 0 || a.wait_count > 8 || (a.wait_count > 0 && a.wait_flags == nullptr))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "tcgen05 conv: at most 8 halo flags");
  if (a.dtype == SV_BFLOAT16) return launch_typed<__nv_bfloat16>(a, tile_order, counter, s);
  return launch_typed<__half>(a, tile_order, counter, s);
}

}  // namespace sv
