// fp32 sparse convolution on the 5th-generation tensor cores by 3xTF32 (tcgen05 kind::tf32).
//
// Computes the Metal kernel's result (src/mlx_diffuser/kernels/sparse.py:14-34) for fp32
// features: out[p, o] = bias[o] + sum over offsets k with nbr[p,k] >= 0 of
// features[nbr[p,k]] . W[k][:, o], accumulated in fp32. A TF32 multiply keeps 10 mantissa bits,
// too few for fp32 results within 1e-4, so every operand x is split exactly into
// hi = x with its low 13 mantissa bits cleared (a TF32 value) and lo = x - hi (exact in fp32), and
// each product is A_hi B_hi + A_hi B_lo + A_lo B_hi: the dropped A_lo B_lo and the rounding of the
// lo parts are ~2^-21 of the product. The two correction products accumulate in a TMEM
// accumulator of their own: summed into the main one, their low bits would be dropped against
// the ~2^10 times larger A_hi B_hi terms of the same MMA (the tensor core aligns a K group's
// products to the largest); the epilogue adds the two accumulators in fp32.
//
// Same scheme as the half-precision kernel (conv_tc.cu): an output-stationary implicit GEMM over
// 128-row tiles of the mask-sorted row schedule, persistent CTAs, the K loop over the offsets a
// tile visits, 32 input channels (128 bytes) per stage. Warp roles (448 threads):
//   warp 0      TMA producer: W_hi and W_lo tiles of the stage (weights split once per call);
//   warp 1      TMEM allocator and MMA issuer: per stage 4 K-steps x 3 tcgen05.mma kind::tf32
//               (A_hi B_hi into the main accumulator, A_hi B_lo and A_lo B_hi into the
//               correction accumulator);
//   warps 2-5   gatherers: load each 16-byte chunk of the 128 neighbour rows (the next stage's
//               loads in flight while this stage is stored), split it in registers and store hi
//               and lo into the two swizzled A buffers of the stage; one arrival per warp;
//   warps 6-9   epilogue: tcgen05.ld of both accumulators, sum, + bias (+ residual), fp32 stores;
//   warps 10-13 stagers: the next work item's rows and neighbour lists.
// Every wait is bounded (2 s, plus a CTA-wide abort flag); on expiry the kernel ORs
// SV_DEVICE_WAIT_TIMEOUT into the status word, all roles unwind and TMEM is freed.
#include <algorithm>

#include "conv.h"

namespace sv {
namespace {

constexpr int FBM = 128;
constexpr int FTHREADS = 448;
constexpr int FMAX_KVOL = 27;
constexpr int FSTAGER_BAR = 1;
constexpr int FBK = 32;           // fp32 input channels per stage
constexpr int FROW_BYTES = 128;   // one swizzle row of the A/B tiles

struct FSlot {
  int32_t item;
  int32_t n0;
  uint32_t umask;
  int32_t pad;
};

template <int BN>
struct TfLayout {
  static constexpr int A_BYTES = FBM * FROW_BYTES;  // 16 KB, one of hi / lo
  static constexpr int B_BYTES = BN * FROW_BYTES;
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int STAGES_FIT = (192 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
  static constexpr int A_OFF = 0;                             // [S][hi, lo]
  static constexpr int B_OFF = STAGES * 2 * A_BYTES;          // [S][hi, lo]
  static constexpr int NBR_OFF = B_OFF + STAGES * 2 * B_BYTES;
  static constexpr int OROW_OFF = NBR_OFF + 2 * FBM * FMAX_KVOL * 4;
  static constexpr int SLOT_OFF = OROW_OFF + 2 * FBM * 4;
  static constexpr int MISC_OFF = SLOT_OFF + 2 * 16;
  static constexpr int BAR_OFF = MISC_OFF + 32;
  static constexpr int NUM_BARS = 2 * STAGES + 8;
  static constexpr int BYTES = BAR_OFF + NUM_BARS * 8;
  static constexpr int SMEM = BYTES + 1024;
  static constexpr uint32_t TMEM_COLS = 4 * BN;  // 2 buffers x (main, correction)
  static_assert(STAGES >= 3, "pipeline depth");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(BAR_OFF % 8 == 0, "mbarrier alignment");
};

struct FSched {
  int32_t* counter;
  const int32_t* tile_order;
  int32_t row_tiles;
  int32_t n_rows;
  int32_t n_tiles;
  int32_t total_items;
};

// Instruction descriptor of kind::tf32: fp32 accumulator, TF32 A and B (format 2), K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_f(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool fstager_bar_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, %2, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "n"(FSTAGER_BAR)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// x = hi + lo with hi a TF32 value (low 13 mantissa bits clear) and lo exact in fp32.
__device__ __forceinline__ void split_tf32(uint32_t x, uint32_t* hi, uint32_t* lo) {
  const uint32_t h = x & 0xFFFFE000u;
  *hi = h;
  *lo = __float_as_uint(__uint_as_float(x) - __uint_as_float(h));
}

template <int BN, bool kResidual>
__global__ void __launch_bounds__(FTHREADS, 1)
    conv_tf32_kernel(const __grid_constant__ CUtensorMap tmap_hi,
                     const __grid_constant__ CUtensorMap tmap_lo, const float* __restrict__ feat,
                     int n, int cin, const int32_t* __restrict__ nbr, int kvol,
                     const int32_t* __restrict__ row_order, const float* __restrict__ bias,
                     const float* residual, int cout, float* out, FSched sc, int32_t* status) {
  using L = TfLayout<BN>;
  constexpr int S = L::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem + L::A_OFF;
  uint8_t* sB = smem + L::B_OFF;
  int32_t* s_nbr = reinterpret_cast<int32_t*>(smem + L::NBR_OFF);
  int32_t* s_orow = reinterpret_cast<int32_t*>(smem + L::OROW_OFF);
  FSlot* slots = reinterpret_cast<FSlot*>(smem + L::SLOT_OFF);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  int32_t* s_fetch = reinterpret_cast<int32_t*>(smem + L::MISC_OFF + 8);
  uint32_t* s_wmask = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF + 16);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;                 // [S]: TMA expect_tx + 4 gatherer warps
  uint64_t* empty = bars + S;            // [S]: tcgen05.commit
  uint64_t* acc_full = bars + 2 * S;     // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]: 4 epilogue warps
  uint64_t* work_full = acc_empty + 2;   // [2]: one stager
  uint64_t* work_empty = work_full + 2;  // [2]: 4 epilogue warps

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kb_per_k = cin / FBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1 + 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
      mbar_init(&work_full[b], 1);
      mbar_init(&work_empty[b], 4);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_hi);
    prefetch_tmap(&tmap_lo);
  }
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
    // ---- TMA producer: W_hi and W_lo tiles ----
    if (lane == 0) {
      int it = 0;
      for (int local = 0; ok; ++local) {
        const int ws = local & 1;
        if (!mbar_wait_bounded(&work_full[ws], (local >> 1) & 1, s_abort)) {
          ok = false;
          break;
        }
        const FSlot w = slots[ws];
        if (w.item < 0) break;
        for (uint32_t m = w.umask; m != 0 && ok; m &= m - 1) {
          const int k = __ffs(m) - 1;
          for (int kb = 0; kb < kb_per_k; ++kb, ++it) {
            const int slot = it % S;
            if (!mbar_wait_bounded(&empty[slot], ((it / S) & 1) ^ 1, s_abort)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[slot], 2 * L::B_BYTES);
            uint8_t* b = sB + slot * 2 * L::B_BYTES;
            tma_load_2d(smem_u32(b), &tmap_hi, &full[slot], k * cin + kb * FBK, w.n0);
            tma_load_2d(smem_u32(b + L::B_BYTES), &tmap_lo, &full[slot], k * cin + kb * FBK,
                        w.n0);
          }
        }
      }
      if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(FBM, BN);
      int it = 0;
      for (int local = 0; ok; ++local) {
        const int ws = local & 1;
        if (!mbar_wait_bounded(&work_full[ws], (local >> 1) & 1, s_abort)) {
          ok = false;
          break;
        }
        const FSlot w = slots[ws];
        if (w.item < 0) break;
        const int ab = local & 1;
        if (!mbar_wait_bounded(&acc_empty[ab], ((local >> 1) & 1) ^ 1, s_abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * 2 * BN);  // main; correction at d + BN
        const uint32_t dc = d + (uint32_t)BN;
        uint32_t acc = 0u;
        for (uint32_t m = w.umask; m != 0 && ok; m &= m - 1) {
          for (int kb = 0; kb < kb_per_k; ++kb, ++it) {
            const int slot = it % S;
            if (!mbar_wait_bounded(&full[slot], (it / S) & 1, s_abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_hi = smem_u32(sA + slot * 2 * L::A_BYTES);
            const uint32_t a_lo = a_hi + L::A_BYTES;
            const uint32_t b_hi = smem_u32(sB + slot * 2 * L::B_BYTES);
            const uint32_t b_lo = b_hi + L::B_BYTES;
#pragma unroll
            for (int kk = 0; kk < FBK / 8; ++kk) {  // K = 8 TF32 values (32 bytes) per MMA
              const uint32_t o = (uint32_t)(kk * 32);
              tc_mma_tf32(d, smem_desc_kmajor(a_hi + o, 2u, 128u),
                          smem_desc_kmajor(b_hi + o, 2u, 128u), idesc, acc);
              tc_mma_tf32(dc, smem_desc_kmajor(a_hi + o, 2u, 128u),
                          smem_desc_kmajor(b_lo + o, 2u, 128u), idesc, acc);
              tc_mma_tf32(dc, smem_desc_kmajor(a_lo + o, 2u, 128u),
                          smem_desc_kmajor(b_hi + o, 2u, 128u), idesc, 1u);
              acc = 1u;
            }
            tc_commit(&empty[slot]);
          }
        }
        tc_commit(&acc_full[ab]);  // also after a timeout, so the epilogue never waits on nothing
      }
      if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else if (warp < 6) {
    // ---- gatherers: 8 chunks of 16 bytes per row, chunk g % 8 of rows g / 8 + 16 i ----
    const int g = threadIdx.x - 64;
    const uint32_t chunk = (uint32_t)(g & 7);
    const int row0 = g >> 3;
    const uint32_t swz = (chunk ^ (uint32_t)(row0 & 7)) << 4;  // 128-byte swizzle (row & 7)
    constexpr int PASSES = 8;
    int it = 0;
    for (int local = 0; ok; ++local) {
      const int ws = local & 1;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(&work_full[ws], (local >> 1) & 1, s_abort))) {
        ok = false;
        break;
      }
      const FSlot w = slots[ws];
      if (w.item < 0) break;
      const int32_t* nb = s_nbr + ws * FBM * FMAX_KVOL;
      // the stages of the item: (offset, 32-channel block); loads run one stage ahead
      uint32_t m = w.umask;
      int kb_next = 0;
      auto next_stage = [&](int* k, int* kb) -> bool {
        if (m == 0) return false;
        *k = __ffs(m) - 1;
        *kb = kb_next;
        if (++kb_next == kb_per_k) {
          kb_next = 0;
          m &= m - 1;
        }
        return true;
      };
      auto load_stage = [&](uint4 (&v)[PASSES], int k, int kb) {
#pragma unroll
        for (int i = 0; i < PASSES; ++i) {
          const int32_t src = nb[(row0 + 16 * i) * FMAX_KVOL + k];
          v[i] = src >= 0 ? __ldg(reinterpret_cast<const uint4*>(
                                feat + (int64_t)src * cin + kb * FBK) + chunk)
                          : make_uint4(0u, 0u, 0u, 0u);
        }
      };
      auto store_stage = [&](const uint4 (&v)[PASSES]) -> bool {
        const int slot = it % S;
        if (!__all_sync(0xffffffffu,
                        mbar_wait_bounded(&empty[slot], ((it / S) & 1) ^ 1, s_abort)))
          return false;
        const uint32_t hi0 = smem_u32(sA + slot * 2 * L::A_BYTES) +
                             (uint32_t)row0 * FROW_BYTES + swz;
#pragma unroll
        for (int i = 0; i < PASSES; ++i) {
          uint4 h, l;
          split_tf32(v[i].x, &h.x, &l.x);
          split_tf32(v[i].y, &h.y, &l.y);
          split_tf32(v[i].z, &h.z, &l.z);
          split_tf32(v[i].w, &h.w, &l.w);
          const uint32_t a = hi0 + (uint32_t)(16 * i * FROW_BYTES);
          sts128(a, h);
          sts128(a + L::A_BYTES, l);
        }
        fence_proxy_async_smem();  // generic-proxy stores, read by the MMA (async proxy)
        __syncwarp();
        if (lane == 0) mbar_arrive_f(&full[slot]);
        ++it;
        return true;
      };
      uint4 va[PASSES], vb[PASSES];
      int k, kb;
      bool has = next_stage(&k, &kb);
      if (has) load_stage(va, k, kb);
      while (has) {
        has = next_stage(&k, &kb);
        if (has) load_stage(vb, k, kb);
        if (!store_stage(va)) {
          ok = false;
          break;
        }
        if (!has) break;
        has = next_stage(&k, &kb);
        if (has) load_stage(va, k, kb);
        if (!store_stage(vb)) {
          ok = false;
          break;
        }
      }
    }
    if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
  } else if (warp < 10) {
    // ---- epilogue: warp w reads TMEM lanes 32*(w % 4) .. +31 ----
    const int q = warp & 3;
    const int er = q * 32 + lane;
    for (int local = 0; ok; ++local) {
      const int ws = local & 1;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(&work_full[ws], (local >> 1) & 1, s_abort))) {
        ok = false;
        break;
      }
      const FSlot w = slots[ws];
      if (w.item < 0) break;
      const int ab = local & 1;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(&acc_full[ab], (local >> 1) & 1, s_abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int32_t orow = s_orow[ws * FBM + er];
      const uint32_t t_row = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * 2 * BN);
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t v[32];
        if (w.umask != 0) {
          uint32_t c[32];
          tmem_ld_32x32b_x32(t_row + ch * 32, v);
          tmem_ld_32x32b_x32(t_row + BN + ch * 32, c);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(c[j]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0u;
        }
        if (orow >= 0 && orow < n) {
          const int c0 = w.n0 + ch * 32;
          float r[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = __uint_as_float(v[j]) + (bias ? bias[c0 + j] : 0.f);
          if constexpr (kResidual) {
            const float4* res = reinterpret_cast<const float4*>(residual + (int64_t)orow * cout + c0);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 x = res[j];
              r[4 * j] += x.x;
              r[4 * j + 1] += x.y;
              r[4 * j + 2] += x.z;
              r[4 * j + 3] += x.w;
            }
          }
          float4* dst = reinterpret_cast<float4*>(out + (int64_t)orow * cout + c0);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            dst[j] = make_float4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_f(&acc_empty[ab]);
        mbar_arrive_f(&work_empty[ws]);
      }
    }
    if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
  } else {
    // ---- stagers: next work item, its rows and their neighbour lists (one row each) ----
    const int r = threadIdx.x - 320;
    for (int local = 0;; ++local) {
      const int ws = local & 1;
      if (r == 0) *s_fetch = atomicAdd(sc.counter, 1);
      if (fstager_bar_any(!ok)) {
        ok = false;
        break;
      }
      const int32_t item = *s_fetch;
      const bool valid = item < sc.total_items;
      int32_t row_tile = 0, n0 = 0;
      if (valid) {
        const int32_t nt = item / sc.row_tiles;
        const int32_t t = item - nt * sc.row_tiles;
        row_tile = sc.tile_order ? __ldg(&sc.tile_order[t]) : t;
        n0 = nt * BN;
      }
      // the row and its neighbour list load before the wait for the slot, all FMAX_KVOL loads in
      // flight together
      int32_t orow = -1;
      if (valid) {
        const int64_t gr = (int64_t)row_tile * FBM + r;
        if (gr < sc.n_rows) orow = row_order ? __ldg(&row_order[gr]) : (int32_t)gr;
      }
      const bool orow_ok = orow >= -1 && orow < n;  // -1: padding between schedule segments
      const int32_t* nrow = nbr + (int64_t)(orow >= 0 && orow_ok ? orow : 0) * kvol;
      int32_t nv[FMAX_KVOL];
#pragma unroll
      for (int k = 0; k < FMAX_KVOL; ++k)
        nv[k] = (k < kvol && orow >= 0 && orow_ok) ? __ldg(&nrow[k]) : -1;
      const bool slot_free =
          mbar_wait_bounded(&work_empty[ws], ((local >> 1) & 1) ^ 1, s_abort);
      uint32_t mask = 0;
      if (valid && slot_free) {
        bool bad = !orow_ok;
        s_orow[ws * FBM + r] = orow_ok ? orow : -1;
        int32_t* nbw = s_nbr + ws * FBM * FMAX_KVOL + r * FMAX_KVOL;
#pragma unroll
        for (int k = 0; k < FMAX_KVOL; ++k) {
          if (k < kvol) {
            int32_t v = nv[k];
            if (v >= n) {
              bad = true;
              v = -1;
            }
            nbw[k] = v;
            mask |= (uint32_t)(v >= 0) << k;
          }
        }
        if (bad) report(status, SV_DEVICE_BAD_INDEX);
      }
      mask = __reduce_or_sync(0xffffffffu, mask);
      if (lane == 0) s_wmask[warp - 10] = mask;
      const bool fail = fstager_bar_any(!slot_free);
      if (r == 0) {
        FSlot w;
        w.item = (valid && !fail) ? item : -1;
        w.n0 = n0;
        w.umask = s_wmask[0] | s_wmask[1] | s_wmask[2] | s_wmask[3];
        w.pad = 0;
        slots[ws] = w;
        mbar_arrive_f(&work_full[ws]);
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

// hi / lo halves of an fp32 weight, elementwise (the same split the gatherers apply to A)
__global__ void split_weight_kernel(const float* __restrict__ w, int64_t count,
                                    float* __restrict__ hi, float* __restrict__ lo) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    uint32_t h, l;
    split_tf32(__float_as_uint(w[i]), &h, &l);
    hi[i] = __uint_as_float(h);
    lo[i] = __uint_as_float(l);
  }
}

typedef CUresult (*EncodeTiledFnTf)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnTf encode_fn_tf() {
  static EncodeTiledFnTf fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnTf>(p);
  }
  return fn;
}

// One half of the split spconv weight as a (Cout, K*Cin) fp32 matrix; box 32 channels x BN rows.
int weight_map_tf32(const ConvArgs& a, const float* w, int box_rows, CUtensorMap* tmap) {
  EncodeTiledFnTf encode = encode_fn_tf();
  if (encode == nullptr) SV_FAIL(SV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t gdim[2] = {(cuuint64_t)a.kvol * a.cin, (cuuint64_t)a.cout};
  const cuuint64_t gstride[1] = {(cuuint64_t)a.kvol * a.cin * 4};
  const cuuint32_t box[2] = {(cuuint32_t)FBK, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1, 1};
  CUresult cr = encode(tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(w), gdim,
                       gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                       CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) SV_FAIL(SV_ERR_CUDA, "cuTensorMapEncodeTiled failed for the weight");
  return SV_OK;
}

template <int BN, bool kResidual>
int launch_tf32_bn(const ConvArgs& a, const float* w_hi, const float* w_lo,
                   const int32_t* tile_order, int32_t* counter, cudaStream_t s) {
  using L = TfLayout<BN>;
  int dev = 0;
  SV_CUDA_TRY(cudaGetDevice(&dev));
  static bool attr_done[256] = {};
  if (dev >= 256 || !attr_done[dev]) {
    SV_CUDA_TRY(cudaFuncSetAttribute(conv_tf32_kernel<BN, kResidual>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM));
    if (dev < 256) attr_done[dev] = true;
  }
  CUtensorMap t_hi, t_lo;
  int rc = weight_map_tf32(a, w_hi, BN, &t_hi);
  if (rc != SV_OK) return rc;
  rc = weight_map_tf32(a, w_lo, BN, &t_lo);
  if (rc != SV_OK) return rc;
  FSched sc;
  sc.counter = counter;
  sc.tile_order = tile_order;
  sc.row_tiles = (int32_t)((a.n_rows + FBM - 1) / FBM);
  sc.n_rows = (int32_t)a.n_rows;
  sc.n_tiles = a.cout / BN;
  const int64_t items = (int64_t)sc.row_tiles * sc.n_tiles;
  if (items > INT32_MAX / 2) SV_FAIL(SV_ERR_UNSUPPORTED, "too many tensor-core work items");
  sc.total_items = (int32_t)items;
  const int grid = (int)std::min<int64_t>(items, num_sms());
  SV_CUDA_TRY(cudaMemsetAsync(counter, 0, sizeof(int32_t), s));
  conv_tf32_kernel<BN, kResidual><<<grid, FTHREADS, L::SMEM, s>>>(
      t_hi, t_lo, static_cast<const float*>(a.features), (int)a.n, a.cin, a.nbr, a.kvol,
      a.row_order, static_cast<const float*>(a.bias), static_cast<const float*>(a.residual),
      a.cout, static_cast<float*>(a.out), sc, a.status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

template <bool kResidual>
int launch_tf32(const ConvArgs& a, const float* w_hi, const float* w_lo,
                const int32_t* tile_order, int32_t* counter, cudaStream_t s) {
  // the widest slab: A (gathered and split per item) is the expensive operand, so halving the
  // slab to fill the last wave costs more than the wave's tail (measured on config 1)
  if (a.cout % 128 == 0)
    return launch_tf32_bn<128, kResidual>(a, w_hi, w_lo, tile_order, counter, s);
  if (a.cout % 64 == 0)
    return launch_tf32_bn<64, kResidual>(a, w_hi, w_lo, tile_order, counter, s);
  return launch_tf32_bn<32, kResidual>(a, w_hi, w_lo, tile_order, counter, s);
}

}  // namespace

bool conv_tf32_supported(const ConvArgs& a) {
  return a.dtype == SV_FLOAT32 && a.layout == SV_WEIGHT_OKI && a.cin > 0 && a.cin % FBK == 0 &&
         a.cout > 0 && a.cout % 32 == 0 && a.kvol >= 1 && a.kvol <= FMAX_KVOL &&
         a.n <= INT32_MAX - FBM && (int64_t)a.kvol * a.cin < INT32_MAX &&
         aligned16(a.features) && aligned16(a.weight) && aligned16(a.out) &&
         aligned16(a.residual);
}

size_t conv_tf32_split_bytes(int kvol, int cin, int cout) {
  return 2 * align_up((size_t)kvol * cin * cout * 4, 256);
}

int conv_tf32_launch(const ConvArgs& a, const int32_t* tile_order, int32_t* counter,
                     void* split, cudaStream_t s) {
  if (a.n_rows == 0) return SV_OK;
  if (!conv_tf32_supported(a))
    SV_FAIL(SV_ERR_UNSUPPORTED, "shape not supported by the 3xTF32 tensor-core kernel");
  if (counter == nullptr || split == nullptr)
    SV_FAIL(SV_ERR_WORKSPACE, "3xTF32 conv needs a scheduler word and the split weight");
  const int64_t count = (int64_t)a.kvol * a.cin * a.cout;
  float* w_hi = static_cast<float*>(split);
  float* w_lo = reinterpret_cast<float*>(static_cast<uint8_t*>(split) +
                                         align_up((size_t)count * 4, 256));
  const unsigned blocks = (unsigned)std::min<int64_t>((count + 255) / 256, 4 * num_sms());
  split_weight_kernel<<<blocks, 256, 0, s>>>(static_cast<const float*>(a.weight), count, w_hi,
                                             w_lo);
  SV_LAUNCH_CHECK();
  if (a.residual) return launch_tf32<true>(a, w_hi, w_lo, tile_order, counter, s);
  return launch_tf32<false>(a, w_hi, w_lo, tile_order, counter, s);
}

}  // namespace sv
