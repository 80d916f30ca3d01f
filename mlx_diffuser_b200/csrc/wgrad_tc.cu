// Weight gradient of the submanifold convolution on the 5th-generation tensor cores.
//
//     dW[o][k][i] = sum over the pairs (src, dst) of offset k of dOut[dst][o] * features[src][i]
//
// (the gradient MLX takes through src/mlx_diffuser/kernels/sparse.py:39-55, written straight
// into spconv's (Cout, K, Cin) layout). For each offset it is a GEMM whose reduction runs over
// the offset's pairs: M = 128 output channels, N = BN input channels, K = pairs in chunks of 64.
// Both operands arrive as rows indexed by the pair lists -- dOut[dst] rows hold M contiguous,
// features[src] rows hold N contiguous -- so both are MN-major. The gather warps copy each
// 128-byte row segment into one K-row of a 128-byte-swizzled MN-major atom (8 K-rows x 64
// elements): A stage = 2 x 8 atoms (16 KB), B stage = BN/64 x 8 atoms. Atoms are laid out
// MN-block-major, K-group-minor: lbo = 8 KB, sbo = 1 KB.
//
// A work item is (offset, 128 output channels, BN input channels); items of one offset are
// adjacent, so the CTAs working on an offset read the same gathered rows out of L2. Persistent
// CTAs take items from an atomic counter. Warp roles (320 threads):
//   warp 0      scheduler: fetches items and publishes them in two slots;
//   warp 1      TMEM allocator (two BN-column accumulators) and the tcgen05.mma issuer;
//   warps 2-5   gatherers: cp.async of the A and B rows of each 64-pair chunk, zero-filled past
//               the end of the offset's list, index loads one chunk ahead;
//   warps 6-9   epilogue: tcgen05.ld, round, 16-byte stores of dW rows.
// Every wait is bounded (2 s, CTA abort flag); on expiry SV_DEVICE_WAIT_TIMEOUT is reported.
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace sv {
namespace {

constexpr int WM = 128;       // output channels per item == TMEM lanes
constexpr int WKC = 64;       // pairs per stage
constexpr int WTHREADS = 320;
constexpr uint32_t ATOM = 1024;     // one 8 x 128-byte swizzle atom
constexpr uint32_t MN_STRIDE = 8 * ATOM;  // next 64-element block along M / N (8 K-groups)

struct WSlot {
  int32_t k;      // < 0: no more work
  int32_t o0;
  int32_t i0;
  int32_t begin;  // first pair of the offset
  int32_t end;
  int32_t pad[3];
};

template <int BN>
struct WLayout {
  static constexpr int A_STAGE = WM * WKC * 2;   // 16 KB
  static constexpr int B_STAGE = BN * WKC * 2;
  static constexpr int STAGES_FIT = (192 * 1024) / (A_STAGE + B_STAGE);
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = STAGES * A_STAGE;
  static constexpr int SLOT_OFF = B_OFF + STAGES * B_STAGE;
  static constexpr int MISC_OFF = SLOT_OFF + 2 * (int)sizeof(WSlot);
  static constexpr int BAR_OFF = MISC_OFF + 16;
  static constexpr int NUM_BARS = 2 * STAGES + 8;
  static constexpr int BYTES = BAR_OFF + NUM_BARS * 8;
  static constexpr int SMEM = BYTES + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(STAGES >= 4, "pipeline depth");
  static_assert(A_STAGE % 1024 == 0 && B_STAGE % 1024 == 0, "swizzle atoms");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ void mbar_arrive_w(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack2w(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

struct WSched {
  int32_t* counter;
  int32_t o_tiles;
  int32_t i_tiles;
  int32_t total_items;
};

template <int BN, typename T>
__global__ void __launch_bounds__(WTHREADS, 1)
    wgrad_tc_kernel(const T* __restrict__ feat, const T* __restrict__ dout, int cin, int cout,
                    int kvol, const int32_t* __restrict__ offsets,
                    const int32_t* __restrict__ pair_src, const int32_t* __restrict__ pair_dst,
                    T* __restrict__ dweight, WSched sc, int32_t* status) {
  using L = WLayout<BN>;
  constexpr int S = L::STAGES;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem + L::A_OFF;
  uint8_t* sB = smem + L::B_OFF;
  WSlot* slots = reinterpret_cast<WSlot*>(smem + L::SLOT_OFF);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* acc_full = bars + 2 * S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* work_full = acc_empty + 2;
  uint64_t* work_empty = work_full + 2;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 128);  // one cp.async arrival per gatherer thread
      mbar_init(&empty[s], 1);   // tcgen05.commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
      mbar_init(&work_full[b], 1);
      mbar_init(&work_empty[b], 128);
    }
    *s_abort = 0;
    fence_mbar_init();
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
    // ---- scheduler ----
    if (lane == 0) {
      const int per_k = sc.o_tiles * sc.i_tiles;
      for (int local = 0;; ++local) {
        const int ws = local & 1;
        if (!mbar_wait_bounded(&work_empty[ws], ((local >> 1) & 1) ^ 1, s_abort)) {
          ok = false;
          WSlot w{};
          w.k = -1;
          slots[ws] = w;
          mbar_arrive_w(&work_full[ws]);
          break;
        }
        const int32_t item = atomicAdd(sc.counter, 1);
        WSlot w{};
        if (item < sc.total_items) {
          w.k = item / per_k;
          const int r = item - w.k * per_k;
          w.o0 = (r / sc.i_tiles) * WM;
          w.i0 = (r % sc.i_tiles) * BN;
          w.begin = __ldg(&offsets[w.k]);
          w.end = __ldg(&offsets[w.k + 1]);
          if (w.end < w.begin) {
            report(status, SV_DEVICE_BAD_INDEX);
            w.end = w.begin;
          }
        } else {
          w.k = -1;
        }
        slots[ws] = w;
        mbar_arrive_w(&work_full[ws]);
        if (w.k < 0) break;
      }
      if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_major(kBF16, WM, BN, true, true);
      int it = 0;
      for (int local = 0; ok; ++local) {
        const int ws = local & 1;
        if (!mbar_wait_bounded(&work_full[ws], (local >> 1) & 1, s_abort)) {
          ok = false;
          break;
        }
        const WSlot w = slots[ws];
        if (w.k < 0) break;
        const int ab = local & 1;
        if (!mbar_wait_bounded(&acc_empty[ab], ((local >> 1) & 1) ^ 1, s_abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * BN);
        const int chunks = (w.end - w.begin + WKC - 1) / WKC;
        for (int c = 0; c < chunks && ok; ++c, ++it) {
          const int slot = it % S;
          if (!mbar_wait_bounded(&full[slot], (it / S) & 1, s_abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          fence_proxy_async_smem();  // cp.async wrote the operands through the generic proxy
          const uint32_t a0 = smem_u32(sA + slot * L::A_STAGE);
          const uint32_t b0 = smem_u32(sB + slot * L::B_STAGE);
#pragma unroll
          for (int kk = 0; kk < WKC / 16; ++kk)  // 16 pairs = two 8-row K groups
            tc_mma_f16(d, smem_desc_mn_sw128(a0 + kk * 2 * ATOM, MN_STRIDE, ATOM),
                       smem_desc_mn_sw128(b0 + kk * 2 * ATOM, MN_STRIDE, ATOM), idesc,
                       (c == 0 && kk == 0) ? 0u : 1u);
          tc_commit(&empty[slot]);
        }
        tc_commit(&acc_full[ab]);  // also for an offset without pairs: the epilogue writes zeros
      }
      if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else if (warp < 6) {
    // ---- gatherers ----
    const int g = threadIdx.x - 64;
    // A: dOut[dst][o0 : o0 + 128] = 16 chunks of 16 bytes per pair; thread g copies chunk
    // g % 16 of pairs g / 16 + 8 * pass (pass = K group, 8 passes).
    const int ca = g % 16, ra = g / 16;
    const uint32_t a_off = (uint32_t)(ca / 8) * MN_STRIDE + (uint32_t)ra * 128u +
                           ((uint32_t)((ca % 8) ^ ra) << 4);
    // B: features[src][i0 : i0 + BN] = CB chunks per pair; RB pairs per pass.
    constexpr int CB = BN / 8, RB = 128 / CB, PB = WKC / RB;
    const int cb = g % CB, rb = g / CB;
    int it = 0;
    for (int local = 0; ok; ++local) {
      const int ws = local & 1;
      if (!mbar_wait_bounded(&work_full[ws], (local >> 1) & 1, s_abort)) {
        ok = false;
        break;
      }
      const WSlot w = slots[ws];
      if (w.k < 0) break;
      const int chunks = (w.end - w.begin + WKC - 1) / WKC;
      const T* a_src = dout + w.o0 + ca * 8;
      const T* b_src = feat + w.i0 + cb * 8;
      // pair indices of the next chunk, loaded one chunk ahead
      int32_t nd[8], ns[PB];
      auto load_idx = [&](int c) {
        const int32_t j0 = w.begin + c * WKC;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const int32_t j = j0 + ra + 8 * p;
          nd[p] = j < w.end ? __ldg(&pair_dst[j]) : -1;
        }
#pragma unroll
        for (int p = 0; p < PB; ++p) {
          const int32_t j = j0 + rb + RB * p;
          ns[p] = j < w.end ? __ldg(&pair_src[j]) : -1;
        }
      };
      if (chunks > 0) load_idx(0);
      for (int c = 0; c < chunks; ++c, ++it) {
        int32_t cd[8], cs[PB];
#pragma unroll
        for (int p = 0; p < 8; ++p) cd[p] = nd[p];
#pragma unroll
        for (int p = 0; p < PB; ++p) cs[p] = ns[p];
        if (c + 1 < chunks) load_idx(c + 1);
        const int slot = it % S;
        if (!mbar_wait_bounded(&empty[slot], ((it / S) & 1) ^ 1, s_abort)) {
          ok = false;
          break;
        }
        const uint32_t a_dst = smem_u32(sA + slot * L::A_STAGE) + a_off;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const bool v = cd[p] >= 0;
          cp_async_16(a_dst + (uint32_t)p * ATOM, a_src + (v ? (int64_t)cd[p] * cout : 0),
                      v ? 16u : 0u);
        }
        const uint32_t b_base = smem_u32(sB + slot * L::B_STAGE) + (uint32_t)(cb / 8) * MN_STRIDE;
#pragma unroll
        for (int p = 0; p < PB; ++p) {
          const int row = rb + RB * p;  // pair index within the chunk
          const uint32_t r = (uint32_t)(row & 7);
          const uint32_t dst = b_base + (uint32_t)(row >> 3) * ATOM + r * 128u +
                               ((uint32_t)((cb % 8) ^ (int)r) << 4);
          const bool v = cs[p] >= 0;
          cp_async_16(dst, b_src + (v ? (int64_t)cs[p] * cin : 0), v ? 16u : 0u);
        }
        cp_async_arrive_noinc(&full[slot]);
      }
    }
    if (!ok) {
      cp_async_wait_all();
      report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 * (w % 4) .. +31 (output channels) ----
    const int q = warp & 3;
    const int m = q * 32 + lane;
    for (int local = 0; ok; ++local) {
      const int ws = local & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&work_full[ws], (local >> 1) & 1, s_abort))) {
        ok = false;
        break;
      }
      const WSlot w = slots[ws];
      if (w.k < 0) break;
      const int ab = local & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&acc_full[ab], (local >> 1) & 1, s_abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool any = w.end > w.begin;
      const uint32_t t_row = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN);
      T* dst_row = dweight + ((int64_t)(w.o0 + m) * kvol + w.k) * cin + w.i0;
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t v[32];
        if (any) {
          tmem_ld_32x32b_x32(t_row + ch * 32, v);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0u;
        }
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          packed[j] = pack2w<T>(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
        uint4* d4 = reinterpret_cast<uint4*>(dst_row + ch * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2],
                             packed[4 * j + 3]);
      }
      tc_fence_before();
      mbar_arrive_w(&acc_empty[ab]);
      mbar_arrive_w(&work_empty[ws]);
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

template <int BN, typename T>
int launch_wgrad(const void* feat, const void* dout, int cin, int cout, int kvol,
                 const int32_t* offsets, const int32_t* src, const int32_t* dst, void* dweight,
                 int32_t* counter, int32_t* status, cudaStream_t s) {
  using L = WLayout<BN>;
  int dev = 0;
  SV_CUDA_TRY(cudaGetDevice(&dev));
  static bool attr_done[256] = {};
  if (dev >= 256 || !attr_done[dev]) {
    SV_CUDA_TRY(cudaFuncSetAttribute(wgrad_tc_kernel<BN, T>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM));
    if (dev < 256) attr_done[dev] = true;
  }
  WSched sc;
  sc.counter = counter;
  sc.o_tiles = cout / WM;
  sc.i_tiles = cin / BN;
  const int64_t items = (int64_t)kvol * sc.o_tiles * sc.i_tiles;
  if (items > INT32_MAX / 2) SV_FAIL(SV_ERR_UNSUPPORTED, "too many weight-gradient items");
  sc.total_items = (int32_t)items;
  const int grid = (int)std::min<int64_t>(items, num_sms());
  SV_CUDA_TRY(cudaMemsetAsync(counter, 0, sizeof(int32_t), s));
  wgrad_tc_kernel<BN, T><<<grid, WTHREADS, L::SMEM, s>>>(
      static_cast<const T*>(feat), static_cast<const T*>(dout), cin, cout, kvol, offsets, src,
      dst, static_cast<T*>(dweight), sc, status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

template <typename T>
int launch_wgrad_typed(const void* feat, const void* dout, int cin, int cout, int kvol,
                       const int32_t* offsets, const int32_t* src, const int32_t* dst,
                       void* dweight, int32_t* counter, int32_t* status, cudaStream_t s) {
  if (cin % 256 == 0)
    return launch_wgrad<256, T>(feat, dout, cin, cout, kvol, offsets, src, dst, dweight, counter,
                                status, s);
  if (cin % 128 == 0)
    return launch_wgrad<128, T>(feat, dout, cin, cout, kvol, offsets, src, dst, dweight, counter,
                                status, s);
  return launch_wgrad<64, T>(feat, dout, cin, cout, kvol, offsets, src, dst, dweight, counter,
                             status, s);
}

}  // namespace
}  // namespace sv

using namespace sv;

// Not exported: sv_conv3d_wgrad (backward.cu) dispatches here.
extern "C" int sv_conv3d_wgrad_tc_supported(int cin, int cout, int kvol, int dtype) {
  return (dtype == SV_FLOAT16 || dtype == SV_BFLOAT16) && cin > 0 && cin % 64 == 0 &&
         cout > 0 && cout % WM == 0 && kvol >= 1 && kvol <= 65535;
}

extern "C" int sv_conv3d_wgrad_tc(const void* features, const void* dout, int cin, int cout,
                                  int kvol, const int32_t* offsets, const int32_t* pair_src,
                                  const int32_t* pair_dst, int dtype, void* dweight,
                                  void* workspace, size_t workspace_bytes, int32_t* status,
                                  sv_stream_t stream) {
  if (!sv_conv3d_wgrad_tc_supported(cin, cout, kvol, dtype))
    SV_FAIL(SV_ERR_UNSUPPORTED,
            "tcgen05 weight gradient needs fp16/bf16, Cin % 64 == 0 and Cout % 128 == 0");
  if (!features || !dout || !offsets || !pair_src || !pair_dst || !dweight)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_wgrad_tc: null pointer");
  if (!aligned16(features) || !aligned16(dout) || !aligned16(dweight))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_conv3d_wgrad_tc: operands must be 16-byte aligned");
  if (!workspace || workspace_bytes < 256 || !aligned16(workspace))
    SV_FAIL(SV_ERR_WORKSPACE, "sv_conv3d_wgrad_tc: needs 256 bytes of workspace");
  cudaStream_t s = to_stream(stream);
  int32_t* counter = static_cast<int32_t*>(workspace);
  if (dtype == SV_BFLOAT16)
    return launch_wgrad_typed<__nv_bfloat16>(features, dout, cin, cout, kvol, offsets, pair_src,
                                             pair_dst, dweight, counter, status, s);
  return launch_wgrad_typed<__half>(features, dout, cin, cout, kvol, offsets, pair_src, pair_dst,
                                    dweight, counter, status, s);
}
