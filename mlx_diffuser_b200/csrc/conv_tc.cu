// Output-stationary sparse convolution on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Computes the Metal kernel's result (src/mlx_diffuser/kernels/sparse.py:14-34) for fp16/bf16
// features: out[p, o] = bias[o] + sum over offsets k with nbr[p,k] >= 0 of
// features[nbr[p,k]] . W[k][:, o], accumulated in fp32 (TMEM) and rounded once.
//
// Shape of the computation: an implicit GEMM whose M dimension is output rows, N is Cout and
// K is (offset, input channel). A CTA owns 128 output rows (the rows of `row_order`, which
// groups rows with equal neighbour masks) x BN output channels. Its K loop visits only the
// offsets for which at least one of its 128 rows has a neighbour -- the union of the rows'
// masks -- and within an offset walks Cin in 64-channel stages.
//
// Warp roles (192 threads):
//   warp 0      TMA producer: W[k][kb*64 : +64, n0 : n0+BN] from the spconv (Cout, K*Cin)
//               matrix, K-major, 128-byte swizzle, one tiled 2-D load per stage;
//   warp 1      TMEM allocator and the single thread that issues tcgen05.mma (M=128,
//               N=BN, K=16, four per stage) and tcgen05.commit;
//   warps 2-5   gatherers: the A stage (128 neighbour rows x 128 bytes) is copied with
//               16-byte cp.async, eight threads per row so each warp instruction reads four
//               whole rows (zero-filled when the neighbour is missing), into the same 128-byte
//               swizzle TMA would write. Then the same warps run the epilogue: tcgen05.ld of
//               32 accumulator columns at a time, + bias, round, 16-byte stores to the row's
//               output.
// Stages are a 4-deep ring of (A 16 KB, B BN*128 B) guarded by full/empty mbarriers. Every
// wait is bounded: on expiry the kernel ORs SV_DEVICE_WAIT_TIMEOUT into the status word,
// drains its own copies and frees TMEM.
#include <type_traits>

#include "conv.h"

namespace sv {
namespace {

constexpr int TBM = 128;       // output rows per tile == TMEM lanes
constexpr int TBK = 64;        // input channels per stage == one 128-byte swizzle row
constexpr int TSTAGES = 4;
constexpr int TTHREADS = 192;
constexpr int TMAX_KVOL = 27;
constexpr int A_STAGE_BYTES = TBM * TBK * 2;

template <int BN>
struct TcLayout {
  static constexpr int B_STAGE_BYTES = BN * TBK * 2;
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = TSTAGES * A_STAGE_BYTES;
  static constexpr int NBR_OFF = B_OFF + TSTAGES * B_STAGE_BYTES;
  static constexpr int OROW_OFF = NBR_OFF + TBM * TMAX_KVOL * 4;
  static constexpr int BAR_OFF = OROW_OFF + TBM * 4;
  static constexpr int MISC_OFF = BAR_OFF + (2 * TSTAGES + 1) * 8;
  static constexpr int BYTES = MISC_OFF + 16;
  static constexpr int SMEM = BYTES + 1024;  // slack for aligning the base to 1024 bytes
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
  static_assert(BAR_OFF % 8 == 0, "mbarriers need 8-byte alignment");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
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

template <int BN, typename T>
__global__ void __launch_bounds__(TTHREADS, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const T* __restrict__ feat,
                   int n, int cin, const int32_t* __restrict__ nbr, int kvol,
                   const int32_t* __restrict__ row_order, const T* __restrict__ bias, int cout,
                   T* __restrict__ out, int32_t* status) {
  using L = TcLayout<BN>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem + L::A_OFF;
  uint8_t* sB = smem + L::B_OFF;
  int32_t* s_nbr = reinterpret_cast<int32_t*>(smem + L::NBR_OFF);
  int32_t* s_orow = reinterpret_cast<int32_t*>(smem + L::OROW_OFF);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + TSTAGES;
  uint64_t* accum = empty + TSTAGES;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  uint32_t* s_union = s_tmem + 1;
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t tile0 = (int64_t)blockIdx.x * TBM;
  const int n0 = blockIdx.y * BN;
  const int kb_per_k = cin / TBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TSTAGES; ++s) {
      mbar_init(&full[s], 1 + TBM);  // TMA expect_tx arrival + one cp.async arrival per row
      mbar_init(&empty[s], 1);       // tcgen05.commit
    }
    mbar_init(accum, 1);
    *s_union = 0;
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&tmap_w);
  if (warp == 1) {
    tmem_alloc(s_tmem, L::TMEM_COLS);
    tmem_relinquish();
  }
  uint32_t my_mask = 0;
  if (warp >= 2) {
    const int r = threadIdx.x - 64;
    const int64_t g = tile0 + r;
    int32_t orow = -1;
    if (g < n) {
      orow = row_order ? __ldg(&row_order[g]) : (int32_t)g;
      if (orow < 0 || orow >= n) {
        report(status, SV_DEVICE_BAD_INDEX);
        orow = -1;
      }
    }
    s_orow[r] = orow;
    // independent loads (unrolled to the 27-offset bound) so their latencies overlap
    const int32_t* nrow = nbr + (int64_t)(orow >= 0 ? orow : 0) * kvol;
#pragma unroll
    for (int k = 0; k < TMAX_KVOL; ++k) {
      if (k < kvol) {
        int32_t v = orow >= 0 ? __ldg(&nrow[k]) : -1;
        if (v >= n) {
          report(status, SV_DEVICE_BAD_INDEX);
          v = -1;
        }
        s_nbr[r * TMAX_KVOL + k] = v;
        my_mask |= (uint32_t)(v >= 0) << k;
      }
    }
  }
  __syncthreads();
  if (warp >= 2) {
    const uint32_t m = __reduce_or_sync(0xffffffffu, my_mask);
    if (lane == 0) atomicOr(s_union, m);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t umask = *s_union;
  const uint32_t tmem = *s_tmem;
  const int total = __popc(umask) * kb_per_k;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (uint32_t m = umask; m != 0 && ok; m &= m - 1) {
        const int k = __ffs(m) - 1;
        for (int kb = 0; kb < kb_per_k; ++kb, ++it) {
          const int slot = it % TSTAGES;
          const uint32_t ph = (it / TSTAGES) & 1;
          if (!mbar_wait_bounded(&empty[slot], ph ^ 1, s_abort)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[slot], L::B_STAGE_BYTES);
          tma_load_2d(smem_u32(sB + slot * L::B_STAGE_BYTES), &tmap_w, &full[slot],
                      k * cin + kb * TBK, n0);
        }
      }
      if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kBF16, TBM, BN);
      int it = 0;
      for (uint32_t m = umask; m != 0 && ok; m &= m - 1) {
        for (int kb = 0; kb < kb_per_k; ++kb, ++it) {
          const int slot = it % TSTAGES;
          const uint32_t ph = (it / TSTAGES) & 1;
          if (!mbar_wait_bounded(&full[slot], ph, s_abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          fence_proxy_async_smem();  // cp.async wrote A through the generic proxy
          const uint32_t a0 = smem_u32(sA + slot * A_STAGE_BYTES);
          const uint32_t b0 = smem_u32(sB + slot * L::B_STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < TBK / 16; ++kk)
            tc_mma_f16(tmem, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32),
                       idesc, (it | kk) != 0 ? 1u : 0u);
          tc_commit(&empty[slot]);
        }
      }
      tc_commit(accum);  // also issued after a timeout, so the epilogue never waits on nothing
      if (!ok) report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
  } else {
    // ---- gather ----
    // Gatherer g copies 16-byte chunk (g % 8) of tile rows g/8 + 16*i, i = 0..7: one warp
    // instruction moves four whole 128-byte rows, so every L2 sector it touches is used in full.
    const int g = threadIdx.x - 64;
    const uint32_t chunk = g & 7;
    const int row0 = g >> 3;
    const uint32_t swz = ((chunk ^ (uint32_t)(row0 & 7)) << 4);  // (row0 + 16*i) & 7 == row0 & 7
    int it = 0;
    for (uint32_t m = umask; m != 0 && ok; m &= m - 1) {
      const int k = __ffs(m) - 1;
      const T* src[8];
      uint32_t nbytes[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int32_t s_row = s_nbr[(row0 + 16 * i) * TMAX_KVOL + k];
        src[i] = feat + (s_row >= 0 ? (int64_t)s_row * cin : 0) + chunk * 8;
        nbytes[i] = s_row >= 0 ? 16u : 0u;
      }
      for (int kb = 0; kb < kb_per_k; ++kb, ++it) {
        const int slot = it % TSTAGES;
        const uint32_t ph = (it / TSTAGES) & 1;
        if (!mbar_wait_bounded(&empty[slot], ph ^ 1, s_abort)) {
          ok = false;
          break;
        }
        const uint32_t dst = smem_u32(sA + slot * A_STAGE_BYTES) + (uint32_t)row0 * 128u + swz;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          cp_async_16(dst + (uint32_t)(16 * i) * 128u, src[i] + kb * TBK, nbytes[i]);
        cp_async_arrive_noinc(&full[slot]);
      }
    }
    if (!ok) {
      cp_async_wait_all();
      report(status, SV_DEVICE_WAIT_TIMEOUT);
    }
    // ---- epilogue: this warp may read TMEM lanes 32*(warp % 4) .. +31 ----
    const int q = warp & 3;
    const int32_t orow = s_orow[q * 32 + lane];
    if (!mbar_wait_bounded(accum, 0, s_abort)) report(status, SV_DEVICE_WAIT_TIMEOUT);
    tc_fence_after();
    const uint32_t t_row = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
    for (int ch = 0; ch < BN / 32; ++ch) {
      uint32_t v[32];
      if (total > 0) {
        tmem_ld_32x32b_x32(t_row + ch * 32, v);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0u;
      }
      if (orow >= 0) {
        const int c0 = n0 + ch * 32;
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float lo = __uint_as_float(v[2 * j]);
          float hi = __uint_as_float(v[2 * j + 1]);
          if (bias) {
            lo += to_f32(bias[c0 + 2 * j]);
            hi += to_f32(bias[c0 + 2 * j + 1]);
          }
          packed[j] = pack2<T>(lo, hi);
        }
        uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)orow * cout + c0);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          dst[j] =
              make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
      }
    }
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

template <int BN, typename T>
int launch_bn(const ConvArgs& a, cudaStream_t s) {
  using L = TcLayout<BN>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  int dev = 0;
  SV_CUDA_TRY(cudaGetDevice(&dev));
  static bool attr_done[128] = {};
  if (dev >= 128 || !attr_done[dev]) {
    SV_CUDA_TRY(cudaFuncSetAttribute(conv_tc_kernel<BN, T>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM));
    if (dev < 128) attr_done[dev] = true;
  }
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr) SV_FAIL(SV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  CUtensorMap tmap;
  const cuuint64_t gdim[2] = {(cuuint64_t)a.kvol * a.cin, (cuuint64_t)a.cout};
  const cuuint64_t gstride[1] = {(cuuint64_t)a.kvol * a.cin * 2};
  const cuuint32_t box[2] = {(cuuint32_t)TBK, (cuuint32_t)BN};
  const cuuint32_t estride[2] = {1, 1};
  CUresult cr = encode(&tmap,
                       kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                       2, const_cast<void*>(a.weight), gdim, gstride, box, estride,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) SV_FAIL(SV_ERR_CUDA, "cuTensorMapEncodeTiled failed for the weight");
  const dim3 grid((unsigned)((a.n + TBM - 1) / TBM), (unsigned)(a.cout / BN));
  conv_tc_kernel<BN, T><<<grid, TTHREADS, L::SMEM, s>>>(
      tmap, static_cast<const T*>(a.features), (int)a.n, a.cin, a.nbr, a.kvol, a.row_order,
      static_cast<const T*>(a.bias), a.cout, static_cast<T*>(a.out), a.status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

template <typename T>
int launch_typed(const ConvArgs& a, cudaStream_t s) {
  if (a.cout % 256 == 0) return launch_bn<256, T>(a, s);
  if (a.cout % 128 == 0) return launch_bn<128, T>(a, s);
  if (a.cout % 64 == 0) return launch_bn<64, T>(a, s);
  return launch_bn<32, T>(a, s);
}

}  // namespace

bool conv_tc_supported(const ConvArgs& a) {
  return (a.dtype == SV_FLOAT16 || a.dtype == SV_BFLOAT16) && a.layout == SV_WEIGHT_OKI &&
         a.cin > 0 && a.cin % TBK == 0 && a.cout > 0 && a.cout % 32 == 0 && a.kvol >= 1 &&
         a.kvol <= TMAX_KVOL && a.n <= INT32_MAX && (int64_t)a.kvol * a.cin < INT32_MAX &&
         aligned16(a.features) && aligned16(a.weight) && aligned16(a.out);
}

int conv_tc_launch(const ConvArgs& a, cudaStream_t s) {
  if (a.n == 0) return SV_OK;
  if (!conv_tc_supported(a))
    SV_FAIL(SV_ERR_UNSUPPORTED, "shape not supported by the tcgen05 kernel");
  if (a.dtype == SV_BFLOAT16) return launch_typed<__nv_bfloat16>(a, s);
  return launch_typed<__half>(a, s);
}

}  // namespace sv
