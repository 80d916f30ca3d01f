// Output-stationary sparse convolution on the CUDA cores (fp32 FFMA).
//
// Computes the Metal kernel's result (src/mlx_diffuser/kernels/sparse.py:14-34): for every
// output row, bias plus the sum over kernel offsets with a valid neighbour of the neighbour's
// feature row times W[k], accumulated in fp32 and rounded once. It serves fp32 features and
// the shapes the tcgen05 kernel does not take (Cin not a multiple of 64, Cout not a multiple
// of 32, kernel volume above 27).
//
// Generic kernel (any dtype, shape and layout): a CTA owns a 64-row x 64-column output tile.
// For each offset it stages the 64 gathered neighbour indices; offsets with no valid neighbour in
// the tile are skipped as a whole. The K loop stages a gathered 64x16 slab of features and a
// 16x64 slab of W[k] in shared memory; each thread accumulates a 4x4 block. fp32 with aligned
// shapes takes the faster kernel below.
#include "conv.h"

namespace sv {
namespace {

constexpr int SBM = 64, SBN = 64, SBK = 16;

template <typename T, int LAYOUT>
__global__ void __launch_bounds__(256) conv_simt_kernel(
    const T* __restrict__ feat, int64_t n, int64_t n_rows, int cin,
    const int32_t* __restrict__ nbr, int kvol,
    const int32_t* __restrict__ row_order, const T* __restrict__ w, const T* __restrict__ bias,
    const T* residual, int cout, T* out, int32_t* status) {
  __shared__ __align__(16) float As[SBK][SBM];
  __shared__ __align__(16) float Bs[SBK][SBN];
  __shared__ int32_t s_src[SBM];
  __shared__ int32_t s_orow[SBM];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t row0 = (int64_t)blockIdx.x * SBM;
  const int col0 = blockIdx.y * SBN;
  if (tid < SBM) {
    const int64_t g = row0 + tid;
    int32_t o = -1;
    if (g < n_rows) {
      o = row_order ? __ldg(&row_order[g]) : (int32_t)g;
      if (o < -1 || o >= n) {  // -1: padding between schedule segments
        report(status, SV_DEVICE_BAD_INDEX);
        o = -1;
      }
    }
    s_orow[tid] = o;
  }
  __syncthreads();
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k = 0; k < kvol; ++k) {
    int valid = 0;
    if (tid < SBM) {
      const int32_t o = s_orow[tid];
      int32_t src = o >= 0 ? __ldg(&nbr[(int64_t)o * kvol + k]) : -1;
      if (src >= n) {
        report(status, SV_DEVICE_BAD_INDEX);
        src = -1;
      }
      s_src[tid] = src;
      valid = src >= 0;
    }
    if (!__syncthreads_or(valid)) continue;
    for (int c0 = 0; c0 < cin; c0 += SBK) {
#pragma unroll
      for (int i = 0; i < (SBM * SBK) / 256; ++i) {
        const int e = tid + i * 256;
        const int r = e / SBK, kk = e % SBK;
        const int32_t src = s_src[r];
        const int ci = c0 + kk;
        As[kk][r] = (src >= 0 && ci < cin) ? to_f32(feat[(int64_t)src * cin + ci]) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < (SBK * SBN) / 256; ++i) {
        const int e = tid + i * 256;
        int kk, j;
        if (LAYOUT == SV_WEIGHT_KIO) {
          kk = e / SBN;
          j = e % SBN;
        } else {
          kk = e % SBK;
          j = e / SBK;
        }
        const int ci = c0 + kk, co = col0 + j;
        float v = 0.f;
        if (ci < cin && co < cout) {
          v = LAYOUT == SV_WEIGHT_KIO ? to_f32(w[((int64_t)k * cin + ci) * cout + co])
                                      : to_f32(w[((int64_t)co * kvol + k) * cin + ci]);
        }
        Bs[kk][j] = v;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < SBK; ++kk) {
        const float4 a = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
        const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
        const float av[4] = {a.x, a.y, a.z, a.w};
        const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int32_t o = s_orow[ty * 4 + i];
    if (o < 0) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int co = col0 + tx * 4 + j;
      if (co < cout) {
        const float b = bias ? to_f32(bias[co]) : 0.f;
        const float r = residual ? to_f32(residual[(int64_t)o * cout + co]) : 0.f;
        out[(int64_t)o * cout + co] = from_f32<T>(acc[i][j] + b + r);
      }
    }
  }
}

// ---- fp32 fast path ---------------------------------------------------------------------------
// For fp32 with Cin and Cout multiples of 4 and at most 27 offsets (every fp32 convolution of the
// reference's models): a CTA owns 128 output rows x 64 output channels and each of its 256
// threads an 8 x 4 block. The 128 rows' neighbour lists are staged once; offsets that no row of
// the tile has are skipped. The K loop runs over (offset, 16-channel chunk) with 16-byte gathers
// of feature rows and weight rows, the next chunk loaded into registers while the current one is
// multiplied out of shared memory (double-buffered, one barrier per chunk).
constexpr int FBM = 128, FBN = 64, FBK = 16, FKMAX = 27;

template <int LAYOUT>
__global__ void __launch_bounds__(256) conv_f32_kernel(
    const float* __restrict__ feat, int64_t n, int64_t n_rows, int cin,
    const int32_t* __restrict__ nbr, int kvol, const int32_t* __restrict__ row_order,
    const float* __restrict__ w, const float* __restrict__ bias, const float* residual,
    int cout, float* out, int32_t* status) {
  __shared__ __align__(16) float As[2][FBK][FBM + 4];
  __shared__ __align__(16) float Bs[2][FBK][FBN + 4];
  __shared__ int32_t s_src[FKMAX][FBM];
  __shared__ int32_t s_orow[FBM];
  __shared__ uint32_t s_mask;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t row0 = (int64_t)blockIdx.x * FBM;
  const int col0 = blockIdx.y * FBN;
  if (tid == 0) s_mask = 0;
  __syncthreads();
  if (tid < FBM) {  // warps 0-3: one tile row each
    const int64_t g = row0 + tid;
    int32_t o = -1;
    if (g < n_rows) {
      o = row_order ? __ldg(&row_order[g]) : (int32_t)g;
      if (o < -1 || o >= n) {  // -1: padding between schedule segments
        report(status, SV_DEVICE_BAD_INDEX);
        o = -1;
      }
    }
    s_orow[tid] = o;
    uint32_t m = 0;
    for (int k = 0; k < kvol; ++k) {
      int32_t src = o >= 0 ? __ldg(&nbr[(int64_t)o * kvol + k]) : -1;
      if (src >= n) {
        report(status, SV_DEVICE_BAD_INDEX);
        src = -1;
      }
      s_src[k][tid] = src;
      m |= (uint32_t)(src >= 0) << k;
    }
    m = __reduce_or_sync(0xffffffffu, m);
    if ((tid & 31) == 0) atomicOr(&s_mask, m);
  }
  __syncthreads();
  uint32_t mask = s_mask;
  const int chunks = (cin + FBK - 1) / FBK;
  const int total = __popc(mask) * chunks;

  // load assignment: A = 128 rows x 16 channels (2 float4 per thread), B = 64 x 16 (1 float4)
  const int ra = tid >> 2, ca = (tid & 3) * 4;
  float4 pa[2], pb;
  auto load = [&](int k, int c0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int32_t src = s_src[k][ra + 64 * i];
      const int ci = c0 + ca;
      pa[i] = (src >= 0 && ci < cin)
                  ? __ldg(reinterpret_cast<const float4*>(feat + (int64_t)src * cin + ci))
                  : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (LAYOUT == SV_WEIGHT_OKI) {
      const int co = col0 + (tid >> 2), ci = c0 + (tid & 3) * 4;
      pb = (co < cout && ci < cin)
               ? __ldg(reinterpret_cast<const float4*>(w + ((int64_t)co * kvol + k) * cin + ci))
               : make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      const int ci = c0 + (tid >> 4), co = col0 + (tid & 15) * 4;
      pb = (ci < cin && co < cout)
               ? __ldg(reinterpret_cast<const float4*>(w + ((int64_t)k * cin + ci) * cout + co))
               : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int r = ra + 64 * i;
      As[buf][ca + 0][r] = pa[i].x;
      As[buf][ca + 1][r] = pa[i].y;
      As[buf][ca + 2][r] = pa[i].z;
      As[buf][ca + 3][r] = pa[i].w;
    }
    if (LAYOUT == SV_WEIGHT_OKI) {
      const int j = tid >> 2, kk = (tid & 3) * 4;
      Bs[buf][kk + 0][j] = pb.x;
      Bs[buf][kk + 1][j] = pb.y;
      Bs[buf][kk + 2][j] = pb.z;
      Bs[buf][kk + 3][j] = pb.w;
    } else {
      *reinterpret_cast<float4*>(&Bs[buf][tid >> 4][(tid & 15) * 4]) = pb;
    }
  };

  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  if (total > 0) {
    int k = __ffs(mask) - 1, c0 = 0;
    load(k, c0);
    store(0);
    __syncthreads();
    for (int it = 0; it < total; ++it) {
      const int buf = it & 1;
      const bool more = it + 1 < total;
      if (more) {  // advance to the next (offset, chunk) and fetch it into registers
        c0 += FBK;
        if (c0 >= cin) {
          c0 = 0;
          mask &= mask - 1;
          k = __ffs(mask) - 1;
        }
        load(k, c0);
      }
#pragma unroll
      for (int kk = 0; kk < FBK; ++kk) {
        const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8]);
        const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8 + 4]);
        const float4 b = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
      if (more) store(buf ^ 1);
      __syncthreads();
    }
  }

  const int co = col0 + tx * 4;
  if (co >= cout) return;
  float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
  if (bias) bv = __ldg(reinterpret_cast<const float4*>(bias + co));
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int32_t o = s_orow[ty * 8 + i];
    if (o < 0) continue;
    float4 v = make_float4(acc[i][0] + bv.x, acc[i][1] + bv.y, acc[i][2] + bv.z,
                           acc[i][3] + bv.w);
    if (residual) {
      const float4 r = *reinterpret_cast<const float4*>(residual + (int64_t)o * cout + co);
      v.x += r.x;
      v.y += r.y;
      v.z += r.z;
      v.w += r.w;
    }
    *reinterpret_cast<float4*>(out + (int64_t)o * cout + co) = v;
  }
}

bool f32_fast_path(const ConvArgs& a) {
  return a.dtype == SV_FLOAT32 && a.cin % 4 == 0 && a.cout % 4 == 0 && a.kvol <= FKMAX &&
         aligned16(a.features) && aligned16(a.weight) && aligned16(a.out) &&
         aligned16(a.bias) && aligned16(a.residual);
}

int launch_f32_fast(const ConvArgs& a, cudaStream_t s) {
  const dim3 grid((unsigned)((a.n_rows + FBM - 1) / FBM), (unsigned)((a.cout + FBN - 1) / FBN));
  const float* f = static_cast<const float*>(a.features);
  const float* w = static_cast<const float*>(a.weight);
  const float* b = static_cast<const float*>(a.bias);
  const float* r = static_cast<const float*>(a.residual);
  float* o = static_cast<float*>(a.out);
  if (a.layout == SV_WEIGHT_KIO)
    conv_f32_kernel<SV_WEIGHT_KIO><<<grid, 256, 0, s>>>(f, a.n, a.n_rows, a.cin, a.nbr, a.kvol,
                                                        a.row_order, w, b, r, a.cout, o,
                                                        a.status);
  else
    conv_f32_kernel<SV_WEIGHT_OKI><<<grid, 256, 0, s>>>(f, a.n, a.n_rows, a.cin, a.nbr, a.kvol,
                                                        a.row_order, w, b, r, a.cout, o,
                                                        a.status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

template <typename T>
int launch_typed(const ConvArgs& a, cudaStream_t s) {
  const dim3 grid((unsigned)((a.n_rows + SBM - 1) / SBM), (unsigned)((a.cout + SBN - 1) / SBN));
  const T* f = static_cast<const T*>(a.features);
  const T* w = static_cast<const T*>(a.weight);
  const T* b = static_cast<const T*>(a.bias);
  const T* r = static_cast<const T*>(a.residual);
  T* o = static_cast<T*>(a.out);
  if (a.layout == SV_WEIGHT_KIO)
    conv_simt_kernel<T, SV_WEIGHT_KIO><<<grid, 256, 0, s>>>(f, a.n, a.n_rows, a.cin, a.nbr, a.kvol,
                                                            a.row_order, w, b, r, a.cout, o,
                                                            a.status);
  else
    conv_simt_kernel<T, SV_WEIGHT_OKI><<<grid, 256, 0, s>>>(f, a.n, a.n_rows, a.cin, a.nbr, a.kvol,
                                                            a.row_order, w, b, r, a.cout, o,
                                                            a.status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

}  // namespace

int conv_simt_launch(const ConvArgs& a, cudaStream_t s) {
  if (a.n_rows == 0 || a.cout == 0) return SV_OK;
  if ((a.n_rows + SBM - 1) / SBM > INT32_MAX || (a.cout + SBN - 1) / SBN > 65535)
    SV_FAIL(SV_ERR_UNSUPPORTED, "conv: problem too large for the grid");
  switch (a.dtype) {
    case SV_FLOAT32: return f32_fast_path(a) ? launch_f32_fast(a, s) : launch_typed<float>(a, s);
    case SV_FLOAT16: return launch_typed<__half>(a, s);
    case SV_BFLOAT16: return launch_typed<__nv_bfloat16>(a, s);
  }
  SV_FAIL(SV_ERR_BAD_DTYPE, "conv: unknown dtype");
}

}  // namespace sv
