// Fused row normalisation of the sparse residual block.
//
// The reference's _SparseResBlock3D (src/mlx_diffuser/models/trellis_slat.py:71-82) runs, around
// its two convolutions,
//     a = silu(LayerNorm32_affine(x))                        (norm1, :77)
//     b = silu(LayerNorm32(h) * (1 + scale[batch]) + shift[batch])   (norm2 + modulation, :79-80)
// as separate element-wise passes. LayerNorm32 (src/mlx_diffuser/layers/trellis.py:16-43) takes
// the mean and the mean squared deviation of each row in fp32, scales by rsqrt(var + eps), applies
// the fp32 affine weight and bias when it has them, and casts back to the feature type. Here one
// kernel does the whole chain per row: one warp per row, the row held in registers, fp32
// throughout, one rounding at the end. `scale` / `shift` are the (B, C) embedding projections,
// picked per row by its batch index (coords column 0), as SparseTensor's broadcasting does
// (src/mlx_diffuser/layers/sparse.py:102-109).
#include "common.cuh"

namespace sv {
namespace {

constexpr int NORM_THREADS = 256;
constexpr int NORM_ROWS = NORM_THREADS / 32;

template <typename T>
struct Pair;
template <>
struct Pair<float> {
  using V = float2;
  static __device__ __forceinline__ float2 load(const float* p) {
    return *reinterpret_cast<const float2*>(p);
  }
  static __device__ __forceinline__ void store(float* p, float a, float b) {
    *reinterpret_cast<float2*>(p) = make_float2(a, b);
  }
  static __device__ __forceinline__ float lo(float2 v) { return v.x; }
  static __device__ __forceinline__ float hi(float2 v) { return v.y; }
};
template <>
struct Pair<__half> {
  using V = __half2;
  static __device__ __forceinline__ __half2 load(const __half* p) {
    return *reinterpret_cast<const __half2*>(p);
  }
  static __device__ __forceinline__ void store(__half* p, float a, float b) {
    *reinterpret_cast<__half2*>(p) = __floats2half2_rn(a, b);
  }
  static __device__ __forceinline__ float lo(__half2 v) { return __low2float(v); }
  static __device__ __forceinline__ float hi(__half2 v) { return __high2float(v); }
};
template <>
struct Pair<__nv_bfloat16> {
  using V = __nv_bfloat162;
  static __device__ __forceinline__ __nv_bfloat162 load(const __nv_bfloat16* p) {
    return *reinterpret_cast<const __nv_bfloat162*>(p);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
  }
  static __device__ __forceinline__ float lo(__nv_bfloat162 v) { return __low2float(v); }
  static __device__ __forceinline__ float hi(__nv_bfloat162 v) { return __high2float(v); }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float silu(float y) { return y / (1.0f + expf(-y)); }

struct NormArgs {
  int64_t n;
  int channels;
  float eps;
  const float* weight;  // [C] or null
  const float* bias;    // [C] or null
  const int32_t* coords;
  int64_t batch;
  int silu;
  int32_t* status;
};

// Lane l holds channel pairs 2*(l + 32*j), j < MAXJ: a warp instruction touches one contiguous
// 64-pair stretch of the row.
template <typename T, int MAXJ>
__global__ void __launch_bounds__(NORM_THREADS)
    rownorm_kernel(const T* x, NormArgs a, const T* __restrict__ scale,
                   const T* __restrict__ shift, T* out) {
  using P = Pair<T>;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * NORM_ROWS + (threadIdx.x >> 5);
  if (row >= a.n) return;
  const int C = a.channels;
  const T* xr = x + row * C;
  float v[2 * MAXJ];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < MAXJ; ++j) {
    const int c = 2 * (lane + 32 * j);
    if (c < C) {
      const typename P::V p = P::load(xr + c);
      v[2 * j] = P::lo(p);
      v[2 * j + 1] = P::hi(p);
      sum += v[2 * j] + v[2 * j + 1];
    }
  }
  const float mean = warp_sum(sum) / (float)C;
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < MAXJ; ++j) {
    if (2 * (lane + 32 * j) < C) {
      const float d0 = v[2 * j] - mean, d1 = v[2 * j + 1] - mean;
      sq += d0 * d0 + d1 * d1;
    }
  }
  const float rstd = rsqrtf(warp_sum(sq) / (float)C + a.eps);
  const T* sc = nullptr;
  const T* sh = nullptr;
  if (scale || shift) {
    const int32_t b = __ldg(&a.coords[row * 4]);
    if (b < 0 || b >= a.batch) {
      if (lane == 0) report(a.status, SV_DEVICE_BAD_INDEX);
    } else {
      sc = scale ? scale + (int64_t)b * C : nullptr;
      sh = shift ? shift + (int64_t)b * C : nullptr;
    }
  }
  T* orow = out + row * C;
#pragma unroll
  for (int j = 0; j < MAXJ; ++j) {
    const int c = 2 * (lane + 32 * j);
    if (c < C) {
      float y0 = (v[2 * j] - mean) * rstd, y1 = (v[2 * j + 1] - mean) * rstd;
      if (a.weight) {
        y0 = y0 * __ldg(&a.weight[c]) + (a.bias ? __ldg(&a.bias[c]) : 0.f);
        y1 = y1 * __ldg(&a.weight[c + 1]) + (a.bias ? __ldg(&a.bias[c + 1]) : 0.f);
      }
      if (sc) {
        const typename P::V s = P::load(sc + c);
        y0 *= 1.0f + P::lo(s);
        y1 *= 1.0f + P::hi(s);
      }
      if (sh) {
        const typename P::V s = P::load(sh + c);
        y0 += P::lo(s);
        y1 += P::hi(s);
      }
      if (a.silu) {
        y0 = silu(y0);
        y1 = silu(y1);
      }
      P::store(orow + c, y0, y1);
    }
  }
}

template <typename T, int MAXJ>
void launch_norm(const void* x, const NormArgs& a, const void* scale, const void* shift,
                 void* out, cudaStream_t s) {
  const unsigned blocks = (unsigned)((a.n + NORM_ROWS - 1) / NORM_ROWS);
  rownorm_kernel<T, MAXJ><<<blocks, NORM_THREADS, 0, s>>>(
      static_cast<const T*>(x), a, static_cast<const T*>(scale), static_cast<const T*>(shift),
      static_cast<T*>(out));
}

template <typename T>
int launch_norm_typed(const void* x, const NormArgs& a, const void* scale, const void* shift,
                      void* out, cudaStream_t s) {
  const int c = a.channels;
  if (c <= 128) launch_norm<T, 2>(x, a, scale, shift, out, s);
  else if (c <= 256) launch_norm<T, 4>(x, a, scale, shift, out, s);
  else if (c <= 512) launch_norm<T, 8>(x, a, scale, shift, out, s);
  else if (c <= 1024) launch_norm<T, 16>(x, a, scale, shift, out, s);
  else if (c <= 2048) launch_norm<T, 32>(x, a, scale, shift, out, s);
  else launch_norm<T, 64>(x, a, scale, shift, out, s);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

}  // namespace
}  // namespace sv

using namespace sv;

extern "C" int sv_rownorm(const void* x, int64_t n, int channels, int dtype, float eps,
                          const float* weight, const float* bias, const void* scale,
                          const void* shift, const int32_t* coords, int64_t batch, int silu,
                          void* out, int32_t* status, sv_stream_t stream) {
  if (n < 0 || channels < 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_rownorm: negative size");
  if (dtype != SV_FLOAT32 && dtype != SV_FLOAT16 && dtype != SV_BFLOAT16)
    SV_FAIL(SV_ERR_BAD_DTYPE, "sv_rownorm: unknown dtype");
  if (channels % 2 != 0 || channels > 4096)
    SV_FAIL(SV_ERR_UNSUPPORTED, "sv_rownorm: channels must be even and at most 4096");
  if (n == 0 || channels == 0) return SV_OK;
  if (!x || !out) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_rownorm: null pointer");
  if (bias && !weight) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_rownorm: bias without weight");
  if ((scale || shift) && (!coords || batch < 1))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_rownorm: modulation needs coords and a batch size");
  const size_t align = dtype == SV_FLOAT32 ? 8 : 4;
  const void* ptrs[4] = {x, out, scale, shift};
  for (const void* p : ptrs)
    if (p && reinterpret_cast<uintptr_t>(p) % align != 0)
      SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_rownorm: misaligned feature pointer");
  if (eps < 0.f) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_rownorm: negative eps");
  NormArgs a{n, channels, eps, weight, bias, coords, batch, silu, status};
  cudaStream_t s = to_stream(stream);
  if (dtype == SV_FLOAT32) return launch_norm_typed<float>(x, a, scale, shift, out, s);
  if (dtype == SV_FLOAT16) return launch_norm_typed<__half>(x, a, scale, shift, out, s);
  return launch_norm_typed<__nv_bfloat16>(x, a, scale, shift, out, s);
}
