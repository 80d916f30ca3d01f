// Fused row normalisation of the sparse residual block.
//
// The reference's _SparseResBlock3D (src/mlx_diffuser/models/trellis_slat.py:71-82) runs, around
// its two convolutions,
//     a = silu(LayerNorm32_affine(x))                        (norm1, :77)
//     b = silu(LayerNorm32(h) * (1 + scale[batch]) + shift[batch])   (norm2 + modulation, :79-80)
// as separate element-wise passes. LayerNorm32 (src/mlx_diffuser/layers/trellis.py:16-43) takes
// the mean and the mean squared deviation of each row in fp32, scales by rsqrt(var + eps), applies
// the fp32 affine weight and bias when it has them, and casts back to the feature type. Here one
// kernel does the whole chain per row: the row held in registers by a group of lanes (16-byte
// accesses; several rows per warp for narrow rows), fp32 throughout, one rounding at the end. `scale` / `shift` are the (B, C) embedding projections,
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

// For half-precision outputs: __expf and __fdividef are within a few float32 ulp, far below
// the 2^-9 / 2^-12 rounding step of the stored value, at a fraction of the instructions.
__device__ __forceinline__ float silu_fast(float y) {
  return __fdividef(y, 1.0f + __expf(-y));
}

struct NormArgs {
  int64_t n;
  int channels;
  float eps;
  const float* weight;  // [C] or null
  const float* bias;    // [C] or null
  int64_t mod_stride;   // elements between rows of scale / shift
  const int32_t* coords;
  int64_t batch;
  int silu;
  int32_t* status;
};

// Per-element epilogue shared by both kernels: affine, modulation, activation.
__device__ __forceinline__ float norm_epilogue(float y, int c, const NormArgs& a, float sc,
                                               float sh, bool mod) {
  if (a.weight) y = y * __ldg(&a.weight[c]) + (a.bias ? __ldg(&a.bias[c]) : 0.f);
  if (mod) y = y * (1.0f + sc) + sh;
  return a.silu ? silu(y) : y;
}

__device__ __forceinline__ bool row_batch(const NormArgs& a, int64_t row, bool report_it,
                                          int64_t* b_out) {
  const int32_t b = __ldg(&a.coords[row * 4]);
  if (b < 0 || b >= a.batch) {
    if (report_it) report(a.status, SV_DEVICE_BAD_INDEX);
    return false;
  }
  *b_out = b;
  return true;
}

// Vector kernel: 16-byte accesses. A row is handled by L consecutive lanes (L a power of two
// <= 32, so a warp covers 32 / L rows); lane i of the group holds vectors i + L*j, j < J.
// Needs C % E == 0 (E elements per 16 bytes) and 16-byte aligned rows.
template <typename T, int L, int J>
__global__ void __launch_bounds__(NORM_THREADS)
    rownorm_vec_kernel(const T* x, NormArgs a, const T* __restrict__ scale,
                       const T* __restrict__ shift, T* out) {
  constexpr int E = 16 / sizeof(T);
  constexpr int RPW = 32 / L;  // rows per warp
  const int lane = threadIdx.x & 31;
  const int sub = lane % L;
  const int64_t row =
      ((int64_t)blockIdx.x * (NORM_THREADS / 32) + (threadIdx.x >> 5)) * RPW + lane / L;
  const bool live = row < a.n;
  const int C = a.channels;
  const int nvec = C / E;
  float v[J][E];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int q = sub + L * j;
    if (live && q < nvec) {
      const uint4 raw = *reinterpret_cast<const uint4*>(x + row * C + (int64_t)q * E);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int k = 0; k < E; ++k) {
        v[j][k] = to_f32(e[k]);
        sum += v[j][k];
      }
    }
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / (float)C;
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    if (live && sub + L * j < nvec) {
#pragma unroll
      for (int k = 0; k < E; ++k) {
        const float d = v[j][k] - mean;
        sq += d * d;
      }
    }
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if (!live) return;
  const float rstd = rsqrtf(sq / (float)C + a.eps);
  int64_t b = 0;
  const bool mod = (scale || shift) && row_batch(a, row, sub == 0, &b);
  constexpr bool kFast = sizeof(T) == 2;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int q = sub + L * j;
    if (q < nvec) {
      const int c0 = q * E;
      // y = (v - mean) * (rstd * w) + b: the centring stays exact before the scale (folding
      // the mean into the bias would cancel badly when |mean| >> std)
      float wk[E], bk[E];
#pragma unroll
      for (int k = 0; k < E; k += 4) {
        float4 w4 = make_float4(1.f, 1.f, 1.f, 1.f), b4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.weight) w4 = __ldg(reinterpret_cast<const float4*>(a.weight + c0 + k));
        if (a.bias) b4 = __ldg(reinterpret_cast<const float4*>(a.bias + c0 + k));
        wk[k] = w4.x * rstd; wk[k + 1] = w4.y * rstd; wk[k + 2] = w4.z * rstd;
        wk[k + 3] = w4.w * rstd;
        bk[k] = b4.x; bk[k + 1] = b4.y; bk[k + 2] = b4.z; bk[k + 3] = b4.w;
      }
      T sc[E], sh[E];
      if (mod) {
        if (scale) *reinterpret_cast<uint4*>(sc) =
            __ldg(reinterpret_cast<const uint4*>(scale + b * a.mod_stride + c0));
        if (shift) *reinterpret_cast<uint4*>(sh) =
            __ldg(reinterpret_cast<const uint4*>(shift + b * a.mod_stride + c0));
      }
      uint4 raw;
      T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
      for (int k = 0; k < E; ++k) {
        float y = fmaf(v[j][k] - mean, wk[k], bk[k]);
        if (mod) y = fmaf(y, 1.0f + (scale ? to_f32(sc[k]) : 0.f), shift ? to_f32(sh[k]) : 0.f);
        if (a.silu) y = kFast ? silu_fast(y) : silu(y);
        e[k] = from_f32<T>(y);
      }
      *reinterpret_cast<uint4*>(out + row * C + c0) = raw;
    }
  }
}

// Scalar-pair kernel for rows that are not 16-byte multiples: one warp per row, lane l holds
// channel pairs 2*(l + 32*j), j < MAXJ.
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
  int64_t b = 0;
  const bool mod = (scale || shift) && row_batch(a, row, lane == 0, &b);
  T* orow = out + row * C;
#pragma unroll
  for (int j = 0; j < MAXJ; ++j) {
    const int c = 2 * (lane + 32 * j);
    if (c < C) {
      float s0 = 0.f, s1 = 0.f, h0 = 0.f, h1 = 0.f;
      if (mod && scale) {
        const typename P::V s = P::load(scale + b * a.mod_stride + c);
        s0 = P::lo(s);
        s1 = P::hi(s);
      }
      if (mod && shift) {
        const typename P::V s = P::load(shift + b * a.mod_stride + c);
        h0 = P::lo(s);
        h1 = P::hi(s);
      }
      P::store(orow + c,
               norm_epilogue((v[2 * j] - mean) * rstd, c, a, s0, h0, mod),
               norm_epilogue((v[2 * j + 1] - mean) * rstd, c + 1, a, s1, h1, mod));
    }
  }
}

template <typename T, int MAXJ>
void launch_pairs(const void* x, const NormArgs& a, const void* scale, const void* shift,
                  void* out, cudaStream_t s) {
  const unsigned blocks = (unsigned)((a.n + NORM_ROWS - 1) / NORM_ROWS);
  rownorm_kernel<T, MAXJ><<<blocks, NORM_THREADS, 0, s>>>(
      static_cast<const T*>(x), a, static_cast<const T*>(scale), static_cast<const T*>(shift),
      static_cast<T*>(out));
}

template <typename T, int L, int J>
void launch_vec(const void* x, const NormArgs& a, const void* scale, const void* shift,
                void* out, cudaStream_t s) {
  constexpr int rows_per_block = (NORM_THREADS / 32) * (32 / L);
  const unsigned blocks = (unsigned)((a.n + rows_per_block - 1) / rows_per_block);
  rownorm_vec_kernel<T, L, J><<<blocks, NORM_THREADS, 0, s>>>(
      static_cast<const T*>(x), a, static_cast<const T*>(scale), static_cast<const T*>(shift),
      static_cast<T*>(out));
}

template <typename T>
int launch_norm_typed(const void* x, const NormArgs& a, const void* scale, const void* shift,
                      void* out, cudaStream_t s) {
  constexpr int E = 16 / sizeof(T);
  const int c = a.channels;
  // the vector variants cover rows of up to 32 lanes x 16 vectors of E elements
  const bool vec = c % E == 0 && c / E <= 512 && aligned16(x) && aligned16(out) &&
                   (!a.weight || aligned16(a.weight)) && (!a.bias || aligned16(a.bias)) &&
                   (!scale || aligned16(scale)) && (!shift || aligned16(shift)) &&
                   (a.mod_stride % E == 0);
  if (vec) {
    const int nvec = c / E;
    if (nvec <= 1) launch_vec<T, 1, 1>(x, a, scale, shift, out, s);
    else if (nvec <= 2) launch_vec<T, 2, 1>(x, a, scale, shift, out, s);
    else if (nvec <= 4) launch_vec<T, 4, 1>(x, a, scale, shift, out, s);
    else if (nvec <= 8) launch_vec<T, 8, 1>(x, a, scale, shift, out, s);
    else if (nvec <= 16) launch_vec<T, 16, 1>(x, a, scale, shift, out, s);
    else if (nvec <= 32) launch_vec<T, 32, 1>(x, a, scale, shift, out, s);
    else if (nvec <= 64) launch_vec<T, 32, 2>(x, a, scale, shift, out, s);
    else if (nvec <= 128) launch_vec<T, 32, 4>(x, a, scale, shift, out, s);
    else if (nvec <= 256) launch_vec<T, 32, 8>(x, a, scale, shift, out, s);
    else launch_vec<T, 32, 16>(x, a, scale, shift, out, s);  // nvec <= 512
  } else if (c <= 128) launch_pairs<T, 2>(x, a, scale, shift, out, s);
  else if (c <= 256) launch_pairs<T, 4>(x, a, scale, shift, out, s);
  else if (c <= 512) launch_pairs<T, 8>(x, a, scale, shift, out, s);
  else if (c <= 1024) launch_pairs<T, 16>(x, a, scale, shift, out, s);
  else if (c <= 2048) launch_pairs<T, 32>(x, a, scale, shift, out, s);
  else launch_pairs<T, 64>(x, a, scale, shift, out, s);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

}  // namespace
}  // namespace sv

using namespace sv;

extern "C" int sv_rownorm(const void* x, int64_t n, int channels, int dtype, float eps,
                          const float* weight, const float* bias, const void* scale,
                          const void* shift, int64_t mod_stride, const int32_t* coords,
                          int64_t batch, int silu, void* out, int32_t* status,
                          sv_stream_t stream) {
  if (n < 0 || channels < 0) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_rownorm: negative size");
  if (dtype != SV_FLOAT32 && dtype != SV_FLOAT16 && dtype != SV_BFLOAT16)
    SV_FAIL(SV_ERR_BAD_DTYPE, "sv_rownorm: unknown dtype");
  if (channels % 2 != 0 || channels > 4096)
    SV_FAIL(SV_ERR_UNSUPPORTED, "sv_rownorm: channels must be even and at most 4096");
  if (n == 0 || channels == 0) return SV_OK;
  if (!x || !out) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_rownorm: null pointer");
  if (bias && !weight) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_rownorm: bias without weight");
  if ((scale || shift) &&
      (!coords || batch < 1 || (mod_stride != 0 && mod_stride < channels) || mod_stride % 2))
    SV_FAIL(SV_ERR_INVALID_ARGUMENT,
            "sv_rownorm: modulation needs coords, a batch size and an even row stride (0 or "
            ">= channels)");
  const size_t align = dtype == SV_FLOAT32 ? 8 : 4;
  const void* ptrs[4] = {x, out, scale, shift};
  for (const void* p : ptrs)
    if (p && reinterpret_cast<uintptr_t>(p) % align != 0)
      SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_rownorm: misaligned feature pointer");
  if (eps < 0.f) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_rownorm: negative eps");
  NormArgs a{n, channels, eps, weight, bias, mod_stride, coords, batch, silu, status};
  cudaStream_t s = to_stream(stream);
  if (dtype == SV_FLOAT32) return launch_norm_typed<float>(x, a, scale, shift, out, s);
  if (dtype == SV_FLOAT16) return launch_norm_typed<__half>(x, a, scale, shift, out, s);
  return launch_norm_typed<__nv_bfloat16>(x, a, scale, shift, out, s);
}
