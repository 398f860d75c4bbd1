// Depthwise 3D convolution over channels-last tokens, forward / input-gradient / weight-gradient,
// plus the small utility kernels (offset magnitude reduction, float32 -> dtype conversion).
//
// Replaces nn.Conv3d(C, C, k, padding=k//2, groups=C) of the reference's dw_conv
// (infinity/video/attention.py:58-65, 102) and offset_net[0] + GELU (attention.py:70-72, 105).
// Tokens are [B, frames*H*W, C] rows (the layout x already has at attention.py:85), so no
// [B, C, T, H, W] transpose is materialised (the reference does it at :99 and :190).

#include <math.h>

#include "dsa_attn.cuh"
#include "msl_common.cuh"

namespace msl {

namespace {

__device__ __forceinline__ float gelu_erf(float u) { return 0.5f * u * (1.f + erff(u * 0.70710678118654752f)); }

__device__ __forceinline__ float gelu_erf_grad(float u) {
  const float cdf = 0.5f * (1.f + erff(u * 0.70710678118654752f));
  const float pdf = 0.39894228040143268f * expf(-0.5f * u * u);
  return fmaf(u, pdf, cdf);
}

template <typename T, int CV>
struct ChanVec;
template <>
struct ChanVec<float, 1> {
  static __device__ __forceinline__ void load(const float* p, float (&o)[1]) { o[0] = __ldg(p); }
  static __device__ __forceinline__ void store(float* p, const float (&o)[1]) { p[0] = o[0]; }
};
template <>
struct ChanVec<float, 2> {
  static __device__ __forceinline__ void load(const float* p, float (&o)[2]) {
    const float2 v = __ldg(reinterpret_cast<const float2*>(p));
    o[0] = v.x; o[1] = v.y;
  }
  static __device__ __forceinline__ void store(float* p, const float (&o)[2]) {
    *reinterpret_cast<float2*>(p) = make_float2(o[0], o[1]);
  }
};
template <>
struct ChanVec<__nv_bfloat16, 1> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&o)[1]) { o[0] = __bfloat162float(p[0]); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&o)[1]) { p[0] = __float2bfloat16_rn(o[0]); }
};
template <>
struct ChanVec<__nv_bfloat16, 2> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&o)[2]) {
    const uint32_t w = __ldg(reinterpret_cast<const unsigned int*>(p));
    o[0] = bf16_lo(w); o[1] = bf16_hi(w);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&o)[2]) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(o[0], o[1]);
  }
};

}  // namespace

// One thread per (output token, CV channels).  FLIP = transposed convolution (input gradient):
// dx[p] = sum_taps w[tap] * dy[p - (tap - pad)].
template <typename T, typename TY, int CV, bool FLIP>
__global__ void __launch_bounds__(256) dwconv_fwd_kernel(const ConvParams P, const T* __restrict__ x, long long x_ld,
                                                         const float* __restrict__ wt, const float* __restrict__ bias,
                                                         const float* __restrict__ bias2, int epi,
                                                         const TY* __restrict__ aux, long long aux_ld,
                                                         TY* __restrict__ y, long long y_ld) {
  const int ncg = P.C / CV;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long rows_out = static_cast<long long>(P.out_frames) * P.HW;
  const long long total = static_cast<long long>(P.B) * rows_out * ncg;
  if (idx >= total) return;
  const int cg = static_cast<int>(idx % ncg);
  const long long pos = idx / ncg;
  const int c = cg * CV;
  const int b = static_cast<int>(pos / rows_out);
  const long long row = pos - static_cast<long long>(b) * rows_out;
  const int tl = static_cast<int>(row / P.HW);
  const int rem = static_cast<int>(row - static_cast<long long>(tl) * P.HW);
  const int h = rem / P.W, w = rem - (rem / P.W) * P.W;
  const int tg = P.out_frame0 + tl;
  const int pt = P.kt / 2, ph = P.kh / 2, pw = P.kw / 2;
  const long long xb = static_cast<long long>(b) * P.in_frames * P.HW;

  float acc[CV];
#pragma unroll
  for (int e = 0; e < CV; ++e) acc[e] = 0.f;
  for (int it = 0; it < P.kt; ++it) {
    const int ti = FLIP ? tg - it + pt : tg + it - pt;
    if (ti < P.in_frame0 || ti >= P.in_frame0 + P.in_frames) continue;  // zero outside the input frames
    const int til = ti - P.in_frame0;
    for (int ih = 0; ih < P.kh; ++ih) {
      const int hi = FLIP ? h - ih + ph : h + ih - ph;
      if (hi < 0 || hi >= P.H) continue;
      const long long rbase = xb + (static_cast<long long>(til) * P.H + hi) * P.W;
      const float* wrow = wt + static_cast<long long>((it * P.kh + ih) * P.kw) * P.C + c;
      for (int iw = 0; iw < P.kw; ++iw) {
        const int wi = FLIP ? w - iw + pw : w + iw - pw;
        if (wi < 0 || wi >= P.W) continue;
        float xv[CV];
        ChanVec<T, CV>::load(x + (rbase + wi) * x_ld + c, xv);
        const float* wp = wrow + static_cast<long long>(iw) * P.C;
#pragma unroll
        for (int e = 0; e < CV; ++e) acc[e] = fmaf(__ldg(wp + e), xv[e], acc[e]);
      }
    }
  }
  float out[CV];
  const long long orow = static_cast<long long>(b) * rows_out + row;
  float av[CV];
  if (epi == MSL_EPI_GELU_GRAD) ChanVec<TY, CV>::load(aux + orow * aux_ld + c, av);
  if (epi == MSL_EPI_ACCUM) ChanVec<TY, CV>::load(y + orow * y_ld + c, av);  // the buffer's own terms
#pragma unroll
  for (int e = 0; e < CV; ++e) {
    float u = acc[e] + (bias ? __ldg(bias + c + e) : 0.f);
    if (epi == MSL_EPI_GELU)
      u = gelu_erf(u);
    else if (epi == MSL_EPI_GELU_GRAD)
      u = av[e] * gelu_erf_grad(u);
    else if (bias2)
      u += __ldg(bias2 + c + e);
    if (epi == MSL_EPI_ACCUM) u += av[e];
    out[e] = u;
  }
  ChanVec<TY, CV>::store(y + orow * y_ld + c, out);
}

// Weight gradient: block = 32 channel lanes x (blockDim.y) tap groups; each thread owns one
// (channel, tap) accumulator at a time and sums dy * shifted x over the block's token rows.
// The extra tap index K accumulates the bias gradient (sum of dy).
template <typename TDY, typename T>
__global__ void __launch_bounds__(512) dwconv_wgrad_kernel(const ConvParams P, const TDY* __restrict__ dy, long long dy_ld,
                                                           const T* __restrict__ x, long long x_ld, float* dw, float* db,
                                                           int rows_per_block) {
  const int c = blockIdx.x * 32 + threadIdx.x;
  const bool cvalid = c < P.C;
  const int cc = cvalid ? c : 0;
  const int K = P.kt * P.kh * P.kw;
  const int ntap = db ? K + 1 : K;
  const long long total_rows = static_cast<long long>(P.B) * P.out_frames * P.H;
  const long long r0 = static_cast<long long>(blockIdx.y) * rows_per_block;
  const long long r1 = min(total_rows, r0 + rows_per_block);
  const int pt = P.kt / 2, ph = P.kh / 2, pw = P.kw / 2;
  for (int tap = threadIdx.y; tap < ntap; tap += blockDim.y) {
    int it = 0, ih = 0, iw = 0;
    if (tap < K) {
      it = tap / (P.kh * P.kw);
      const int r = tap - it * P.kh * P.kw;
      ih = r / P.kw;
      iw = r - ih * P.kw;
    }
    float acc = 0.f;
    for (long long rr = r0; rr < r1; ++rr) {
      const int b = static_cast<int>(rr / (static_cast<long long>(P.out_frames) * P.H));
      const int rem = static_cast<int>(rr - static_cast<long long>(b) * P.out_frames * P.H);
      const int tl = rem / P.H, h = rem - (rem / P.H) * P.H;
      const TDY* dyrow = dy + ((static_cast<long long>(b) * P.out_frames + tl) * P.H + h) * P.W * dy_ld + cc;
      if (tap == K) {
        for (int w = 0; w < P.W; ++w) acc += to_f32<TDY>(dyrow[w * dy_ld]);
        continue;
      }
      const int ti = P.out_frame0 + tl + it - pt;
      const int hi = h + ih - ph;
      if (ti < P.in_frame0 || ti >= P.in_frame0 + P.in_frames || hi < 0 || hi >= P.H) continue;
      const int til = ti - P.in_frame0;
      const T* xrow = x + ((static_cast<long long>(b) * P.in_frames + til) * P.H + hi) * P.W * x_ld + cc;
      const int wlo = max(0, pw - iw), whi = min(P.W, P.W + pw - iw);
      for (int w = wlo; w < whi; ++w)
        acc = fmaf(to_f32<TDY>(dyrow[static_cast<long long>(w) * dy_ld]),
                   to_f32<T>(xrow[static_cast<long long>(w + iw - pw) * x_ld]), acc);
    }
    if (cvalid) {
      if (tap < K)
        atomicAdd(dw + static_cast<long long>(tap) * P.C + c, acc);
      else
        atomicAdd(db + c, acc);
    }
  }
}

template <typename T, typename TY>
static cudaError_t dwconv_fwd_t(const ConvParams& P, const void* x, long long x_ld, const float* wt,
                                const float* bias, const float* bias2, int epi, const void* aux,
                                long long aux_ld, void* y, long long y_ld, bool flip, bool vec2,
                                cudaStream_t s) {
  const int cv = vec2 ? 2 : 1;
  const long long total = static_cast<long long>(P.B) * P.out_frames * P.HW * (P.C / cv);
  const dim3 grid(static_cast<unsigned>((total + 255) / 256)), block(256);
  const T* xp = static_cast<const T*>(x);
  const TY* ap = static_cast<const TY*>(aux);
  TY* yp = static_cast<TY*>(y);
  if (vec2) {
    if (flip)
      dwconv_fwd_kernel<T, TY, 2, true><<<grid, block, 0, s>>>(P, xp, x_ld, wt, bias, bias2, epi, ap, aux_ld, yp, y_ld);
    else
      dwconv_fwd_kernel<T, TY, 2, false><<<grid, block, 0, s>>>(P, xp, x_ld, wt, bias, bias2, epi, ap, aux_ld, yp, y_ld);
  } else {
    if (flip)
      dwconv_fwd_kernel<T, TY, 1, true><<<grid, block, 0, s>>>(P, xp, x_ld, wt, bias, bias2, epi, ap, aux_ld, yp, y_ld);
    else
      dwconv_fwd_kernel<T, TY, 1, false><<<grid, block, 0, s>>>(P, xp, x_ld, wt, bias, bias2, epi, ap, aux_ld, yp, y_ld);
  }
  return cudaGetLastError();
}

cudaError_t launch_dwconv_fwd(const ConvParams& P, const void* x, long long x_ld, const float* wt,
                              const float* bias, const float* bias2, int epi, const void* aux,
                              long long aux_ld, void* y, long long y_ld, int y_dtype, bool flip, cudaStream_t s) {
  const cudaError_t te = launch_dwconv_fwd_tiled(P, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, y_dtype, flip, s);
  if (te != cudaErrorNotSupported) return te;
  const size_t es = P.dtype == MSL_DTYPE_BF16 ? 2 : 4;
  const size_t ys = y_dtype == MSL_DTYPE_BF16 ? 2 : 4;
  const bool vec2 = (P.C % 2 == 0) && (x_ld % 2 == 0) && (y_ld % 2 == 0) &&
                    (epi != MSL_EPI_GELU_GRAD || aux_ld % 2 == 0) &&
                    (reinterpret_cast<uintptr_t>(x) % (2 * es) == 0) && (reinterpret_cast<uintptr_t>(y) % (2 * ys) == 0) &&
                    (epi != MSL_EPI_GELU_GRAD || reinterpret_cast<uintptr_t>(aux) % (2 * ys) == 0);
  if (P.dtype == MSL_DTYPE_BF16) {
    if (y_dtype == MSL_DTYPE_BF16)
      return dwconv_fwd_t<__nv_bfloat16, __nv_bfloat16>(P, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, flip, vec2, s);
    return dwconv_fwd_t<__nv_bfloat16, float>(P, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, flip, vec2, s);
  }
  if (y_dtype == MSL_DTYPE_BF16)
    return dwconv_fwd_t<float, __nv_bfloat16>(P, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, flip, vec2, s);
  return dwconv_fwd_t<float, float>(P, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, flip, vec2, s);
}

template <typename TDY, typename T>
static void wgrad_t(const ConvParams& P, dim3 grid, dim3 block, const void* dy, long long dy_ld, const void* x,
                    long long x_ld, float* dw, float* db, int rows_per_block, cudaStream_t s) {
  dwconv_wgrad_kernel<TDY, T><<<grid, block, 0, s>>>(P, static_cast<const TDY*>(dy), dy_ld, static_cast<const T*>(x),
                                                      x_ld, dw, db, rows_per_block);
}

cudaError_t launch_dwconv_wgrad(const ConvParams& P, const void* dy, long long dy_ld, int dy_dtype, const void* x,
                                long long x_ld, float* dw, float* db, cudaStream_t s) {
  const cudaError_t te = launch_dwconv_wgrad_tiled(P, dy, dy_ld, dy_dtype, x, x_ld, dw, db, s);
  if (te != cudaErrorNotSupported) return te;
  const long long total_rows = static_cast<long long>(P.B) * P.out_frames * P.H;
  const int rows_per_block = max(1, 2048 / max(1, P.W));
  const dim3 grid(static_cast<unsigned>((P.C + 31) / 32),
                  static_cast<unsigned>((total_rows + rows_per_block - 1) / rows_per_block));
  const dim3 block(32, 16);
  const bool xb = P.dtype == MSL_DTYPE_BF16, yb = dy_dtype == MSL_DTYPE_BF16;
  if (yb && xb) wgrad_t<__nv_bfloat16, __nv_bfloat16>(P, grid, block, dy, dy_ld, x, x_ld, dw, db, rows_per_block, s);
  else if (yb) wgrad_t<__nv_bfloat16, float>(P, grid, block, dy, dy_ld, x, x_ld, dw, db, rows_per_block, s);
  else if (xb) wgrad_t<float, __nv_bfloat16>(P, grid, block, dy, dy_ld, x, x_ld, dw, db, rows_per_block, s);
  else wgrad_t<float, float>(P, grid, block, dy, dy_ld, x, x_ld, dw, db, rows_per_block, s);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ utilities
// Per-axis max |(offset + bias) * oscale|.  Blocks stride over rows; in a row the threads stride over
// column quads (16-byte loads when every row start is 16-byte aligned).  Column 4i + e has axis
// (4i + e) mod 3 = (i + e) mod 3.
template <bool VEC>
__global__ void __launch_bounds__(256) offsets_absmax_kernel(const float* __restrict__ off, long long rows, long long ld,
                                                             const float* __restrict__ bias, int ncol, float oscale,
                                                             float* out3) {
  float m[3] = {0.f, 0.f, 0.f};
  const int nq = VEC ? ncol / 4 : 0;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* row = off + r * ld;
    if (VEC) {
      for (int i = threadIdx.x; i < nq; i += blockDim.x) {
        float4 v = __ldcs(reinterpret_cast<const float4*>(row) + i);
        if (bias) {
          const float4 b = __ldg(reinterpret_cast<const float4*>(bias) + i);
          v.x = __fadd_rn(v.x, b.x); v.y = __fadd_rn(v.y, b.y); v.z = __fadd_rn(v.z, b.z); v.w = __fadd_rn(v.w, b.w);
        }
        const int a = i % 3;
        const float e0 = fabsf(v.x * oscale), e1 = fabsf(v.y * oscale), e2 = fabsf(v.z * oscale),
                    e3 = fabsf(v.w * oscale);
        // axes of the four elements: a, a+1, a+2, a (mod 3)
        if (a == 0) { m[0] = fmaxf(m[0], fmaxf(e0, e3)); m[1] = fmaxf(m[1], e1); m[2] = fmaxf(m[2], e2); }
        else if (a == 1) { m[1] = fmaxf(m[1], fmaxf(e0, e3)); m[2] = fmaxf(m[2], e1); m[0] = fmaxf(m[0], e2); }
        else { m[2] = fmaxf(m[2], fmaxf(e0, e3)); m[0] = fmaxf(m[0], e1); m[1] = fmaxf(m[1], e2); }
      }
    }
    for (int c = 4 * nq + threadIdx.x; c < ncol; c += blockDim.x) {  // tail columns, or every column
      const float o = bias ? __fadd_rn(row[c], __ldg(bias + c)) : row[c];
      const int a = c % 3;
      m[a] = fmaxf(m[a], fabsf(o * oscale));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m[0] = fmaxf(m[0], __shfl_xor_sync(kFull, m[0], o));
    m[1] = fmaxf(m[1], __shfl_xor_sync(kFull, m[1], o));
    m[2] = fmaxf(m[2], __shfl_xor_sync(kFull, m[2], o));
  }
  __shared__ float red[3][8];
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    red[0][warp] = m[0];
    red[1][warp] = m[1];
    red[2][warp] = m[2];
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    float v = 0.f;
    for (int w = 0; w < (blockDim.x >> 5); ++w) v = fmaxf(v, red[threadIdx.x][w]);
    // non-negative floats order like their bit patterns
    atomicMax(reinterpret_cast<int*>(out3) + threadIdx.x, __float_as_int(v));
  }
}

cudaError_t launch_offsets_absmax(const float* off, long long rows, long long ld, const float* bias, int heads, int taps,
                                  float oscale, float* out3, cudaStream_t s) {
  const int ncol = heads * taps * 3;
  long long blocks = rows < 148LL * 8 ? rows : 148LL * 8;
  if (blocks < 1) blocks = 1;
  const bool vec = (reinterpret_cast<uintptr_t>(off) & 15u) == 0 && (ld & 3) == 0 && ncol >= 4 &&
                   (!bias || (reinterpret_cast<uintptr_t>(bias) & 15u) == 0);
  if (vec)
    offsets_absmax_kernel<true><<<static_cast<unsigned>(blocks), 256, 0, s>>>(off, rows, ld, bias, ncol, oscale, out3);
  else
    offsets_absmax_kernel<false><<<static_cast<unsigned>(blocks), 256, 0, s>>>(off, rows, ld, bias, ncol, oscale, out3);
  return cudaGetLastError();
}

template <typename T>
__global__ void __launch_bounds__(256) convert_f32_kernel(const float* __restrict__ src, long long src_ld, T* __restrict__ dst,
                                                          long long dst_ld, long long rows, long long cols) {
  const long long n = rows * cols;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / cols, c = i - (i / cols) * cols;
    dst[r * dst_ld + c] = from_f32<T>(src[r * src_ld + c]);
  }
}

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 8 elements per thread (two 16-byte loads, one 16-byte bf16 or two float32 stores); n = rows * cols / 8
// vectors, below 2^31
template <typename T>
__global__ void __launch_bounds__(256) convert_f32_vec8_kernel(const float* __restrict__ src, long long src_ld,
                                                               T* __restrict__ dst, long long dst_ld, unsigned cv,
                                                               unsigned n) {
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned r = i / cv, c = (i - r * cv) * 8u;
    const float4* s4 = reinterpret_cast<const float4*>(src + static_cast<long long>(r) * src_ld + c);
    const float4 a = __ldg(s4), b = __ldg(s4 + 1);
    T* d = dst + static_cast<long long>(r) * dst_ld + c;
    if constexpr (sizeof(T) == 2) {
      uint4 o;
      o.x = bf16x2_bits(a.x, a.y);
      o.y = bf16x2_bits(a.z, a.w);
      o.z = bf16x2_bits(b.x, b.y);
      o.w = bf16x2_bits(b.z, b.w);
      *reinterpret_cast<uint4*>(d) = o;
    } else {
      reinterpret_cast<float4*>(d)[0] = a;
      reinterpret_cast<float4*>(d)[1] = b;
    }
  }
}

cudaError_t launch_convert_f32(const float* src, long long src_ld, void* dst, long long dst_ld, int dtype,
                               long long rows, long long cols, cudaStream_t s) {
  const long long n = rows * cols;
  const long long es = dtype == MSL_DTYPE_BF16 ? 2 : 4;
  if (cols % 8 == 0 && n / 8 < (1LL << 31) && (reinterpret_cast<uintptr_t>(src) & 15u) == 0 && src_ld % 4 == 0 &&
      (reinterpret_cast<uintptr_t>(dst) & 15u) == 0 && (dst_ld * es) % 16 == 0) {
    const unsigned nv = static_cast<unsigned>(n / 8), cv = static_cast<unsigned>(cols / 8);
    long long vblocks = (nv + 255) / 256;
    if (vblocks > 148LL * 16) vblocks = 148LL * 16;
    if (vblocks < 1) vblocks = 1;
    if (dtype == MSL_DTYPE_BF16)
      convert_f32_vec8_kernel<__nv_bfloat16><<<static_cast<unsigned>(vblocks), 256, 0, s>>>(
          src, src_ld, static_cast<__nv_bfloat16*>(dst), dst_ld, cv, nv);
    else
      convert_f32_vec8_kernel<float><<<static_cast<unsigned>(vblocks), 256, 0, s>>>(src, src_ld, static_cast<float*>(dst),
                                                                                  dst_ld, cv, nv);
    return cudaGetLastError();
  }
  long long blocks = (n + 255) / 256;
  if (blocks > 148LL * 32) blocks = 148LL * 32;
  if (blocks < 1) blocks = 1;
  if (dtype == MSL_DTYPE_BF16)
    convert_f32_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        src, src_ld, static_cast<__nv_bfloat16*>(dst), dst_ld, rows, cols);
  else
    convert_f32_kernel<float><<<static_cast<unsigned>(blocks), 256, 0, s>>>(src, src_ld, static_cast<float*>(dst),
                                                                            dst_ld, rows, cols);
  return cudaGetLastError();
}

}  // namespace msl
